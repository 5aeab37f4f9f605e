// The cross-rank steps of the tensor-parallel decoder over peer memory (NVLink),
// in place of NCCL's all-reduce of the O / down partial sums and all-gather of the
// argmax pairs (iron_b200/tp.py).
//
// Every rank allocates one symmetric buffer (the same size on every rank, each rank
// holding the others' base addresses): data [2 slots][world][cap] 32-bit words, then
// flags [2 slots][world][chunks] 32-bit words.  A call pushes: CTA c copies words
// [c*CHUNK, (c+1)*CHUNK) of the rank's input with plain stores into slot s of every
// rank's buffer (its own row `rank`), fences at system scope and stores the epoch
// into flag [s][rank][c] of every rank.  It then waits (bounded) until the flags
// [s][r][c] of its own buffer carry the epoch for every r, and reads the rows from
// its own memory: a sum in rank order (float32, deterministic) or a gather.  The
// epoch is a per-CTA counter in the caller's device memory, incremented by the call,
// so a captured CUDA graph replays correctly; the slot is its parity.  Slot s is
// written again two calls later, when every rank has passed the wait of the call in
// between, which it can only do after finishing its reads of slot s: no rank
// overwrites words another is still reading.
//
// A wait that times out stores 1 in the caller's error word and leaves its outputs
// unwritten; the decoder reads the word with the step's tokens.  No multicast, no
// TMA: plain loads and stores.
#include "common.cuh"

namespace iron {

constexpr int PEER_THREADS = 512;
constexpr int PEER_CHUNK = 4096;  // 32-bit words per CTA
constexpr unsigned long long PEER_TIMEOUT_NS = 200ull * 1000 * 1000;

struct PeerArgs {
  const unsigned long long* peers;  // [world] base address of every rank's buffer
  int world, rank, cap, nchunk, n, mode;
  const uint32_t* in;
  uint32_t* out;
  uint32_t* epochs;  // [nchunk] this rank's call counters
  int* err;
};

__device__ __forceinline__ unsigned long long ptimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(PEER_THREADS) peer_exchange_kernel(PeerArgs a) {
  const int c = blockIdx.x, t = threadIdx.x;
  __shared__ int s_ok;
  const uint32_t e = a.epochs[c] + 1u;
  const int slot = (int)(e & 1u);
  const int i0 = c * PEER_CHUNK, i1 = min(a.n, i0 + PEER_CHUNK);
  const size_t flags0 = (size_t)2 * a.world * a.cap;  // words before the flags
  // 1. push this chunk into row `rank` of slot `slot` of every rank's buffer
  for (int r = 0; r < a.world; ++r) {
    uint32_t* dst = (uint32_t*)a.peers[r] + ((size_t)slot * a.world + a.rank) * a.cap;
    for (int i = i0 + t; i < i1; i += PEER_THREADS) dst[i] = a.in[i];
  }
  if (t == 0) s_ok = 1;
  __syncthreads();
  // 2. publish: the CTA's stores before the flags, at system scope
  if (t < a.world) {
    __threadfence_system();
    uint32_t* f = (uint32_t*)a.peers[t] + flags0 + ((size_t)slot * a.world + a.rank) * a.nchunk + c;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
  }
  // 3. wait (bounded) for every rank's chunk of this call in this rank's buffer
  if (t < a.world) {
    const uint32_t* f = (const uint32_t*)a.peers[a.rank] + flags0 + ((size_t)slot * a.world + t) * a.nchunk + c;
    const unsigned long long t0 = ptimer();
    for (unsigned it = 0;; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v == e) break;
      if ((it & 63) == 63 && ptimer() - t0 > PEER_TIMEOUT_NS) {
        atomicExch(a.err, 1);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    // 4. the rows of slot `slot` in this rank's own memory
    const uint32_t* base = (const uint32_t*)a.peers[a.rank] + (size_t)slot * a.world * a.cap;
    if (a.mode == 0) {
      for (int i = i0 + t; i < i1; i += PEER_THREADS) {
        float s = 0.f;
        for (int r = 0; r < a.world; ++r) s += __uint_as_float(__ldcg(base + (size_t)r * a.cap + i));
        a.out[i] = __float_as_uint(s);
      }
    } else {
      for (int r = 0; r < a.world; ++r)
        for (int i = i0 + t; i < i1; i += PEER_THREADS) a.out[(size_t)r * a.n + i] = __ldcg(base + (size_t)r * a.cap + i);
    }
  }
  __syncthreads();
  if (t == 0) a.epochs[c] = e;
}

static int peer_chunks(int cap) { return cap < 1 ? 1 : (cap + PEER_CHUNK - 1) / PEER_CHUNK; }

}  // namespace iron

using namespace iron;

extern "C" int64_t iron_peer_buffer_bytes(int world, int cap_words) {
  if (world < 1 || cap_words < 1) return 0;
  const int64_t words = (int64_t)2 * world * cap_words + (int64_t)2 * world * peer_chunks(cap_words);
  return (words * 4 + 255) & ~(int64_t)255;
}

extern "C" int iron_peer_epoch_words(int cap_words) { return peer_chunks(cap_words); }

extern "C" int iron_peer_exchange(const unsigned long long* peers_dev, int world, int rank, int cap_words,
                                  const void* in, void* out, int n_words, int mode, uint32_t* epochs_dev,
                                  int* err_dev, void* stream) {
  IRON_REQUIRE(peers_dev && in && out && epochs_dev && err_dev, IRON_ERR_ARG, "peer_exchange: null pointer");
  IRON_REQUIRE(world >= 1 && rank >= 0 && rank < world, IRON_ERR_ARG, "peer_exchange: rank %d of %d", rank, world);
  IRON_REQUIRE(n_words >= 1 && n_words <= cap_words, IRON_ERR_ARG, "peer_exchange: %d words, capacity %d", n_words,
               cap_words);
  IRON_REQUIRE(mode == 0 || mode == 1, IRON_ERR_ARG, "peer_exchange: mode %d (0 sum, 1 gather)", mode);
  PeerArgs a;
  a.peers = peers_dev;
  a.world = world;
  a.rank = rank;
  a.cap = cap_words;
  a.nchunk = peer_chunks(cap_words);
  a.n = n_words;
  a.mode = mode;
  a.in = (const uint32_t*)in;
  a.out = (uint32_t*)out;
  a.epochs = epochs_dev;
  a.err = err_dev;
  // every CTA of the capacity runs (the flags and epochs are per chunk of the capacity);
  // chunks past n_words only exchange their flags
  peer_exchange_kernel<<<a.nchunk, PEER_THREADS, 0, (cudaStream_t)stream>>>(a);
  return iron_check_launch("peer_exchange_kernel");
}
