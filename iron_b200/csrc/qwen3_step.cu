// One greedy Qwen3 decode token (batch 1) as ONE persistent cooperative kernel.
//
// Why one kernel.  At batch 1 a Qwen3-0.6B token streams ~0.9 GB (weights, K/V),
// but a single projection is only a few microseconds of HBM time: the token is
// bound by the latency of the dependency chain between projections.  Weights and
// cached K/V do not depend on activations, so a producer warp per CTA streams them
// into a shared-memory ring (CTA-local cp.async.bulk) about a layer ahead, and the
// compute warps only ever wait for activations.
//
// Hand-offs.  Activations move between CTAs as flagged 64-bit words: the payload
// and the (token, layer) epoch in one store, so a reader that sees the epoch it
// waits for also has the data.  There is no grid barrier, no fence on the hand-off
// path and no floating-point atomic: every sum is formed in a fixed order, and two
// runs from the same state give the same bits.  Per layer (CTAs form Hkv KV-head
// groups of N / Hkv CTAs):
//
//   x  --(all CTAs)-->  RMSNorm + QKV rows of KV head h (group h's CTAs, 16-row tiles)
//   q/k/v words  -->   every CTA of group h: q/k RMSNorm + RoPE, one split of head h's
//                      positions (flash decoding); the split's (m, l, o) as words
//   split words  -->   the group's first CTA merges the splits: the bf16 heads as words
//   merged heads -->   the CTAs holding O row tiles: x1 = x + Wo attn, rows as words
//   x1 words     -->   every CTA: RMSNorm, its
//                      gate/up tiles (8 gate rows over the matching 8 up rows), SiLU * up:
//                      h values as words
//   h words      -->   every CTA: its slices of the down projection (a 16-row tile cut
//                      into DSL pieces along K) as partial-sum words
//   down partials -->  every CTA: x_next = x1 + sum over the slices (fixed order)
//
// Projections.  Weight tiles of 16 rows are pre-packed in the A-fragment order of
// mma.sync m16n8k32 (s8): a lane loads its fragment of a 32-column block with one
// conflict-free 16-byte shared load.  Activations are staged as exact 31-bit block
// floating point, four balanced signed bytes per value (the B fragment: digit d of
// value k in column d), so one MMA gives exact integer sums of 16 rows x 32 columns;
// the sums are scaled by weight scale x activation scale in float64 (exact) and
// accumulated in float64.  The warps split a tile's k-blocks into slices whose sums
// are added in slice order.  One bf16 rounding per output, as the per-operator
// kernels (iron_gemv_w8a16) do.
//
// Every wait is bounded by %globaltimer: on timeout a CTA records an error code in
// the sync words and leaves; the other CTAs see it in their own waits and leave too.
// In-flight bulk copies are drained (bounded) before a CTA exits.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace iron {
namespace qstep {

// 8 compute warps and one producer warp
constexpr int NT = 256, NWARP = NT / 32;
constexpr int HDIM = 128;         // head_dim of the step kernel
constexpr int TR = 16;            // rows per weight tile (the MMA's M)
constexpr int NMB = 16;           // ring slots (chunks in flight at most)
constexpr int GMAX = 24;          // most CTAs in one KV-head group (attention splits)
constexpr int KVP = 64;           // cached positions per K/V chunk (32 KB)
constexpr int NTMAX = 16;         // most tiles of one projection in one CTA
constexpr int LMT = 4;            // int8 lm_head tiles per chunk
constexpr int DSL = 4;            // K slices of a down-projection tile
constexpr int XBS = 288;          // bytes of one 32-column block of B fragments (padded)
constexpr int PIECE = 32768;      // bytes per cp.async.bulk instruction
constexpr int SMEM_MAX = 227 * 1024;
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;  // per wait

enum { SYNC_ERR = 1, SYNC_ARGMAX = 2, SYNC_EPOCH = 3, SYNC_WORDS = 8 };
enum { ERR_WAIT = 1, ERR_COPY = 2, ERR_INPUT = 3 };

struct Kp {
  iron_qwen3_model m;
  int embed_input, advance;
  int ring;     // ring bytes
  int lm_rows;  // bf16 lm_head rows per chunk
  int kmax;     // longest staged activation (max of D, Hq*HD, FF)
  int hbn;      // bf16 values of the polled-vector buffer
};

__host__ __device__ inline int rowb(int K, int G) { return K + 2 * (K / G); }
// bytes of one packed tile of 16 rows x K
__host__ __device__ inline size_t tileb(int K, int G) { return (size_t)TR * rowb(K, G); }

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier, bulk copies, flagged words, timer
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(sa(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   sa(dst)),
               "l"(src), "r"(bytes), "r"(sa(b))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const int32_t* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const int32_t* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// D = A (16x32 s8, row) * B (32x8 s8, col), exact int32
__device__ __forceinline__ void mma_s8(int (&c)[4], const uint4& a, uint2 b) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(0));
}

// Flagged words.  Two forms: (epoch << 32 | 32-bit payload) for bf16 pairs and
// float32 values, and (16-bit tag << 48 | the top 48 bits of a float64) for the O
// partial sums (sign, exponent and 36 significand bits: 2^-37 relative, far below
// the bf16 rounding that follows).  Each word is written once per (token, layer)
// with a value that differs from its previous one; zero is never a valid tag.
__device__ __forceinline__ void ll_put(unsigned long long* p, uint32_t data, uint32_t epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | data;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ll_put_d(unsigned long long* p, double v, uint32_t tag16) {
  const unsigned long long w =
      ((unsigned long long)tag16 << 48) | ((unsigned long long)__double_as_longlong(v) >> 16);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ double ll_val_d(unsigned long long w) {
  return __longlong_as_double((long long)(w << 16));
}
__device__ __forceinline__ unsigned long long ll_ld(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ uint32_t tag16_of(uint32_t epoch) { return epoch % 65535u + 1u; }

// Wait (bounded) until the U words addr(0..U-1) whose bit is set in `want` carry the
// tag (their bits from `tshift` up equal `tag`).  v[u] holds word u's last load (the
// caller issues the first loads together); each round reloads every word still
// pending at once, so a round costs one memory round trip however many words lag.
// False when the wait gave up (timeout, or the grid's error word is set).
template <int U, class Addr>
__device__ __forceinline__ bool poll_rounds(Addr addr, unsigned long long (&v)[U], uint32_t want, uint32_t tag,
                                            int tshift, int32_t* sync) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
    uint32_t pending = 0;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (((want >> u) & 1u) && (uint32_t)(v[u] >> tshift) != tag) pending |= 1u << u;
    if (!pending) return true;
    if (it == 0) {
      t0 = gtimer();
    } else if ((it & 7) == 0) {
      if (ld_relaxed(&sync[SYNC_ERR]) != 0) return false;
      if (gtimer() - t0 > TIMEOUT_NS) {
        atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_WAIT);
        return false;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if ((pending >> u) & 1u) v[u] = ll_ld(addr(u));
  }
}

// Wait (bounded) until every word w[i], i = threadIdx.x + j * NT < n, carries the tag;
// then f(i, word) for each, in increasing i.  The U words of a thread are loaded and
// reloaded together (U <= 32).
template <int U, class F>
__device__ __forceinline__ bool poll(const unsigned long long* w, int n, uint32_t tag, int tshift, int32_t* sync,
                                     F f) {
  for (int base = 0; base < n; base += U * NT) {
    unsigned long long v[U];
    uint32_t want = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * NT + threadIdx.x;
      v[u] = i < n ? ll_ld(w + i) : 0ull;
      if (i < n) want |= 1u << u;
    }
    const unsigned long long* wb = w + base + threadIdx.x;
    if (!poll_rounds<U>([&](int u) { return wb + u * NT; }, v, want, tag, tshift, sync)) return false;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if ((want >> u) & 1u) f(base + u * NT + threadIdx.x, v[u]);
  }
  return true;
}

// Phase timestamps for profiling builds (-DIRON_STEP_PROFILE): thread 0 of each CTA
// stores %globaltimer at the marked points into a buffer registered with
// iron_qwen3_step_profile_buffer ([CTA][64 layer rows][32 marks] u64).  Compiled
// out otherwise.
#ifdef IRON_STEP_PROFILE
__device__ unsigned long long* g_step_prof;
#define STEP_MARK(row, k)                                                                                      \
  do {                                                                                                         \
    if (threadIdx.x == 0 && g_step_prof) g_step_prof[((size_t)blockIdx.x * 64 + (row)) * 32 + (k)] = gtimer(); \
  } while (0)
#else
#define STEP_MARK(row, k) \
  do {                    \
  } while (0)
#endif

// barrier of the NT compute threads only (the producer warp runs on its own)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

// barrier of the compute threads that also returns whether any of them passed true
__device__ __forceinline__ bool cvote_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NT)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ double csum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum_d(v);
  csync();
  if (lane == 0) red[wid] = v;
  csync();
  double t = lane < NWARP ? red[lane] : 0.0;
  return warp_sum_d(t);
}

// ---------------------------------------------------------------------------
// work partition of one CTA (identical in all its threads)
// ---------------------------------------------------------------------------
__host__ __device__ inline void part(int M, int c, int N, int& lo, int& hi) {
  lo = (int)((long long)M * c / N);
  hi = (int)((long long)M * (c + 1) / N);
}

// KV-head group of CTA c: CTAs [h*N/Hkv, (h+1)*N/Hkv)
__host__ __device__ inline void head_group(int c, int N, int Hkv, int& h, int& c0, int& c1) {
  h = 0;
  while (h + 1 < Hkv && (int)((long long)(h + 1) * N / Hkv) <= c) ++h;
  c0 = (int)((long long)h * N / Hkv);
  c1 = (int)((long long)(h + 1) * N / Hkv);
}

struct Plan {
  int h, gi, gsz;       // KV-head group, index in the group, group size
  int qt0, qnt;         // QKV tiles of group h (q rows of its heads, then k, then v)
  int ot0, ont;         // O row tiles (all Hq * HD columns)
  int gt0, gnt;         // gate/up tiles (8 gate rows over the matching 8 up rows)
  int ds0, dns;         // down slices (tile ds / DSL, K slice ds % DSL)
  int kst, ken, own;    // cached K/V positions [kst, ken) of this split; it holds pos
  int nkv, cpl;         // K/V chunks per layer; chunks per layer (4 + nkv)
  int hlo, hhi, hnch;   // lm_head rows (bf16) or tiles (int8), chunks
  int total;            // chunks of the token
};

// Tiles per CTA: QKV within the KV-head group; O row tiles, gate/up tiles and down
// slices (a 16-row tile cut into DSL pieces along K) over all CTAs.
__host__ __device__ inline void plan_tiles(const iron_qwen3_model& m, int c, int N, Plan& P) {
  const int GQ = m.Hq / m.Hkv;
  int c0, c1;
  head_group(c, N, m.Hkv, P.h, c0, c1);
  P.gi = c - c0;
  P.gsz = c1 - c0;
  int lo, hi;
  part((GQ + 2) * HDIM / TR, P.gi, P.gsz, lo, hi);
  P.qt0 = lo;
  P.qnt = hi - lo;
  part(m.D / TR, c, N, lo, hi);
  P.ot0 = lo;
  P.ont = hi - lo;
  part(m.FF / 8, c, N, lo, hi);
  P.gt0 = lo;
  P.gnt = hi - lo;
  part(m.D / TR * DSL, c, N, lo, hi);
  P.ds0 = lo;
  P.dns = hi - lo;
}

__device__ Plan make_plan(const Kp& p, int pos) {
  const iron_qwen3_model& m = p.m;
  Plan P;
  const int N = gridDim.x, c = blockIdx.x;
  plan_tiles(m, c, N, P);
  const int L = pos + 1, chunk = (L + P.gsz - 1) / P.gsz;
  const int st = min(L, P.gi * chunk), en = min(L, st + chunk);
  P.own = pos >= st && pos < en;
  P.kst = st;
  P.ken = max(st, min(en, pos));
  P.nkv = (P.ken - P.kst + KVP - 1) / KVP;
  P.cpl = 4 + P.nkv;
  if (m.lm_w8) {
    part((m.V + TR - 1) / TR, c, N, P.hlo, P.hhi);
    P.hnch = (P.hhi - P.hlo + LMT - 1) / LMT;
  } else {
    part(m.V, c, N, P.hlo, P.hhi);
    P.hnch = (P.hhi - P.hlo + p.lm_rows - 1) / p.lm_rows;
  }
  P.total = P.cpl * m.n_layers + P.hnch;
  return P;
}

// ---------------------------------------------------------------------------
// shared memory
// ---------------------------------------------------------------------------
struct RingState {                // shared by the producer lane and compute thread 0
  unsigned long long tail;        // bytes released by the compute threads (monotonic)
  int issued, consumed, abort;    // chunks issued / released; compute threads left early
  uint32_t slot[NMB];             // ring offset of the chunk in each slot
  unsigned long long end[NMB];    // allocation offset after the chunk
};

struct Smem {
  uint8_t* ring;
  uint8_t* xb;     // [kmax / 32][XBS] B fragments of the staged activation
  int* xse;        // [kmax / G] activation group scale exponents: scale 2^xse (the 2^-15 included)
  double* part;    // [NTMAX][TR] slice sums of a projection
  uint16_t* sx;    // [D] residual x (bf16 bits)
  uint16_t* sx1;   // [D] residual x1
  uint16_t* nw;    // [D] weights of the next RMSNorm
  uint16_t* hb;    // [hbn] polled bf16 vectors (q/k/v rows, merged heads, h)
  uint16_t* outb;  // [NTMAX * TR] bf16 outputs of a projection before they are published
  float* att;      // q [GQ][HD], k [HD], v [HD], warp partials [NWARP][GQ][HD + 2]
  float* ml;       // [GMAX][GQ][2] the group's split (m, l)
  float* xf;       // [D] final normed x (lm_head)
  iron_qwen3_layer* lay;  // [n_layers] copy of the layer pointer table
  double* red;     // [32]
  uint64_t* mbar;  // [NMB]
  RingState* rs;
  int* flag;       // [8]
};

__host__ __device__ inline size_t att_floats(int GQ) {
  return (size_t)GQ * HDIM + 2 * HDIM + (size_t)NWARP * GQ * (HDIM + 2);
}

// bytes of everything but the ring (carve's layout: 16 arrays, each rounded up to 16 bytes)
__host__ __device__ inline size_t fixed_smem(int kmax, int hbn, int D, int G, int GQ, int n_layers) {
  size_t o = 32 * 8 + NMB * 8 + sizeof(RingState) + 8 * 4;
  o += (size_t)(kmax / 32) * XBS + (size_t)(kmax / G) * 4 + NTMAX * TR * 8;
  o += (size_t)D * 2 * 3 + (size_t)hbn * 2 + NTMAX * TR * 2;
  o += att_floats(GQ) * 4 + (size_t)GMAX * GQ * 2 * 4 + (size_t)D * 4;
  o += (size_t)n_layers * sizeof(iron_qwen3_layer);
  return o + 16 * 16 + 64;
}

__device__ Smem carve(uint8_t* base, const Kp& p, int GQ) {
  Smem s;
  size_t o = (size_t)p.ring;
  s.ring = base;
  auto take = [&](size_t bytes) {  // every array starts on a 16-byte boundary (vector loads, bulk copies)
    uint8_t* r = base + o;
    o += (bytes + 15) & ~(size_t)15;
    return r;
  };
  const iron_qwen3_model& m = p.m;
  s.red = (double*)take(32 * 8);
  s.mbar = (uint64_t*)take(NMB * 8);
  s.rs = (RingState*)take((sizeof(RingState) + 15) & ~(size_t)15);
  s.flag = (int*)take(8 * 4);
  s.xb = take((size_t)(p.kmax / 32) * XBS);
  s.xse = (int*)take((size_t)(p.kmax / m.group) * 4);
  s.part = (double*)take(NTMAX * TR * 8);
  s.sx = (uint16_t*)take((size_t)m.D * 2);
  s.sx1 = (uint16_t*)take((size_t)m.D * 2);
  s.nw = (uint16_t*)take((size_t)m.D * 2);
  s.hb = (uint16_t*)take((size_t)p.hbn * 2);
  s.outb = (uint16_t*)take(NTMAX * TR * 2);
  s.att = (float*)take(att_floats(GQ) * 4);
  s.ml = (float*)take((size_t)GMAX * GQ * 2 * 4);
  s.xf = (float*)take((size_t)m.D * 4);
  s.lay = (iron_qwen3_layer*)take((size_t)m.n_layers * sizeof(iron_qwen3_layer));
  return s;
}

// ---------------------------------------------------------------------------
// the chunk stream: per layer QKV tiles, the split's K/V pieces, O tiles, gate/up
// pair tiles, down tiles; then the lm_head
// ---------------------------------------------------------------------------
struct Seg {
  const uint8_t* src;
  uint32_t bytes;
};

// segments of chunk i, copied back to back into one ring slot; returns their count
__device__ int chunk_segs(const Kp& p, const Plan& P, const Smem& S, int i, Seg (&sg)[2]) {
  const iron_qwen3_model& m = p.m;
  const int G = m.group, D = m.D, GQ = m.Hq / m.Hkv;
  const int lay = i / P.cpl;
  if (lay >= m.n_layers) {
    const int j = i - P.cpl * m.n_layers;
    if (m.lm_w8) {
      const int t0 = P.hlo + j * LMT, t1 = min(P.hhi, t0 + LMT);
      sg[0] = {(const uint8_t*)m.lm_w8 + (size_t)t0 * tileb(D, G), (uint32_t)((t1 - t0) * tileb(D, G))};
    } else {
      const int r0 = P.hlo + j * p.lm_rows, r1 = min(P.hhi, r0 + p.lm_rows);
      sg[0] = {(const uint8_t*)m.embed + (size_t)r0 * D * 2, (uint32_t)(r1 - r0) * D * 2};
    }
    return 1;
  }
  const iron_qwen3_layer& L = S.lay[lay];
  const int r = i - lay * P.cpl;
  if (r == 0) {  // QKV: group h's tiles are contiguous (rows packed in head-group order)
    const size_t tb = tileb(D, G);
    sg[0] = {(const uint8_t*)L.wqkv_t + ((size_t)P.h * ((GQ + 2) * HDIM / TR) + P.qt0) * tb, (uint32_t)(P.qnt * tb)};
    return 1;
  }
  if (r <= P.nkv) {  // cached K/V rows [K_t | V_t] of positions p0 .. p0 + n
    const int p0 = P.kst + (r - 1) * KVP, n = min(KVP, P.ken - p0);
    const uint16_t* head = m.kv + ((size_t)lay * m.Hkv + P.h) * 2 * (size_t)m.max_seq * HDIM;
    sg[0] = {(const uint8_t*)(head + (size_t)p0 * 2 * HDIM), (uint32_t)n * 4 * HDIM};
    return 1;
  }
  const int k = r - P.nkv;
  if (k == 1) {  // O: row tiles [ot0, ot0 + ont)
    const size_t tb = tileb(m.Hq * HDIM, G);
    sg[0] = {(const uint8_t*)L.wo_t + (size_t)P.ot0 * tb, (uint32_t)(P.ont * tb)};
    return 1;
  }
  if (k == 2) {  // gate/up tiles [gt0, gt0 + gnt)
    const size_t tb = tileb(D, G);
    sg[0] = {(const uint8_t*)L.wgu_t + (size_t)P.gt0 * tb, (uint32_t)(P.gnt * tb)};
    return 1;
  }
  const size_t tb = tileb(m.FF / DSL, G);  // down slices [ds0, ds0 + dns), tile-major
  sg[0] = {(const uint8_t*)L.wd_t + (size_t)P.ds0 * tb, (uint32_t)(P.dns * tb)};
  return 1;
}

// wait (bounded) until the copies of chunks [from, to) have landed
__device__ void drain(const Smem& S, int from, int to) {
  for (int k = from; k < to; ++k) {
    const unsigned long long t0 = gtimer();
    while (!mbar_test(&S.mbar[k % NMB], (uint32_t)((k / NMB) & 1)) && gtimer() - t0 < 20ull * 1000 * 1000) {
    }
  }
}

// The producer lane: issue every chunk of the token in stream order, each as soon
// as its ring space and slot are released.  Every wait is bounded; it stops when
// the compute threads leave early or the grid's error word is set, and then waits
// for its copies in flight.  A chunk of 0 bytes completes its slot's phase at once.
__device__ __forceinline__ void producer(const Kp& p, const Plan& P, const Smem& S, int32_t* sync) {
  volatile RingState& rs = *S.rs;
  const uint32_t R = (uint32_t)p.ring;
  unsigned long long head = 0;
  bool stop = false;
  for (int i = 0; i < P.total && !stop; ++i) {
    Seg sg[2];
    const int ns = chunk_segs(p, P, S, i, sg);
    const uint32_t bytes = sg[0].bytes + (ns > 1 ? sg[1].bytes : 0u);
    unsigned long long start = head;
    const uint32_t off = (uint32_t)(start % R);
    if (off + bytes > R) start += R - off;  // does not fit before the end: wrap
    const unsigned long long t0 = gtimer();
    for (unsigned it = 0;; ++it) {
      if (start + bytes - rs.tail <= R && i - rs.consumed < NMB) break;
      if (rs.abort) {
        stop = true;
        break;
      }
      if ((it & 15) == 15) {
        if (ld_acquire(&sync[SYNC_ERR]) != 0) {
          stop = true;
          break;
        }
        if (gtimer() - t0 > TIMEOUT_NS) {
          atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_COPY);
          stop = true;
          break;
        }
      }
      __nanosleep(32);
    }
    if (stop) break;
    const int sl = i % NMB;
    rs.slot[sl] = (uint32_t)(start % R);
    rs.end[sl] = start + bytes;
    head = start + bytes;
    uint8_t* dst = S.ring + (uint32_t)(start % R);
    fence_proxy_async();  // the compute threads' reads of this space happen before the async writes
    mbar_expect(&S.mbar[sl], bytes);
    for (int s = 0; s < ns; ++s) {
      for (uint32_t o = 0; o < sg[s].bytes; o += PIECE)
        bulk_g2s(dst + o, sg[s].src + o, min((uint32_t)PIECE, sg[s].bytes - o), &S.mbar[sl]);
      dst += sg[s].bytes;
    }
    rs.issued = i + 1;
  }
  if (stop) drain(S, rs.consumed, rs.issued);
}

__device__ bool wait_slot(uint64_t* mb, int32_t* sync, uint32_t parity) {
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    if (mbar_test(mb, parity)) return true;
    if ((it & 63) == 63) {
      if (ld_acquire(&sync[SYNC_ERR]) != 0) return false;
      if (gtimer() - t0 > TIMEOUT_NS) {
        atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_COPY);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// activation staging: K values -> B fragments of exact 31-bit block floating point
// (the arithmetic of gemv_mma_kernel's prologue, one batch row)
// ---------------------------------------------------------------------------
// src(k, v) fills v[0..7] with the values k..k+7 (bf16-representable floats).  Eight
// consecutive values per thread, G / 8 lanes per quantisation group.
template <int G, class Src>
__device__ __forceinline__ void stage_digits(const Smem& S, int K, Src src, int k_ofs = 0) {
  constexpr int TEAM = G / 8;
  const int nchunk = K >> 3;
  for (int c0 = 0; c0 < nchunk; c0 += NT) {
    const int c = c0 + threadIdx.x;
    const bool ok = c < nchunk;  // a group's TEAM lanes are all in range or all out
    float v[8];
    if (ok) {
      src(c * 8, v);  // values k_ofs + c * 8 ..
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    float mx = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
#pragma unroll
    for (int o = 1; o < TEAM; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(~0u, mx, o));
    if (!ok) continue;
    float sc, inv;
    bfp_scale(mx, sc, inv);
    // X = rn(v * 2^(30-e)); Y = (X + 0x808080) ^ 0x808080 has the balanced base-256
    // digits d0..d3 of X as its four bytes
    uint32_t Y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) Y[e] = (uint32_t)(__float2int_rn(v[e] * sc * 32768.0f) + 0x808080) ^ 0x808080u;
    const int k = k_ofs + c * 8;  // staged position (k_ofs: a multiple of the group)
    uint8_t* blk = S.xb + (size_t)(k >> 5) * XBS;
#pragma unroll
    for (int qd = 0; qd < 2; ++qd) {  // 4 values -> one word per digit (4x4 byte transpose)
      const uint32_t t0 = __byte_perm(Y[4 * qd], Y[4 * qd + 1], 0x5140);
      const uint32_t t1 = __byte_perm(Y[4 * qd], Y[4 * qd + 1], 0x7362);
      const uint32_t t2 = __byte_perm(Y[4 * qd + 2], Y[4 * qd + 3], 0x5140);
      const uint32_t t3 = __byte_perm(Y[4 * qd + 2], Y[4 * qd + 3], 0x7362);
      const uint32_t wd[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632),
                              __byte_perm(t1, t3, 0x5410), __byte_perm(t1, t3, 0x7632)};
      // B fragment: column n = digit, lane n * 4 + (kk & 15) / 4, register kk / 16
      const int kk = (k & 31) + 4 * qd;
#pragma unroll
      for (int d = 0; d < 4; ++d) *(uint32_t*)(blk + ((d * 4 + ((kk & 15) >> 2)) * 8 + (kk >> 4) * 4)) = wd[d];
    }
    // the group's scale inv * 2^-15 is a power of two: keep its exponent (inv == 0 only
    // for an all-zero group, whose digits are all zero)
    if (k % G == 0) S.xse[k / G] = inv == 0.f ? 0 : (int)((__float_as_uint(inv) >> 23) & 0xffu) - 127 - 15;
  }
  csync();
}

// RMSNorm (mode 0 kernel form, 1 golden form) of the D bf16 values x (shared) with
// the weights nw (shared) -> bf16 -> staged digits; outf (shared) gets the values.
template <int G>
__device__ __forceinline__ void norm_stage(const Smem& S, const uint16_t* x, int D, float eps, int mode,
                                           float* outf) {
  double ss = 0.0;
  for (int i = threadIdx.x; i < D; i += NT) ss += rms_sq(bf2f(x[i]), mode);
  ss = csum_d(ss, S.red);  // its barriers also publish x and nw
  const RmsCoef rc = rms_coef(ss, D, eps, mode);
  stage_digits<G>(S, D, [&](int k, float(&v)[8]) {
    const uint4 xa = *(const uint4*)(x + k), wa = *(const uint4*)(S.nw + k);
    const uint32_t xw[4] = {xa.x, xa.y, xa.z, xa.w}, ww[4] = {wa.x, wa.y, wa.z, wa.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xv = bf2f((uint16_t)(xw[e >> 1] >> (16 * (e & 1))));
      const float wv = bf2f((uint16_t)(ww[e >> 1] >> (16 * (e & 1))));
      v[e] = rbf(rms_apply(xv, wv, rc));
      if (outf) outf[k + e] = v[e];
    }
  });
}

// stage K bf16 values from shared memory (no norm)
template <int G>
__device__ __forceinline__ void plain_stage(const Smem& S, const uint16_t* x, int K, int k_ofs = 0) {
  stage_digits<G>(
      S, K,
      [&](int k, float(&v)[8]) {
        const uint4 xa = *(const uint4*)(x + k);
        const uint32_t xw[4] = {xa.x, xa.y, xa.z, xa.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = bf2f((uint16_t)(xw[e >> 1] >> (16 * (e & 1))));
      },
      k_ofs);
}

// Digits of the four consecutive values v at position k (k % 4 == 0) into the B
// fragments: G / 4 consecutive lanes hold a quantisation group and take its block
// scale together.  Every lane of the warp calls (own = false: no values).
template <int G>
__device__ __forceinline__ void stage_quad(const Smem& S, int k, const float (&v)[4], bool own) {
  constexpr int TEAM = G / 4;
  float mx = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) mx = fmaxf(mx, own ? fabsf(v[e]) : 0.f);
#pragma unroll
  for (int o = 1; o < TEAM; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(~0u, mx, o));
  if (!own) return;
  float sc, inv;
  bfp_scale(mx, sc, inv);
  uint32_t Y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) Y[e] = (uint32_t)(__float2int_rn(v[e] * sc * 32768.0f) + 0x808080) ^ 0x808080u;
  const uint32_t t0 = __byte_perm(Y[0], Y[1], 0x5140), t1 = __byte_perm(Y[0], Y[1], 0x7362);
  const uint32_t t2 = __byte_perm(Y[2], Y[3], 0x5140), t3 = __byte_perm(Y[2], Y[3], 0x7362);
  const uint32_t wd[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632), __byte_perm(t1, t3, 0x5410),
                          __byte_perm(t1, t3, 0x7632)};
  uint8_t* blk = S.xb + (size_t)(k >> 5) * XBS;
  const int kk = k & 31;
#pragma unroll
  for (int d = 0; d < 4; ++d) *(uint32_t*)(blk + ((d * 4 + ((kk & 15) >> 2)) * 8 + (kk >> 4) * 4)) = wd[d];
  if (k % G == 0) S.xse[k / G] = inv == 0.f ? 0 : (int)((__float_as_uint(inv) >> 23) & 0xffu) - 127 - 15;
}

// RMSNorm (mode 0 kernel form, 1 golden form) of D values held four per thread (thread
// t: values 4t..4t+3 in vx; threads with 4t >= D hold none) with the weights nw (shared)
// -> bf16 -> staged digits; outf (shared) gets the normalised values.  One block
// reduction: every thread adds the warps' partial sums in warp order.
template <int G>
__device__ __forceinline__ void norm_stage_q(const Smem& S, const float (&vx)[4], int D, float eps, int mode,
                                             float* outf) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, k = 4 * threadIdx.x;
  const bool own = k < D;
  double ss = 0.0;
  if (own) {
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += rms_sq(vx[e], mode);
  }
  ss = warp_sum_d(ss);
  if (lane == 0) S.red[wid] = ss;
  csync();
  double tot = 0.0;
#pragma unroll
  for (int w = 0; w < NWARP; ++w) tot += S.red[w];
  const RmsCoef rc = rms_coef(tot, D, eps, mode);
  float v[4];
  if (own) {
    const uint2 wa = *(const uint2*)(S.nw + k);
    const uint32_t ww[2] = {wa.x, wa.y};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[e] = rbf(rms_apply(vx[e], bf2f((uint16_t)(ww[e >> 1] >> (16 * (e & 1)))), rc));
      if (outf) outf[k + e] = v[e];
    }
  }
  stage_quad<G>(S, k, v, own);
  csync();
}

// the four bf16 values of the two words w0 (values 0, 1) and w1 (2, 3)
__device__ __forceinline__ void quad_of(uint32_t w0, uint32_t w1, float (&v)[4]) {
  v[0] = bf_lo(w0);
  v[1] = bf_hi(w0);
  v[2] = bf_lo(w1);
  v[3] = bf_hi(w1);
}

// K bf16 values (K % 8 == 0, read-only data) into shared memory with 16-byte loads
__device__ __forceinline__ void load_ro(uint16_t* dst, const uint16_t* src, int K) {
  for (int i = threadIdx.x; i < (K >> 3); i += NT) ((uint4*)dst)[i] = __ldg(((const uint4*)src) + i);
}

// ---------------------------------------------------------------------------
// Projection of nt packed weight tiles (16 rows x K) in a ring slot against the
// staged activation.  Tile layout: K/32 blocks of 512 bytes (lane L's A fragment at
// L * 16), then K/G groups of 8 x 2 bf16 scales (rows g and g + 8 in one word).  Tile
// t reads the staged 32-column blocks from xkb0 + t * xkbs on (xkbs = 0: one shared
// activation vector).  The warps split each tile's blocks into SL slices; the slice
// sums meet in shared memory and are added in slice order.  PAIR: rows 8..15 of a
// tile are the up rows of its gate rows 0..7, and epi(t, i, gate sum, up sum) runs
// for i < 8; otherwise epi(t, r, sum, 0) for r < 16.
//
// Per 32-column block a lane turns its two exact integer sums c into c * 2^e (the
// activation group's power-of-two scale) by building the double 2^52 + c + 2^31 at
// exponent e and subtracting 2^52 + 2^31 at the same exponent (both exact), then
// multiplies by the bf16 weight scale and accumulates in float64: the products are
// exact, as before any rounding of the sum.
// ---------------------------------------------------------------------------
template <int G, bool PAIR, class Epi>
__device__ __forceinline__ void gemv_tiles(const uint8_t* slot, int nt, int K, int xkb0, int xkbs, const Smem& S,
                                           Epi epi) {
  if (nt <= 0) return;  // uniform across the CTA
  constexpr int UN = 4;  // blocks whose loads go out together
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int KB = K >> 5;
  const size_t TB = tileb(K, G);
  const int lsl = nt >= NWARP ? 0 : (nt >= 4 ? 1 : (nt >= 2 ? 2 : 3));  // log2 of the slices per tile
  const int SL = 1 << lsl, items = nt << lsl;
  for (int it = wid; it < items; it += NWARP) {
    const int t = it >> lsl, s = it & (SL - 1);
    const int kb0 = (s * KB) >> lsl, kb1 = ((s + 1) * KB) >> lsl;
    const uint8_t* tb = slot + (size_t)t * TB;
    const uint8_t* scb = tb + (size_t)KB * 512 + (lane >> 2) * 4;
    const int xk = xkb0 + t * xkbs;  // this tile's first staged block
    double a0 = 0.0, a1 = 0.0;
    auto step = [&](uint4 a, uint2 bv, uint32_t sw, int ex) {
      int cc[4];
      mma_s8(cc, a, bv);
      const uint32_t hi = (uint32_t)(0x433 + ex) << 20;
      const double bias = __hiloint2double((int)hi, (int)0x80000000u);
      const double d0 = __hiloint2double((int)hi, (int)((uint32_t)(cc[0] + 256 * cc[1]) ^ 0x80000000u)) - bias;
      const double d1 = __hiloint2double((int)hi, (int)((uint32_t)(cc[2] + 256 * cc[3]) ^ 0x80000000u)) - bias;
      a0 = fma(d0, (double)bf_lo(sw), a0);
      a1 = fma(d1, (double)bf_hi(sw), a1);
    };
    int kb = kb0;
    for (; kb + UN <= kb1; kb += UN) {
      uint2 bv[UN];
      uint4 a[UN];
      uint32_t sw[UN];
      int ex[UN];
#pragma unroll
      for (int u = 0; u < UN; ++u) {
        bv[u] = *(const uint2*)(S.xb + (size_t)(xk + kb + u) * XBS + lane * 8);
        a[u] = *(const uint4*)(tb + (size_t)(kb + u) * 512 + lane * 16);
        sw[u] = *(const uint32_t*)(scb + (((kb + u) * 32) / G) * 32);
        ex[u] = S.xse[((xk + kb + u) * 32) / G];
      }
#pragma unroll
      for (int u = 0; u < UN; ++u) step(a[u], bv[u], sw[u], ex[u]);
    }
    for (; kb < kb1; ++kb)
      step(*(const uint4*)(tb + (size_t)kb * 512 + lane * 16), *(const uint2*)(S.xb + (size_t)(xk + kb) * XBS + lane * 8),
           *(const uint32_t*)(scb + ((kb * 32) / G) * 32), S.xse[((xk + kb) * 32) / G]);
    // odd lanes hold the digit pieces weighted 2^16; after the pair sum lanes 4g hold
    // rows g and g + 8 (lanes 4g + 2 hold the empty second batch row)
    a0 = (lane & 1) ? 65536.0 * a0 : a0;
    a1 = (lane & 1) ? 65536.0 * a1 : a1;
    a0 += __shfl_xor_sync(~0u, a0, 1);
    a1 += __shfl_xor_sync(~0u, a1, 1);
    if ((lane & 3) == 0) {
      S.part[(size_t)it * TR + (lane >> 2)] = a0;
      S.part[(size_t)it * TR + (lane >> 2) + 8] = a1;
    }
  }
  csync();
  if (PAIR) {
    for (int e = threadIdx.x; e < nt * 8; e += NT) {
      const int t = e >> 3, i = e & 7;
      double g = 0.0, u = 0.0;
      for (int s = 0; s < SL; ++s) {
        g += S.part[(size_t)((t << lsl) + s) * TR + i];
        u += S.part[(size_t)((t << lsl) + s) * TR + i + 8];
      }
      epi(t, i, g, u);
    }
  } else {
    for (int e = threadIdx.x; e < nt * TR; e += NT) {
      const int t = e >> 4, r = e & 15;
      double a = 0.0;
      for (int s = 0; s < SL; ++s) a += S.part[(size_t)((t << lsl) + s) * TR + r];
      epi(t, r, a, 0.0);
    }
  }
}

// bf16 rows with this lane's activations held in registers: xr[k] = xf[(lane + 32k)*8 ..]
// (the lm_head arithmetic of gemv_bf16_kernel)
template <int R, int KC>
__device__ __forceinline__ void rows_dot_bf16_reg(const uint8_t* const (&rp)[R], const float (&xr)[KC][8],
                                                  float (&out)[R]) {
  const int lane = threadIdx.x & 31;
  float a[R];
#pragma unroll
  for (int i = 0; i < R; ++i) a[i] = 0.f;
#pragma unroll
  for (int k = 0; k < KC; ++k) {
    uint4 w[R];
#pragma unroll
    for (int i = 0; i < R; ++i) w[i] = *(const uint4*)(rp[i] + (lane + 32 * k) * 16);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      a[i] = fmaf(bf_lo(w[i].x), xr[k][0], a[i]);
      a[i] = fmaf(bf_hi(w[i].x), xr[k][1], a[i]);
      a[i] = fmaf(bf_lo(w[i].y), xr[k][2], a[i]);
      a[i] = fmaf(bf_hi(w[i].y), xr[k][3], a[i]);
      a[i] = fmaf(bf_lo(w[i].z), xr[k][4], a[i]);
      a[i] = fmaf(bf_hi(w[i].z), xr[k][5], a[i]);
      a[i] = fmaf(bf_lo(w[i].w), xr[k][6], a[i]);
      a[i] = fmaf(bf_hi(w[i].w), xr[k][7], a[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) out[i] = warp_sum(a[i]);
}

// the same for any D (a multiple of 256) with the activations in shared memory
template <int R>
__device__ __forceinline__ void rows_dot_bf16(const uint8_t* const (&rp)[R], int K, const float* xf, float (&out)[R]) {
  const int lane = threadIdx.x & 31;
  float a[R];
#pragma unroll
  for (int i = 0; i < R; ++i) a[i] = 0.f;
  for (int c = lane; c < (K >> 3); c += 32) {
    const float4 x0 = *(const float4*)(xf + c * 8), x1 = *(const float4*)(xf + c * 8 + 4);
    uint4 w[R];
#pragma unroll
    for (int i = 0; i < R; ++i) w[i] = *(const uint4*)(rp[i] + c * 16);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      a[i] = fmaf(bf_lo(w[i].x), x0.x, a[i]);
      a[i] = fmaf(bf_hi(w[i].x), x0.y, a[i]);
      a[i] = fmaf(bf_lo(w[i].y), x0.z, a[i]);
      a[i] = fmaf(bf_hi(w[i].y), x0.w, a[i]);
      a[i] = fmaf(bf_lo(w[i].z), x1.x, a[i]);
      a[i] = fmaf(bf_hi(w[i].z), x1.y, a[i]);
      a[i] = fmaf(bf_lo(w[i].w), x1.z, a[i]);
      a[i] = fmaf(bf_hi(w[i].w), x1.w, a[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) out[i] = warp_sum(a[i]);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// attention of one split: online softmax state of a warp over U positions at a time
// (the arithmetic of attn_split_kernel)
// ---------------------------------------------------------------------------
template <int GQ, int U>
__device__ __forceinline__ void attn_update(const float (&q)[GQ][4], const float (&kf)[U][4], const float (&vf)[U][4],
                                            int nvalid, float scale, float (&mm)[GQ], float (&ll)[GQ],
                                            float (&o)[GQ][4]) {
#pragma unroll
  for (int g = 0; g < GQ; ++g) {
    float sv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) d = fmaf(q[g][e], kf[u][e], d);
      sv[u] = warp_sum(d) * scale;
      if (u >= nvalid) sv[u] = -INFINITY;
    }
    float mn = mm[g];
#pragma unroll
    for (int u = 0; u < U; ++u) mn = fmaxf(mn, sv[u]);
    const float corr = exp2f(mm[g] - mn);
    float ls = ll[g] * corr;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[g][e] *= corr;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float pu = exp2f(sv[u] - mn);
      ls += pu;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[g][e] = fmaf(pu, vf[u][e], o[g][e]);
    }
    ll[g] = ls;
    mm[g] = mn;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int G, int GQ>
__global__ void __launch_bounds__(NT + 32, 1) qwen3_step_kernel(const __grid_constant__ Kp p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const iron_qwen3_model& m = p.m;
  const Smem S = carve(smem_raw, p, GQ);
  int32_t* sync = m.sync;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int N = gridDim.x, D = m.D, NL = m.n_layers, FF = m.FF;
  const int pos = m.pos[0];
  // a position outside the cache or a token outside the vocabulary: record and leave
  // before touching memory (every CTA takes the same decision)
  if (pos < 0 || pos >= m.max_seq || (p.embed_input && (m.tok[0] < 0 || m.tok[0] >= m.V))) {
    if (tid == 0) atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_INPUT);
    return;
  }
  const Plan P = make_plan(p, pos);
  const uint32_t tok_epoch = (uint32_t)__ldcg((const int*)&sync[SYNC_EPOCH]);
  // hand-off words (zeroed by iron_qwen3_sync_reset)
  constexpr int RAWW = (GQ + 2) * HDIM / 2;  // q/k/v words of one KV-head group
  constexpr int ATTW = GQ * (HDIM + 2);      // words of one attention split
  unsigned long long* dpw = (unsigned long long*)m.attn_ws;         // [D / TR][DSL][TR] down partial sums
  unsigned long long* raww = dpw + (size_t)DSL * D;                 // [Hkv][RAWW]
  unsigned long long* attw = raww + (size_t)m.Hkv * RAWW;           // [Hkv][GMAX][ATTW]
  unsigned long long* mw = attw + (size_t)m.Hkv * GMAX * ATTW;      // [Hkv][GQ * HD / 2] merged heads
  unsigned long long* x1w = mw + (size_t)m.Hq * HDIM / 2;           // [D / 2] x1 rows
  unsigned long long* hw = x1w + D / 2;                             // [FF / 2] SwiGLU outputs
  if (tid < NT) {
    // the layer pointer table, read once; the unused second batch row of the B
    // fragments stays zero
    const int nw = NL * (int)(sizeof(iron_qwen3_layer) / 8);
    for (int i = tid; i < nw; i += NT) ((unsigned long long*)S.lay)[i] = __ldg(((const unsigned long long*)m.layers) + i);
    for (int i = tid; i < (p.kmax / 32) * XBS / 16; i += NT) ((uint4*)S.xb)[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (tid == 0) {
    for (int i = 0; i < NMB; ++i) mbar_init(&S.mbar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    S.rs->tail = 0;
    S.rs->issued = S.rs->consumed = S.rs->abort = 0;
  }
  __syncthreads();  // the last barrier of all NT + 32 threads
  if (tid >= NT) {
    if (tid == NT) producer(p, P, S, sync);
    return;
  }
  // layer-0 input: the token's embedding row, or the hidden state given in x (thread t
  // loads values 4t..4t+3, the ones it normalises)
  {
    const uint16_t* src = p.embed_input ? m.embed + (size_t)m.tok[0] * D : m.x;
    if (4 * tid < D) *(uint2*)(S.sx + 4 * tid) = __ldg((const uint2*)(src + 4 * tid));
  }

  bool ok = true;
  volatile RingState& vrs = *S.rs;
  int ci = 0;  // next chunk
  // consume the next chunk: fn(buffer) once its copy landed, then release its space
  // (mark: the profiling stamp taken when the copy has landed, in row mrow)
  auto consume = [&](int mrow, int mark, auto&& fn) -> bool {
    const int i = ci++;
    const int sl = i % NMB;
    if (tid == 0) S.flag[2] = wait_slot(&S.mbar[sl], sync, (uint32_t)((i / NMB) & 1)) ? 1 : 0;
    csync();
    if (!S.flag[2]) return false;
    if (mark >= 0) STEP_MARK(mrow, mark);
    (void)mrow;
    fn(S.ring + vrs.slot[sl]);
    csync();
    if (tid == 0) {
      fence_proxy_async();
      vrs.tail = vrs.end[sl];
      vrs.consumed = i + 1;
    }
    return true;
  };
  // a bounded poll by every compute thread, then a CTA-wide verdict
  auto all_ok = [&](bool mine) -> bool { return !cvote_any(!mine); };

  // x = bf16(x1 + bf16(sum of the DSL down slices, in slice order)) for rows 4t..4t+3
  // of thread t (D <= 4 * NT), from the words of the layer tagged tg; all 4 * DSL words
  // of a thread are loaded and reloaded together.  The values go to xv and to sx.
  auto next_x = [&](uint32_t tg, float (&xv)[4]) -> bool {
    constexpr int NU = 4 * DSL;
    unsigned long long v[NU];
    const bool own = 4 * tid < D;
    auto d_addr = [&](int u) {
      const int r = 4 * tid + u / DSL;
      return dpw + ((size_t)(r >> 4) * DSL + (u % DSL)) * TR + (r & 15);
    };
#pragma unroll
    for (int u = 0; u < NU; ++u) v[u] = own ? ll_ld(d_addr(u)) : 0ull;
    const bool mine = poll_rounds<NU>(d_addr, v, own ? 0xffffu : 0u, tg, 48, sync);
    if (!all_ok(mine)) return false;
    if (own) {
      uint16_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        double acc = 0.0;
#pragma unroll
        for (int j = 0; j < DSL; ++j) acc += ll_val_d(v[e * DSL + j]);
        o[e] = f2bf(bf2f(S.sx1[4 * tid + e]) + rbf_d(acc));
        xv[e] = bf2f(o[e]);
      }
      *(uint2*)(S.sx + 4 * tid) = make_uint2(o[0] | ((uint32_t)o[1] << 16), o[2] | ((uint32_t)o[3] << 16));
    }
    return true;
  };

  const int h = P.h;
  const float scale = 1.4426950408889634f / sqrtf((float)HDIM);
  for (int layer = 0; layer < NL && ok; ++layer) {
    const iron_qwen3_layer& Lw = S.lay[layer];
    const uint32_t ep = tok_epoch * (uint32_t)NL + (uint32_t)layer + 1u;  // this layer's flag value
    const uint32_t tg = tag16_of(ep);
    STEP_MARK(layer, 0);
    // ---- x: the previous layer's output rows ----
    load_ro(S.nw, Lw.norm1, D);
    float xv[4];
    if (layer > 0) {  // the previous layer's down slices, with its epoch
      if (!(ok = next_x(tag16_of(ep - 1u), xv))) break;
    } else {  // the embedding row (or x) as this thread loaded it into sx
      if (4 * tid < D) {
        const uint2 w2 = *(const uint2*)(S.sx + 4 * tid);
        quad_of(w2.x, w2.y, xv);
      }
    }
    STEP_MARK(layer, 1);
    // ---- QKV rows of group h: raw = bf16(Wqkv @ RMSNorm_golden(x, norm1)) ----
    norm_stage_q<G>(S, xv, D, m.eps, 1, nullptr);  // its barriers also publish sx and nw
    if (m.trace && blockIdx.x == 0)
      for (int i = tid; i < D; i += NT) m.trace[(size_t)layer * D + i] = S.sx[i];
    STEP_MARK(layer, 2);
    ok = consume(layer, 3, [&](const uint8_t* wb) {
      gemv_tiles<G, false>(wb, P.qnt, D, 0, 0, S, [&](int t, int r, double a, double) {
        S.outb[t * TR + r] = f2bf((float)a);
      });
    });
    if (!ok) break;
    for (int i = tid; i < P.qnt * TR / 2; i += NT)
      ll_put(raww + (size_t)h * RAWW + P.qt0 * TR / 2 + i, ((const uint32_t*)S.outb)[i], ep);
    STEP_MARK(layer, 4);
    // ---- attention: KV head h, one split of the positions ----
    ok = all_ok(poll<2>(raww + (size_t)h * RAWW, RAWW, ep, 32, sync, [&](int i, unsigned long long w) {
      ((uint32_t*)S.hb)[i] = (uint32_t)w;
    }));
    if (!ok) break;
    STEP_MARK(layer, 5);
    float* qf = S.att;           // [GQ][HD]
    float* kt = qf + GQ * HDIM;  // [HD]
    float* vt = kt + HDIM;       // [HD]
    float* wpart = vt + HDIM;    // [NWARP][GQ][HD + 2]
    uint16_t* head = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
    {
      // per-head q/k RMSNorm (golden form) + RoPE and the v copy: the arithmetic of
      // qk_norm_rope_kv_kernel; the split that holds pos writes K_t, V_t
      const uint16_t* ang = m.angles + (size_t)pos * HDIM;
      for (int t = wid; t < GQ + 2; t += NWARP) {
        const uint16_t* src = S.hb + t * HDIM;
        if (t == GQ + 1) {
          for (int i = lane; i < HDIM; i += 32) {
            vt[i] = bf2f(src[i]);
            if (P.own) head[(size_t)pos * 2 * HDIM + HDIM + i] = src[i];
          }
          continue;
        }
        const bool isq = t < GQ;
        const uint16_t* nwt = isq ? Lw.qn : Lw.kn;
        constexpr int PER = HDIM / 32;
        float v[PER], wv[PER], cs[PER / 2], sn[PER / 2];
#pragma unroll
        for (int j = 0; j < PER / 2; ++j) {
          const int i = lane + 32 * j;
          v[2 * j] = bf2f(src[i]);
          v[2 * j + 1] = bf2f(src[i + HDIM / 2]);
          wv[2 * j] = bf2f(__ldg(nwt + i));
          wv[2 * j + 1] = bf2f(__ldg(nwt + i + HDIM / 2));
          cs[j] = bf2f(__ldg(ang + 2 * i));
          sn[j] = bf2f(__ldg(ang + 2 * i + 1));
        }
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < PER; ++e) ss += rms_sq(v[e], 1);
        ss = warp_sum_d(ss);
        const RmsCoef rc = rms_coef(ss, HDIM, m.eps, 1);
        float* dst = isq ? qf + t * HDIM : kt;
#pragma unroll
        for (int j = 0; j < PER / 2; ++j) {
          const int i = lane + 32 * j;
          const float x1 = rbf(rms_apply(v[2 * j], wv[2 * j], rc));
          const float x2 = rbf(rms_apply(v[2 * j + 1], wv[2 * j + 1], rc));
          const uint16_t o1 = f2bf(__fsub_rn(__fmul_rn(x1, cs[j]), __fmul_rn(x2, sn[j])));
          const uint16_t o2 = f2bf(__fadd_rn(__fmul_rn(x2, cs[j]), __fmul_rn(x1, sn[j])));
          dst[i] = bf2f(o1);
          dst[i + HDIM / 2] = bf2f(o2);
          if (!isq && P.own) {
            head[(size_t)pos * 2 * HDIM + i] = o1;
            head[(size_t)pos * 2 * HDIM + i + HDIM / 2] = o2;
          }
        }
      }
    }
    csync();
    STEP_MARK(layer, 6);
    // flash decoding over the cached positions (K/V chunks in the ring) and, in the
    // split that holds it, the current position (K/V from the registers above)
    float q[GQ][4], mm[GQ], ll[GQ], o[GQ][4];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      mm[g] = -INFINITY;
      ll[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[g][e] = qf[g * HDIM + lane * 4 + e];
        o[g][e] = 0.f;
      }
    }
    constexpr int U = 4;
    for (int j = 0; j < P.nkv && ok; ++j) {
      const int n = min(KVP, P.ken - (P.kst + j * KVP));
      ok = consume(layer, -1, [&](const uint8_t* kvb) {
        for (int j0 = wid * U; j0 < n; j0 += NWARP * U) {
          float kf[U][4], vf[U][4];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int jj = min(j0 + u, n - 1);
            const uint2 kk = *(const uint2*)(kvb + (size_t)jj * 4 * HDIM + lane * 8);
            const uint2 vv = *(const uint2*)(kvb + (size_t)jj * 4 * HDIM + 2 * HDIM + lane * 8);
            kf[u][0] = bf_lo(kk.x);
            kf[u][1] = bf_hi(kk.x);
            kf[u][2] = bf_lo(kk.y);
            kf[u][3] = bf_hi(kk.y);
            vf[u][0] = bf_lo(vv.x);
            vf[u][1] = bf_hi(vv.x);
            vf[u][2] = bf_lo(vv.y);
            vf[u][3] = bf_hi(vv.y);
          }
          attn_update<GQ, U>(q, kf, vf, n - j0, scale, mm, ll, o);
        }
      });
    }
    if (!ok) break;
    if (P.own && wid == NWARP - 1) {
      float kf[1][4], vf[1][4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        kf[0][e] = kt[lane * 4 + e];
        vf[0][e] = vt[lane * 4 + e];
      }
      attn_update<GQ, 1>(q, kf, vf, 1, scale, mm, ll, o);
    }
    STEP_MARK(layer, 7);
    // merge the warps; publish this split's partial (o, m, l) per head
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      float* pw = wpart + (wid * GQ + g) * (HDIM + 2);
#pragma unroll
      for (int e = 0; e < 4; ++e) pw[lane * 4 + e] = o[g][e];
      if (lane == 0) {
        pw[HDIM] = mm[g];
        pw[HDIM + 1] = ll[g];
      }
    }
    csync();
    {
      unsigned long long* ws = attw + ((size_t)h * GMAX + P.gi) * ATTW;
      for (int t = tid; t < GQ * HDIM; t += NT) {
        const int g = t / HDIM, d = t - g * HDIM;
        float M = -INFINITY;
        for (int w = 0; w < NWARP; ++w) M = fmaxf(M, wpart[(w * GQ + g) * (HDIM + 2) + HDIM]);
        float oo = 0.f, lsum = 0.f;
        if (M != -INFINITY) {
          for (int w = 0; w < NWARP; ++w) {
            const float* pw = wpart + (w * GQ + g) * (HDIM + 2);
            const float f = exp2f(pw[HDIM] - M);
            oo = fmaf(pw[d], f, oo);
            lsum = fmaf(pw[HDIM + 1], f, lsum);
          }
        }
        ll_put(ws + g * (HDIM + 2) + d, __float_as_uint(oo), ep);
        if (d == 0) {
          ll_put(ws + g * (HDIM + 2) + HDIM, __float_as_uint(M), ep);
          ll_put(ws + g * (HDIM + 2) + HDIM + 1, __float_as_uint(lsum), ep);
        }
      }
    }
    STEP_MARK(layer, 8);
    // ---- the group's first CTA merges its splits (attn_combine_kernel's arithmetic) and
    //      publishes the merged heads as bf16 words ----
    if (P.gi == 0) {
      const unsigned long long* gws = attw + (size_t)h * GMAX * ATTW;
      bool mine = true;
      // (m, l) of every split and head into shared memory
      {
        const int nml = P.gsz * GQ * 2;
        unsigned long long v[2];
        uint32_t want = 0;
        auto ml_addr = [&](int u) {
          const int t = tid + u * NT, s = t / (2 * GQ), r = t - s * 2 * GQ;
          return gws + (size_t)s * ATTW + (r >> 1) * (HDIM + 2) + HDIM + (r & 1);
        };
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          v[u] = 0ull;
          if (tid + u * NT < nml) {
            v[u] = ll_ld(ml_addr(u));
            want |= 1u << u;
          }
        }
        mine = poll_rounds<2>(ml_addr, v, want, ep, 32, sync);
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if ((want >> u) & 1u) S.ml[tid + u * NT] = __uint_as_float((uint32_t)v[u]);
      }
      for (int t0 = 0; t0 < GQ * HDIM; t0 += NT) {
        const int t = t0 + tid;
        const int g = t / HDIM, d = t - g * HDIM;
        // the split outputs o[s][g][d]: loaded and reloaded together
        float ov[GMAX];
        unsigned long long v[GMAX];
        uint32_t want = 0;
        const unsigned long long* ob = gws + g * (HDIM + 2) + d;
#pragma unroll
        for (int s = 0; s < GMAX; ++s) {
          v[s] = 0ull;
          if (s < P.gsz && t < GQ * HDIM) {
            v[s] = ll_ld(ob + (size_t)s * ATTW);
            want |= 1u << s;
          }
        }
        mine = mine && poll_rounds<GMAX>([&](int s) { return ob + (size_t)s * ATTW; }, v, want, ep, 32, sync);
#pragma unroll
        for (int s = 0; s < GMAX; ++s) ov[s] = __uint_as_float((uint32_t)v[s]);
        if (!all_ok(mine)) {  // also publishes ml
          ok = false;
          break;
        }
        if (t < GQ * HDIM) {
          const float* mlg = S.ml + g * 2;
          float M = -INFINITY;
          for (int s = 0; s < P.gsz; ++s) M = fmaxf(M, mlg[s * 2 * GQ]);
          float oo = 0.f, lsum = 0.f;
          if (M != -INFINITY) {
#pragma unroll
            for (int s = 0; s < GMAX; ++s) {
              if (s >= P.gsz) continue;
              const float f = exp2f(mlg[s * 2 * GQ] - M);
              oo = fmaf(ov[s], f, oo);
              lsum = fmaf(mlg[s * 2 * GQ + 1], f, lsum);
            }
          }
          S.hb[t] = f2bf(lsum > 0.f ? oo / lsum : 0.f);
        }
      }
      if (!ok) break;
      csync();  // the merged heads, one value per thread, go out two per word
      for (int i = tid; i < GQ * HDIM / 2; i += NT)
        ll_put(mw + (size_t)h * (GQ * HDIM / 2) + i, ((const uint32_t*)S.hb)[i], ep);
    }
    STEP_MARK(layer, 9);
    // ---- O row tiles over all heads: x1 = bf16(x + bf16(Wo @ attn)) ----
    if (P.ont > 0) {  // quad q = tid + j * NT: words 2q, 2q + 1 -> staged values 4q..4q+3
      const int nq = m.Hq * HDIM / 4;
      bool mine = true;
      for (int q0 = 0; q0 < nq; q0 += NT) {
        const int q = q0 + tid;
        const bool own = q < nq;
        unsigned long long v[2] = {own ? ll_ld(mw + 2 * q) : 0ull, own ? ll_ld(mw + 2 * q + 1) : 0ull};
        mine = mine && poll_rounds<2>([&](int u) { return mw + 2 * q + u; }, v, own ? 3u : 0u, ep, 32, sync);
        float hv[4];
        quad_of((uint32_t)v[0], (uint32_t)v[1], hv);
        stage_quad<G>(S, 4 * q, hv, own);
      }
      if (!(ok = all_ok(mine))) break;  // also publishes the staged digits
    }
    STEP_MARK(layer, 10);
    ok = consume(layer, 11, [&](const uint8_t* wb) {
      gemv_tiles<G, false>(wb, P.ont, m.Hq * HDIM, 0, 0, S, [&](int t, int r, double a, double) {
        S.outb[t * TR + r] = f2bf(bf2f(S.sx[(P.ot0 + t) * TR + r]) + rbf_d(a));
      });
    });
    if (!ok) break;
    for (int i = tid; i < P.ont * TR / 2; i += NT) ll_put(x1w + P.ot0 * TR / 2 + i, ((const uint32_t*)S.outb)[i], ep);
    STEP_MARK(layer, 12);
    // ---- x1 rows from the O tiles; MLP RMSNorm ----
    load_ro(S.nw, Lw.norm2, D);
    {  // thread t: x1 rows 4t..4t+3 (words 2t, 2t + 1)
      const bool own = 4 * tid < D;
      unsigned long long v[2] = {own ? ll_ld(x1w + 2 * tid) : 0ull, own ? ll_ld(x1w + 2 * tid + 1) : 0ull};
      if (!(ok = all_ok(poll_rounds<2>([&](int u) { return x1w + 2 * tid + u; }, v, own ? 3u : 0u, ep, 32, sync))))
        break;
      quad_of((uint32_t)v[0], (uint32_t)v[1], xv);
      if (own) *(uint2*)(S.sx1 + 4 * tid) = make_uint2((uint32_t)v[0], (uint32_t)v[1]);
    }
    STEP_MARK(layer, 13);
    norm_stage_q<G>(S, xv, D, m.eps, 0, nullptr);
    STEP_MARK(layer, 14);
    // ---- gate/up: gh = bf16(silu_tanh(bf16(Wg@hf)) * bf16(Wu@hf)) for the CTA's tiles ----
    ok = consume(layer, 15, [&](const uint8_t* wb) {
      gemv_tiles<G, true>(wb, P.gnt, D, 0, 0, S, [&](int t, int i, double g, double u) {
        S.outb[t * 8 + i] = f2bf(silu_tanh_bf16(rbf_d(g)) * rbf_d(u));
      });
    });
    if (!ok) break;
    for (int i = tid; i < P.gnt * 4; i += NT) ll_put(hw + P.gt0 * 4 + i, ((const uint32_t*)S.outb)[i], ep);
    STEP_MARK(layer, 16);
    // ---- down: this CTA's slices, partial[t][j][r] = Wd[tile t rows, K slice j] @ gh[slice j] ----
    {
      const int KS = FF / DSL;  // columns of a slice
      // the gh values of the CTA's slices, staged side by side: staged quad i (value 4i)
      // is quad i % (KS / 4) of slice i / (KS / 4)
      const int nq = P.dns * (KS / 4);
      bool mine = true;
      for (int q0 = 0; q0 < nq; q0 += NT) {
        const int q = q0 + tid;
        const bool own = q < nq;
        const int sl = own ? q / (KS / 4) : 0, qi = q - sl * (KS / 4);
        const unsigned long long* wp = hw + (size_t)((P.ds0 + sl) % DSL) * (KS / 2) + 2 * qi;
        unsigned long long v[2] = {own ? ll_ld(wp) : 0ull, own ? ll_ld(wp + 1) : 0ull};
        mine = mine && poll_rounds<2>([&](int u) { return wp + u; }, v, own ? 3u : 0u, ep, 32, sync);
        float hv[4];
        quad_of((uint32_t)v[0], (uint32_t)v[1], hv);
        stage_quad<G>(S, 4 * q, hv, own);
      }
      if (!(ok = all_ok(mine))) break;  // also publishes the staged digits
      STEP_MARK(layer, 17);
      STEP_MARK(layer, 18);
      ok = consume(layer, 19, [&](const uint8_t* wb) {
        gemv_tiles<G, false>(wb, P.dns, KS, 0, KS / 32, S, [&](int q, int r, double a, double) {
          ll_put_d(dpw + (size_t)(P.ds0 + q) * TR + r, a, tg);
        });
      });
      if (!ok) break;
    }
    STEP_MARK(layer, 20);
  }

  STEP_MARK(NL, 0);
  if (ok) {
    // ---- final: x = the last layer's output, RMSNorm (golden) + lm_head + greedy argmax ----
    const uint32_t ep = tok_epoch * (uint32_t)NL + (uint32_t)NL;
    load_ro(S.nw, m.final_norm, D);
    float xv[4];
    ok = next_x(tag16_of(ep), xv);
    csync();  // sx, written four values per thread, is read across threads below
  }
  if (ok) {
    if (blockIdx.x == 0) {
      for (int i = tid; i < D; i += NT) {
        m.x[i] = S.sx[i];
        if (m.trace) m.trace[(size_t)NL * D + i] = S.sx[i];
      }
    }
    if (m.lm_w8) {
      norm_stage<G>(S, S.sx, D, m.eps, 1, S.xf);
    } else {
      // golden RMSNorm -> float activations (no staging)
      double ss = 0.0;
      for (int i = tid; i < D; i += NT) ss += rms_sq(bf2f(S.sx[i]), 1);
      ss = csum_d(ss, S.red);
      const RmsCoef rc = rms_coef(ss, D, m.eps, 1);
      for (int i = tid; i < D; i += NT) S.xf[i] = rbf(rms_apply(bf2f(S.sx[i]), bf2f(S.nw[i]), rc));
      csync();
    }
    STEP_MARK(NL, 1);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    auto track = [&](int idx, uint16_t o) {
      if (m.logits) m.logits[idx] = o;
      if (better(bf2f(o), idx, bv, bi)) {
        bv = bf2f(o);
        bi = idx;
      }
    };
    float xr[4][8];  // this lane's activations for the D == 1024 bf16 rows
    if (D == 1024 && !m.lm_w8) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[k][e] = S.xf[(lane + 32 * k) * 8 + e];
    }
    for (int j = 0; j < P.hnch && ok; ++j) {
      if (m.lm_w8) {
        const int t0 = P.hlo + j * LMT, nt = min(P.hhi, t0 + LMT) - t0;
        ok = consume(NL, -1, [&](const uint8_t* wb) {
          gemv_tiles<G, false>(wb, nt, D, 0, 0, S, [&](int t, int r, double a, double) {
            const int row = (t0 + t) * TR + r;
            if (row < m.V) track(row, f2bf((float)a));
          });
        });
      } else {
        const int r0 = P.hlo + j * p.lm_rows, n = min(P.hhi, r0 + p.lm_rows) - r0;
        ok = consume(NL, -1, [&](const uint8_t* wb) {
          constexpr int R = 4;
          for (int rr = wid * R; rr < n; rr += NWARP * R) {
            const uint8_t* rp[R];
#pragma unroll
            for (int i = 0; i < R; ++i) rp[i] = wb + (size_t)min(rr + i, n - 1) * D * 2;
            float out[R];
            if (D == 1024)
              rows_dot_bf16_reg<R, 4>(rp, xr, out);
            else
              rows_dot_bf16<R>(rp, D, S.xf, out);
            if (lane == 0) {
#pragma unroll
              for (int i = 0; i < R; ++i)
                if (rr + i < n) track(r0 + rr + i, f2bf(out[i]));
            }
          }
        });
      }
    }
    STEP_MARK(NL, 2);
    if (ok) {
      // CTA-best over the threads that tracked rows, then publish and let the last CTA reduce
      float* cv_s = S.att;
      int* ci_s = (int*)(S.att + NT);
      cv_s[tid] = bv;
      ci_s[tid] = bi;
      csync();
      if (tid == 0) {
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int t = 0; t < NT; ++t)
          if (better(cv_s[t], ci_s[t], v, i)) {
            v = cv_s[t];
            i = ci_s[t];
          }
        float* cv = (float*)m.cand;
        int* cix = (int*)m.cand + 1024;
        cv[blockIdx.x] = v;
        cix[blockIdx.x] = i;
        __threadfence();
        const int old = atomicAdd((int*)&sync[SYNC_ARGMAX], 1);
        if (old == N - 1) {
          __threadfence();
          float bv2 = -INFINITY;
          int bi2 = 0x7fffffff;
          for (int c = 0; c < N; ++c) {
            const float cvv = __ldcg(cv + c);
            const int cii = __ldcg(cix + c);
            if (better(cvv, cii, bv2, bi2)) {
              bv2 = cvv;
              bi2 = cii;
            }
          }
          m.tok[0] = bi2;
          if (p.advance) {
            const int np = pos + 1;
            m.pos[0] = np;
            m.seq_len[0] = np + 1;
            m.kv_off[0] = np * 2 * HDIM;
          }
          // every CTA has read every word of this token: the next token's epoch
          sync[SYNC_ARGMAX] = 0;
          sync[SYNC_EPOCH] = (int)(tok_epoch + 1u);
          __threadfence();
        }
      }
    }
  }
  // after an early exit: stop the producer and wait for the copies in flight
  if (tid == 0 && vrs.consumed < P.total) {
    vrs.abort = 1;
    drain(S, vrs.consumed, vrs.issued);
  }
}

// ---------------------------------------------------------------------------
// weight packing for the step kernel: 16-row tiles in mma.sync A-fragment order
// ---------------------------------------------------------------------------
// Rows [0, M) of a plain wire (row stride `stride` bytes: K_full int8, then K_full/G
// bf16 scales), columns [col0, col0 + K) -> tiles: per 32-column block kb, 32 lanes x
// 16 bytes {row g, cols 4t..4t+3 | row g+8, same | row g, cols 16+4t.. | row g+8, same}
// (g = lane / 4, t = lane % 4); then per group 8 x {scale row g, scale row g + 8}.
// Rows past M are zero.
__global__ void pack_tiles_kernel(const uint8_t* wire, long long stride, int M, int K_full, int col0, int K, int G,
                                  uint8_t* out) {
  const int KB = K / 32, KG = K / G;
  const int ntile = (M + TR - 1) / TR;
  const int tw = KB * 32 * 4 + KG * 8;  // 4-byte words per tile
  const long long words = (long long)ntile * tw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / tw);
    const int w = (int)(i - (long long)t * tw);
    uint32_t v = 0;
    if (w < KB * 128) {
      const int kb = w / 128, r4 = w - kb * 128, lane = r4 >> 2, reg = r4 & 3;
      const int row = t * TR + (lane >> 2) + ((reg & 1) ? 8 : 0);
      const int col = col0 + kb * 32 + (lane & 3) * 4 + ((reg & 2) ? 16 : 0);
      if (row < M) v = *(const uint32_t*)(wire + (size_t)row * stride + col);
    } else {
      const int s = w - KB * 128, gl = s / 8, g = s - gl * 8;
      const size_t soff = (size_t)K_full + 2 * (size_t)(col0 / G + gl);
      const int r0 = t * TR + g, r1 = r0 + 8;
      const uint32_t lo = r0 < M ? *(const uint16_t*)(wire + (size_t)r0 * stride + soff) : 0u;
      const uint32_t hi = r1 < M ? *(const uint16_t*)(wire + (size_t)r1 * stride + soff) : 0u;
      v = lo | (hi << 16);
    }
    *(uint32_t*)(out + (long long)i * 4) = v;
  }
}

template <int G, int GQ>
static int launch(const Kp& p, int grid, size_t smem, cudaStream_t st) {
  auto fn = qwen3_step_kernel<G, GQ>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
    attr[dev] = true;
  }
  void* args[] = {(void*)&p};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)fn, dim3(grid), dim3(NT + 32), args, smem, st);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 step launch: %s", cudaGetErrorString(e));
  iron_count_launch();
  return IRON_OK;
}

static int grid_for(const iron_qwen3_model* m) {
  (void)m;
  return iron_num_sms();
}

// host mirror of the per-CTA weight chunks: the largest of any CTA
static size_t max_chunk(const iron_qwen3_model* m, int N, int lm_rows) {
  const int G = m->group, GQ = m->Hq / m->Hkv, D = m->D;
  size_t mx = std::max((size_t)KVP * 4 * HDIM, m->lm_w8 ? (size_t)LMT * tileb(D, G) : (size_t)lm_rows * D * 2);
  for (int c = 0; c < N; ++c) {
    Plan P;
    plan_tiles(*m, c, N, P);
    mx = std::max(mx, (size_t)P.qnt * tileb(D, G));
    mx = std::max(mx, (size_t)P.ont * tileb(m->Hq * HDIM, G));
    mx = std::max(mx, (size_t)P.gnt * tileb(D, G));
    mx = std::max(mx, (size_t)P.dns * tileb(m->FF / DSL, G));
  }
  return mx;
}

static int max_tiles(const iron_qwen3_model* m, int N) {
  int mx = 0;
  for (int c = 0; c < N; ++c) {
    Plan P;
    plan_tiles(*m, c, N, P);
    mx = std::max(std::max(mx, P.qnt), std::max(P.ont, std::max(P.gnt, P.dns)));
  }
  return mx;
}

static int validate(const iron_qwen3_model* m, int grid) {
  IRON_REQUIRE(m != nullptr, IRON_ERR_ARG, "qwen3 step: null model");
  IRON_REQUIRE(m->HD == HDIM, IRON_ERR_UNSUPPORTED, "qwen3 step: head_dim %d (supported: 128)", m->HD);
  IRON_REQUIRE(m->Hkv >= 1 && m->Hq % m->Hkv == 0, IRON_ERR_ARG, "qwen3 step: Hq=%d, Hkv=%d", m->Hq, m->Hkv);
  const int GQ = m->Hq / m->Hkv;
  IRON_REQUIRE(GQ == 1 || GQ == 2 || GQ == 4, IRON_ERR_UNSUPPORTED, "qwen3 step: GQA group %d", GQ);
  IRON_REQUIRE(m->group == 32 || m->group == 64 || m->group == 128, IRON_ERR_ARG, "qwen3 step: group %d",
               m->group);
  IRON_REQUIRE(m->D % m->group == 0 && m->FF % m->group == 0 && (GQ * HDIM) % m->group == 0 && m->D % 256 == 0 &&
                   m->FF % 32 == 0 && m->D <= 4 * NT,
               IRON_ERR_ARG, "qwen3 step: D=%d FF=%d must be multiples of the group, D a multiple of 256 (<= %d)",
               m->D, m->FF, 4 * NT);
  IRON_REQUIRE(m->FF <= 12288 && m->FF % (DSL * 128) == 0, IRON_ERR_UNSUPPORTED,
               "qwen3 step: intermediate size %d (a multiple of %d up to 12288)", m->FF, DSL * 128);
  IRON_REQUIRE(grid >= m->Hkv && (grid + m->Hkv - 1) / m->Hkv <= GMAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: %d CTAs cannot form %d KV-head groups of at most %d", grid, m->Hkv, GMAX);
  IRON_REQUIRE(max_tiles(m, grid) <= NTMAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: more than %d row tiles of one projection per CTA", NTMAX);
  for (int c = 0; c < grid; ++c) {  // the down slices of a CTA are staged side by side
    Plan P;
    plan_tiles(*m, c, grid, P);
    IRON_REQUIRE(P.dns <= DSL, IRON_ERR_UNSUPPORTED, "qwen3 step: %d down slices on one CTA", P.dns);
  }
  IRON_REQUIRE(grid <= 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: grid %d exceeds the candidate slots", grid);
  IRON_REQUIRE(m->layers && m->final_norm && m->embed && m->angles && m->kv && m->x && m->attn_ws && m->cand &&
                   m->tok && m->pos && m->seq_len && m->kv_off && m->sync,
               IRON_ERR_ARG, "qwen3 step: null buffer in the model descriptor");
  return IRON_OK;
}

}  // namespace qstep
}  // namespace iron

using namespace iron::qstep;

#ifdef IRON_STEP_PROFILE
extern "C" int iron_qwen3_step_profile_buffer(void* buf) {
  return cudaMemcpyToSymbol(g_step_prof, &buf, sizeof(buf)) == cudaSuccess ? IRON_OK : IRON_ERR_CUDA;
}
#endif

extern "C" int iron_qwen3_sync_words(const iron_qwen3_model* m) {
  (void)m;
  return SYNC_WORDS;
}
extern "C" int64_t iron_qwen3_cand_bytes(void) { return 1024 * 8; }
extern "C" int iron_qwen3_grid(const iron_qwen3_model* m) { return grid_for(m); }

extern "C" int64_t iron_qwen3_attn_ws_bytes(const iron_qwen3_model* m) {
  if (!m || m->Hkv < 1 || m->Hq % m->Hkv != 0) return 0;
  const int GQ = m->Hq / m->Hkv;
  const int64_t words = (int64_t)DSL * m->D + (int64_t)m->Hkv * (GQ + 2) * HDIM / 2 +
                        (int64_t)m->Hkv * GMAX * GQ * (HDIM + 2) + (int64_t)m->Hq * HDIM / 2 + m->D / 2 +
                        m->FF / 2;
  return words * 8;
}

extern "C" int iron_qwen3_sync_reset(const iron_qwen3_model* m, void* stream) {
  IRON_REQUIRE(m && m->sync && m->attn_ws, IRON_ERR_ARG, "qwen3 sync reset: null");
  cudaError_t e = cudaMemsetAsync(m->sync, 0, (size_t)SYNC_WORDS * 4, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(m->attn_ws, 0, (size_t)iron_qwen3_attn_ws_bytes(m), (cudaStream_t)stream);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 sync reset: %s", cudaGetErrorString(e));
  return IRON_OK;
}

extern "C" int64_t iron_qwen3_tiles_bytes(int M, int K, int group) {
  if (M < 1 || K < 32 || K % 32 || group < 32 || K % group) return -1;
  return (int64_t)((M + TR - 1) / TR) * (int64_t)tileb(K, group);
}

extern "C" int iron_qwen3_pack_tiles(const void* wire, int64_t row_stride, int M, int K_full, int col0, int K,
                                     int group, void* out, void* stream) {
  IRON_REQUIRE(wire && out, IRON_ERR_ARG, "pack_tiles: null pointer");
  IRON_REQUIRE(M >= 1 && K >= 32 && K % 32 == 0 && (group == 32 || group == 64 || group == 128) && K % group == 0 &&
                   col0 >= 0 && col0 % group == 0 && col0 + K <= K_full && K_full % group == 0 &&
                   row_stride >= K_full + 2 * (K_full / group) && row_stride % 4 == 0,
               IRON_ERR_ARG, "pack_tiles: M=%d K_full=%d col0=%d K=%d group=%d stride=%lld", M, K_full, col0, K, group,
               (long long)row_stride);
  IRON_REQUIRE(iron_aligned(wire, 4) && iron_aligned(out, 16), IRON_ERR_ALIGN, "pack_tiles: misaligned pointer");
  const long long words = iron_qwen3_tiles_bytes(M, K, group) / 4;
  const int blocks = (int)std::min<long long>((words + 255) / 256, 8192);
  pack_tiles_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)wire, (long long)row_stride, M, K_full,
                                                               col0, K, group, (uint8_t*)out);
  return iron_check_launch("pack_tiles_kernel");
}

// Launch parameters of one model descriptor on one device.  A decode loop passes the
// same descriptor every token and the checks walk every CTA's plan (~15 us of host
// time), so the last checked descriptor is kept per host thread and compared bytewise.
struct Prepared {
  bool valid = false;
  int dev = -1, grid = 0;
  size_t smem = 0;
  iron_qwen3_model m;
  Kp p;
};

static int prepare(const iron_qwen3_model* m, Prepared& out) {
  const int grid = grid_for(m);
  int rc = validate(m, grid);
  if (rc) return rc;
  const int GQ = m->Hq / m->Hkv;
  Kp& p = out.p;
  p.m = *m;
  p.embed_input = 0;
  p.advance = 0;
  p.kmax = std::max(std::max(m->D, m->Hq * HDIM), m->FF);
  p.hbn = std::max(std::max(m->FF, m->Hq * HDIM), (GQ + 2) * HDIM);
  const size_t fixed = fixed_smem(p.kmax, p.hbn, m->D, m->group, GQ, m->n_layers);
  IRON_REQUIRE(fixed + 64 * 1024 <= (size_t)SMEM_MAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: %zu bytes of fixed shared memory leave no room for the weight ring", fixed);
  p.ring = (int)(((size_t)SMEM_MAX - fixed) & ~(size_t)1023);
  p.lm_rows = 4 * NWARP;  // one pass of the lm_head row loop per chunk (64 KB of bf16 rows)
  const size_t mc = max_chunk(m, grid, p.lm_rows);
  IRON_REQUIRE(mc <= (size_t)p.ring, IRON_ERR_UNSUPPORTED,
               "qwen3 step: a %zu-byte weight share exceeds the %d-byte ring (model too large for one launch)", mc,
               p.ring);
  IRON_REQUIRE((m->group == 32 && (GQ == 1 || GQ == 2 || GQ == 4)) || (m->group == 64 && (GQ == 2 || GQ == 4)) ||
                   (m->group == 128 && (GQ == 2 || GQ == 4)),
               IRON_ERR_UNSUPPORTED, "qwen3 step: group %d with GQA group %d", m->group, GQ);
  out.grid = grid;
  out.smem = (size_t)p.ring + fixed;
  out.m = *m;
  return IRON_OK;
}

static int prepared_for(const iron_qwen3_model* m, const Prepared*& P) {
  static thread_local Prepared cache;
  IRON_REQUIRE(m != nullptr, IRON_ERR_ARG, "qwen3 step: null model");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  if (!(cache.valid && cache.dev == dev && std::memcmp(&cache.m, m, sizeof(*m)) == 0)) {
    cache.valid = false;
    Prepared fresh;
    const int rc = prepare(m, fresh);
    if (rc) return rc;
    fresh.dev = dev;
    fresh.valid = true;
    cache = fresh;
  }
  P = &cache;
  return IRON_OK;
}

extern "C" int iron_qwen3_decode_step(const iron_qwen3_model* m, int embed_input, int advance, void* stream) {
  const Prepared* P = nullptr;
  const int rc = prepared_for(m, P);
  if (rc) return rc;
  Kp p = P->p;
  p.embed_input = embed_input;
  p.advance = advance;
  const int GQ = m->Hq / m->Hkv;
  cudaStream_t st = (cudaStream_t)stream;
#define IRON_STEP_CASE(g, gq) \
  if (m->group == g && GQ == gq) return launch<g, gq>(p, P->grid, P->smem, st);
  IRON_STEP_CASE(32, 2) IRON_STEP_CASE(32, 1) IRON_STEP_CASE(32, 4) IRON_STEP_CASE(64, 2) IRON_STEP_CASE(64, 4)
  IRON_STEP_CASE(128, 2) IRON_STEP_CASE(128, 4)
#undef IRON_STEP_CASE
  return iron_set_error(IRON_ERR_UNSUPPORTED, "qwen3 step: group %d with GQA group %d", m->group, GQ);
}

extern "C" int iron_qwen3_step_host(const iron_qwen3_model* m, const int32_t* host_in, int32_t* host_out,
                                    int embed_input, void* stream) {
  IRON_REQUIRE(m && host_in && host_out && m->tok && m->pos && m->sync, IRON_ERR_ARG,
               "qwen3 host step: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  if (m->pos == m->tok + 1) {  // token and position side by side: one 8-byte copy
    e = cudaMemcpyAsync(m->tok, host_in, 8, cudaMemcpyHostToDevice, st);
  } else {
    e = cudaMemcpyAsync(m->tok, host_in, 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, host_in + 1, 4, cudaMemcpyHostToDevice, st);
  }
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 host step: input copy: %s", cudaGetErrorString(e));
  const int rc = iron_qwen3_decode_step(m, embed_input, 0, stream);
  if (rc) return rc;
  e = cudaMemcpyAsync(host_out, m->tok, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(host_out + 1, m->sync + SYNC_ERR, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 host step: %s", cudaGetErrorString(e));
  if (host_out[1] != 0)
    return iron_set_error(IRON_ERR_TIMEOUT,
                          "qwen3 step aborted on a bounded device wait (code %d); iron_qwen3_sync_reset clears it",
                          host_out[1]);
  return IRON_OK;
}
