// One greedy Qwen3 decode token (batch 1) as ONE persistent cooperative kernel.
//
// Why one kernel.  At batch 1 a decode token streams ~0.9 GB (weights, KV) but
// each projection is only a few microseconds of HBM time, so the token is bound
// by the latency of the dependency chain between projections, not by bandwidth.
// The kernel keeps that chain short:
//
//   - One CTA per SM.  The CTAs form Hkv KV-head groups of about N / Hkv CTAs.
//     Group h computes the q/k/v rows of KV head h (QKV rows are taken in head
//     order), runs head h's attention with one split of the positions per CTA,
//     merges the splits and multiplies the merged heads by head h's column block
//     of Wo.  Inside the attention block only the group's own CTAs wait for one
//     another.
//   - The O and down projections are split along K: O by KV head, down by the
//     slice of gate/up rows a CTA computed itself, so the SwiGLU output never
//     leaves the CTA.  Partial sums are float64 and meet through float64 atomics
//     in per-layer accumulators.
//   - Per layer that leaves two grid barriers (after O, after down) and two
//     group barriers (after QKV, after the attention splits).
//   - Weights do not depend on activations, so each CTA's weight share streams
//     through a shared-memory ring by cp.async.bulk (CTA-local copies).  A producer
//     warp issues the copies as far ahead as the ring allows (about a layer), so
//     issuing never sits on the compute path.  The attention KV range is
//     prefetched to L2 one phase early.
//
// Weight layouts.  QKV and gate/up rows use the native wire (tile_m = 1, row
// [K int8 | K/G bf16 scales]).  O uses wo_heads: for each KV head h the rows of Wo
// restricted to h's GQ*HD columns, [GQ*HD int8 | GQ*HD/G bf16 | pad to 16 bytes].
// Down uses wd_cols: int8 [FF/4][D][4] (four consecutive K columns of one row in a
// 32-bit word) and scales [FF/G][D] bf16, so a CTA's K slice is contiguous.
// iron_qwen3_pack_wo_heads / iron_qwen3_pack_wd_cols build both from the wires.
//
// Arithmetic.  The stages use the device arithmetic of the per-operator entry
// points: activations staged as exact int16 block floating point (hi + lo words),
// dp2a sums per 16 (or 4) columns, float64 accumulation, the golden RMSNorm form
// for the QKV input, q/k and the final norm, the kernel form for the MLP norm, and
// the same bf16 roundings between stages.  The K-split partial sums meet in
// float64, so a projection output equals the unsplit float64 sum up to float64
// summation order before its single bf16 rounding.
//
// Synchronisation.  Barriers are int32 counters in global memory whose targets
// grow with the layer; the last CTA of the token resets them.  Every wait is
// bounded by %globaltimer: on timeout the CTA records an error code and returns;
// the other CTAs see the code in their own waits and return too.  In-flight bulk
// copies are drained (bounded) before a CTA exits.
#include <algorithm>

#include "common.cuh"

namespace iron {
namespace qstep {

// 8 compute warps and one producer warp (168 registers a thread, no spills; more warps
// cap registers at 128 and spill in the inner loops)
constexpr int NT = 256, NWARP = NT / 32;
constexpr int HDIM = 128;        // head_dim of the step kernel
constexpr int NMB = 16;          // ring slots (chunks in flight at most)
constexpr int GMAX = 24;         // most CTAs in one KV-head group (attention splits)
constexpr int XREP = 4;          // down-projection accumulator replicas: KV-head group h adds into
                                 // replica h % XREP (atomics to one address serialise in L2)
constexpr int SLICE_MAX = 32;    // widest down-projection K slice of one CTA
constexpr int PIECE = 32768;     // bytes per cp.async.bulk instruction
constexpr int SMEM_MAX = 227 * 1024;
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;  // per wait

// sync words (the G2 counters follow the Hkv G1 counters)
enum { SYNC_B1 = 0, SYNC_ERR = 1, SYNC_ARGMAX = 2, SYNC_B2 = 3, SYNC_PARITY = 4, SYNC_EPOCH = 5, SYNC_G1 = 8 };
enum { ERR_BARRIER = 1, ERR_COPY = 2, ERR_INPUT = 3 };
// chunk kinds of a layer, in stream order; the lm_head chunks follow the last layer
enum { CK_QKV = 0, CK_O = 1, CK_GU = 2, CK_D = 3 };

struct Kp {
  iron_qwen3_model m;
  int embed_input, advance;
  int ring;     // ring bytes
  int lm_rows;  // lm_head rows per chunk
  int kst;      // staging length max(D, GQ*HD)
};

__host__ __device__ inline int rowb(int K, int G) { return K + 2 * (K / G); }
__host__ __device__ inline int rowb_heads(int GQ, int G) { return (rowb(GQ * HDIM, G) + 15) & ~15; }

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier, bulk copies, acquire loads, timer
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
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// float64 add to global memory with no value returned (the accumulators only need the sum)
__device__ __forceinline__ void red_add(double* p, double v) {
  asm volatile("red.global.add.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed(const int32_t* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flagged words: (epoch << 32 | data) written by one 64-bit store, so a reader that
// finds the epoch it waits for also has the data; no fence, counter or poll of a
// separate word sits between producer and consumer.  Every word is rewritten each
// token with a larger epoch; the buffers are zeroed with the sync words.
__device__ __forceinline__ void ll_put(unsigned long long* p, uint32_t data, uint32_t epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | data;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_ld(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// the data of word p once it carries `epoch` (bounded: on timeout or a set error word
// *bad is set and 0 returned)
__device__ __forceinline__ uint32_t ll_get(const unsigned long long* p, uint32_t epoch, int32_t* sync, int& bad) {
  unsigned long long w = ll_ld(p);
  if ((uint32_t)(w >> 32) == epoch) return (uint32_t)w;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    w = ll_ld(p);
    if ((uint32_t)(w >> 32) == epoch) return (uint32_t)w;
    if ((it & 15) == 15) {
      if (ld_relaxed(&sync[SYNC_ERR]) != 0) break;
      if (gtimer() - t0 > TIMEOUT_NS) {
        atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_BARRIER);
        break;
      }
    }
  }
  bad = 1;
  return 0;
}

__device__ __forceinline__ unsigned ld_acquire(const int32_t* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
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
#define STEP_CLK(row, k)                                                                                          \
  do {                                                                                                            \
    if (threadIdx.x == 0 && g_step_prof) g_step_prof[((size_t)blockIdx.x * 64 + (row)) * 32 + (k)] = clock64(); \
  } while (0)
#else
#define STEP_MARK(row, k) \
  do {                    \
  } while (0)
#define STEP_CLK(row, k) \
  do {                   \
  } while (0)
#endif

// barrier of the NT compute threads only (the producer warp runs on its own)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

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
  int q0, q1;           // group-local QKV rows: q rows of the group's GQ heads, then k, then v
  int o0, o1;           // O rows (against head h's column block)
  int u0, u1;           // gate/up rows / 4 = down-projection K slice / 4
  int ga, nsg;          // first scale group of the slice, scale groups it touches
  int hlo, hhi, hnch;   // lm_head rows, chunks
  int total;            // chunks of the token
  uint32_t bytes[4];    // chunk bytes per layer kind
};

__device__ Plan make_plan(const Kp& p) {
  const iron_qwen3_model& m = p.m;
  Plan P;
  const int N = gridDim.x, c = blockIdx.x, G = m.group, GQ = m.Hq / m.Hkv, D = m.D;
  int c0, c1;
  head_group(c, N, m.Hkv, P.h, c0, c1);
  P.gi = c - c0;
  P.gsz = c1 - c0;
  part((GQ + 2) * HDIM, P.gi, P.gsz, P.q0, P.q1);
  part(D, P.gi, P.gsz, P.o0, P.o1);
  part(m.FF / 4, c, N, P.u0, P.u1);
  const int k0 = 4 * P.u0, k1 = 4 * P.u1;
  P.ga = k0 / G;
  P.nsg = k1 > k0 ? (k1 - 1) / G - P.ga + 1 : 0;
  P.bytes[CK_QKV] = (uint32_t)(P.q1 - P.q0) * rowb(D, G);
  P.bytes[CK_O] = (uint32_t)(P.o1 - P.o0) * rowb_heads(GQ, G);
  P.bytes[CK_GU] = 2u * (uint32_t)(k1 - k0) * rowb(D, G);
  P.bytes[CK_D] = (uint32_t)(P.u1 - P.u0) * D * 4 + (uint32_t)P.nsg * D * 2;
  part(m.V, c, N, P.hlo, P.hhi);
  P.hnch = (P.hhi - P.hlo + p.lm_rows - 1) / p.lm_rows;
  P.total = 4 * m.n_layers + P.hnch;
  return P;
}

// source row of group-local QKV row r of KV head h (q rows of heads h*GQ.., k, v)
__device__ __forceinline__ int qkv_src_row(int r, int h, int GQ, int Hq, int Hkv) {
  if (r < GQ * HDIM) return h * GQ * HDIM + r;
  if (r < (GQ + 1) * HDIM) return Hq * HDIM + h * HDIM + (r - GQ * HDIM);
  return (Hq + Hkv) * HDIM + h * HDIM + (r - (GQ + 1) * HDIM);
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
  uint16_t* xhi;   // [kst] bf16 bits, then int16 hi words
  uint16_t* xlo;   // [kst] norm weights before the BFP pass, then lo words
  float* xs;       // [kst / 16] block factors
  uint16_t* sx;    // [D] residual x (bf16 bits)
  uint16_t* sx1;   // [D] residual x1
  float* xf;       // [D] final normed x (bf16 lm_head path)
  float* ghv;      // [SLICE_MAX] this CTA's SwiGLU outputs
  uint16_t* dh;    // [SLICE_MAX] their int16 hi words
  uint16_t* dl;    // [SLICE_MAX] lo words
  float* att;      // attention scratch
  float* mst;      // [GMAX][GQ][HD + 2] the split partials of this CTA's KV head
  iron_qwen3_layer* lay;  // [n_layers] copy of the layer pointer table
  double* red;     // [32]
  uint64_t* mbar;  // [NMB + 1]
  RingState* rs;
  int* flag;       // [8]; flag[4] holds the down slice's block factor (float bits)
};

__host__ __device__ inline size_t att_floats(int GQ) {
  return (size_t)GQ * HDIM + 2 * HDIM + (size_t)NWARP * GQ * (HDIM + 2);
}

// bytes of everything but the ring (carve's layout: 17 arrays, each rounded up to 16 bytes)
__host__ __device__ inline size_t fixed_smem(int kst, int D, int GQ, int n_layers) {
  size_t o = 32 * 8 + (NMB + 1) * 8 + sizeof(RingState) + 8 * 4;
  o += (size_t)kst * 4 + (size_t)(kst / 16) * 4;
  o += (size_t)D * 2 * 2 + (size_t)D * 4;
  o += SLICE_MAX * 4 + SLICE_MAX * 2 * 2;
  o += att_floats(GQ) * 4 + (size_t)GMAX * GQ * (HDIM + 2) * 4;
  o += (size_t)n_layers * sizeof(iron_qwen3_layer);
  return o + 17 * 16 + 64;
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
  s.red = (double*)take(32 * 8);
  s.mbar = (uint64_t*)take((NMB + 1) * 8);  // ring slots, then the split-merge copy
  s.rs = (RingState*)take((sizeof(RingState) + 15) & ~(size_t)15);
  s.flag = (int*)take(8 * 4);
  s.xhi = (uint16_t*)take((size_t)p.kst * 2);
  s.xlo = (uint16_t*)take((size_t)p.kst * 2);
  s.xs = (float*)take((size_t)(p.kst / 16) * 4);
  s.sx = (uint16_t*)take((size_t)p.m.D * 2);
  s.sx1 = (uint16_t*)take((size_t)p.m.D * 2);
  s.xf = (float*)take((size_t)p.m.D * 4);
  s.ghv = (float*)take(SLICE_MAX * 4);
  s.dh = (uint16_t*)take(SLICE_MAX * 2);
  s.dl = (uint16_t*)take(SLICE_MAX * 2);
  s.att = (float*)take(att_floats(GQ) * 4);
  s.mst = (float*)take((size_t)GMAX * GQ * (HDIM + 2) * 4);
  s.lay = (iron_qwen3_layer*)take((size_t)p.m.n_layers * sizeof(iron_qwen3_layer));
  return s;
}

// ---------------------------------------------------------------------------
// the chunk stream: per layer QKV, O, gate/up, down; then the lm_head
// ---------------------------------------------------------------------------
struct Seg {
  const uint8_t* src;
  uint32_t bytes;
};

// segments of chunk i, copied back to back into one ring slot; returns their count
__device__ int chunk_segs(const Kp& p, const Plan& P, const Smem& S, int i, Seg (&sg)[3]) {
  const iron_qwen3_model& m = p.m;
  const int G = m.group, D = m.D, GQ = m.Hq / m.Hkv;
  const int lay = i >> 2;
  if (lay >= m.n_layers) {
    const int j = i - 4 * m.n_layers;
    const int r0 = P.hlo + j * p.lm_rows, r1 = min(P.hhi, r0 + p.lm_rows);
    const uint32_t rb = m.lm_w8 ? rowb(D, G) : D * 2;
    const uint8_t* base = m.lm_w8 ? (const uint8_t*)m.lm_w8 : (const uint8_t*)m.embed;
    sg[0] = {base + (size_t)r0 * rb, (uint32_t)(r1 - r0) * rb};
    return 1;
  }
  const iron_qwen3_layer& L = S.lay[lay];
  switch (i & 3) {
    case CK_QKV: {
      const uint32_t rb = rowb(D, G);
      int n = 0, r = P.q0;
      while (r < P.q1) {  // split at the q / k / v boundaries of the group-local order
        const int lim = r < GQ * HDIM ? GQ * HDIM : (r < (GQ + 1) * HDIM ? (GQ + 1) * HDIM : (GQ + 2) * HDIM);
        const int e = min(P.q1, lim);
        sg[n++] = {(const uint8_t*)L.wqkv + (size_t)qkv_src_row(r, P.h, GQ, m.Hq, m.Hkv) * rb,
                   (uint32_t)(e - r) * rb};
        r = e;
      }
      return n;
    }
    case CK_O: {
      const uint32_t rb = rowb_heads(GQ, G);
      sg[0] = {(const uint8_t*)L.wo_heads + ((size_t)P.h * D + P.o0) * rb, (uint32_t)(P.o1 - P.o0) * rb};
      return 1;
    }
    case CK_GU: {
      const uint32_t rb = rowb(D, G);
      const size_t off = (size_t)(4 * P.u0) * rb;
      const uint32_t bytes = (uint32_t)(4 * (P.u1 - P.u0)) * rb;
      sg[0] = {(const uint8_t*)L.wg + off, bytes};
      sg[1] = {(const uint8_t*)L.wu + off, bytes};
      return 2;
    }
    default: {
      sg[0] = {(const uint8_t*)L.wd_cols + (size_t)P.u0 * D * 4, (uint32_t)(P.u1 - P.u0) * D * 4};
      sg[1] = {(const uint8_t*)L.wd_col_scales + (size_t)P.ga * D * 2, (uint32_t)P.nsg * D * 2};
      return 2;
    }
  }
}

__device__ __forceinline__ uint32_t chunk_bytes(const Kp& p, const Plan& P, int i) {
  if ((i >> 2) < p.m.n_layers) {  // a switch, not an indexed array: P stays in registers
    switch (i & 3) {
      case CK_QKV: return P.bytes[CK_QKV];
      case CK_O: return P.bytes[CK_O];
      case CK_GU: return P.bytes[CK_GU];
      default: return P.bytes[CK_D];
    }
  }
  const int j = i - 4 * p.m.n_layers;
  const int r0 = P.hlo + j * p.lm_rows, r1 = min(P.hhi, r0 + p.lm_rows);
  return (uint32_t)(r1 - r0) * (p.m.lm_w8 ? rowb(p.m.D, p.m.group) : p.m.D * 2);
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
// for its copies in flight.
// (inlined: a call that takes P or S by address would move the compute threads' copies
// to local memory, which the small L1 left beside 227 KB of shared memory does not keep)
__device__ __forceinline__ void producer(const Kp& p, const Plan& P, const Smem& S, int32_t* sync) {
  volatile RingState& rs = *S.rs;
  const uint32_t R = (uint32_t)p.ring;
  unsigned long long head = 0;
  bool stop = false;
  for (int i = 0; i < P.total && !stop; ++i) {
    const uint32_t bytes = chunk_bytes(p, P, i);
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
    Seg sg[3];
    const int ns = chunk_segs(p, P, S, i, sg);
    uint8_t* dst = S.ring + (uint32_t)(start % R);
    fence_proxy_async();  // the compute threads' reads of this space happen before the async writes
    mbar_expect(&S.mbar[sl], bytes);
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      if (s >= ns) break;
      for (uint32_t o = 0; o < sg[s].bytes; o += PIECE)
        bulk_g2s(dst + o, sg[s].src + o, min((uint32_t)PIECE, sg[s].bytes - o), &S.mbar[sl]);
      dst += sg[s].bytes;
    }
    rs.issued = i + 1;
  }
  if (stop) drain(S, rs.consumed, rs.issued);
}

// ---------------------------------------------------------------------------
// bounded waits (thread 0)
// ---------------------------------------------------------------------------
__device__ bool wait_count(int32_t* sync, int word, unsigned target) {
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    if (ld_acquire(&sync[word]) >= target) return true;
    if (ld_acquire(&sync[SYNC_ERR]) != 0) return false;
    if ((it & 63) == 63 && gtimer() - t0 > TIMEOUT_NS) {
      atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_BARRIER);
      return false;
    }
  }
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
// activation staging (the arithmetic of gemv_w8_kernel's prologue)
// ---------------------------------------------------------------------------
// In place: xhi holds the bf16 bits of K values -> int16 hi words; xlo lo words;
// xs the group factors.  Eight lanes per quant group.
__device__ __forceinline__ void bfp_stage_p(uint16_t* xhi, uint16_t* xlo, float* xs, int K, int G) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane >> 3, sl = lane & 7, per = G / 8;
  const int ng = K / G;
  for (int g0 = wid * 4; g0 < ng; g0 += NWARP * 4) {
    const int gi = g0 + sub;
    const bool valid = gi < ng;
    uint16_t* base = xhi + (size_t)(valid ? gi : 0) * G + sl * per;
    float v[16];
    float mx = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (e < per) {
        v[e] = valid ? bf2f(base[e]) : 0.f;
        mx = fmaxf(mx, fabsf(v[e]));
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    float sc, inv;
    bfp_scale(mx, sc, inv);
    if (valid) {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (e < per) {
          const float t = v[e] * sc;
          const int hi = __float2int_rn(t);
          base[e] = (uint16_t)(int16_t)hi;
          xlo[(base - xhi) + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
        }
      if (sl == 0) xs[gi] = inv;
    }
  }
}

__device__ __forceinline__ void bfp_stage(const Smem& S, int K, int G) { bfp_stage_p(S.xhi, S.xlo, S.xs, K, G); }

// RMSNorm of the bf16 bits in `src` (shared) with the weight bits already in xlo
// -> bf16 bits in xhi (mode 0 kernel form, 1 golden form); `outf` (shared)
// receives the values as floats when non-null.
__device__ __forceinline__ void stage_norm_p(uint16_t* xhi, const uint16_t* xlo, double* red, const uint16_t* src, int K,
                                         float eps, int mode, float* outf) {
  double ss = 0.0;
  for (int i = threadIdx.x; i < K; i += NT) ss += rms_sq(bf2f(src[i]), mode);
  ss = csum_d(ss, red);
  const RmsCoef rc = rms_coef(ss, K, eps, mode);
  for (int i = threadIdx.x; i < K; i += NT) {
    const uint16_t o = f2bf(rms_apply(bf2f(src[i]), bf2f(xlo[i]), rc));
    xhi[i] = o;
    if (outf) outf[i] = bf2f(o);
  }
}

__device__ __forceinline__ void stage_norm(const Smem& S, const uint16_t* src, int K, float eps, int mode, float* outf) {
  stage_norm_p(S.xhi, S.xlo, S.red, src, K, eps, mode, outf);
}

// dst[i] = bf16(src[i] + bf16(sum over the nrep replicas acc[r*D + i])) over the D
// residual rows, replicas summed in a fixed order; every accumulator load of a thread
// is issued before the first store (D <= 4 * NT)
template <int NREP>
__device__ __forceinline__ void resid_add(uint16_t* dst, const uint16_t* src, const double* acc, int D) {
  constexpr int MAXV = 4;
  double v[MAXV][NREP];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * NT;
#pragma unroll
    for (int r = 0; r < NREP; ++r) v[k][r] = i < D ? __ldcg(acc + (size_t)r * D + i) : 0.0;
  }
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * NT;
    double a = v[k][0];
#pragma unroll
    for (int r = 1; r < NREP; ++r) a += v[k][r];
    if (i < D) dst[i] = f2bf(bf2f(src[i]) + rbf_d(a));
  }
}

// A layer-phase prologue in one pass.  With acc: x = bf16(src + bf16(sum of the NREP
// accumulator replicas)) into dst (every load of a thread issued first); without: x is
// dst as it stands.  Then RMSNorm(x) * w (w's bf16 bits already in xlo; mode 0 kernel
// form, 1 golden form) goes straight into exact int16 block floating point (xhi, xlo,
// xs), eight lanes per quant group: the arithmetic of stage_norm + bfp_stage with one
// shared-memory pass.  outf (shared) gets the normalised values, trace (global) gets x.
template <int G, int NREP>
__device__ __forceinline__ void prologue(const Smem& S, uint16_t* dst, const uint16_t* src, const double* acc, int D,
                                         float eps, int mode, float* outf, uint16_t* trace) {
  constexpr int MAXV = 4;  // D <= 4 * NT
  double ss = 0.0;
  if (acc) {
    double v[MAXV][NREP];
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      const int i = threadIdx.x + k * NT;
#pragma unroll
      for (int r = 0; r < NREP; ++r) v[k][r] = i < D ? __ldcg(acc + (size_t)r * D + i) : 0.0;
    }
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      const int i = threadIdx.x + k * NT;
      double a = v[k][0];
#pragma unroll
      for (int r = 1; r < NREP; ++r) a += v[k][r];
      if (i < D) {
        const uint16_t x = f2bf(bf2f(src[i]) + rbf_d(a));
        dst[i] = x;
        ss += rms_sq(bf2f(x), mode);
        if (trace) trace[i] = x;
      }
    }
  } else {
    for (int i = threadIdx.x; i < D; i += NT) {
      ss += rms_sq(bf2f(dst[i]), mode);
      if (trace) trace[i] = dst[i];
    }
  }
  ss = csum_d(ss, S.red);  // its barriers also publish dst
  const RmsCoef rc = rms_coef(ss, D, eps, mode);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane >> 3, sl = lane & 7, per = G / 8;
  const int ng = D / G;
  for (int g0 = wid * 4; g0 < ng; g0 += NWARP * 4) {
    const int gi = g0 + sub;
    const bool valid = gi < ng;
    const int base = (valid ? gi : 0) * G + sl * per;
    float v[16];
    float mx = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (e < per) {
        v[e] = valid ? bf2f(f2bf(rms_apply(bf2f(dst[base + e]), bf2f(S.xlo[base + e]), rc))) : 0.f;
        mx = fmaxf(mx, fabsf(v[e]));
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    float sc, inv;
    bfp_scale(mx, sc, inv);
    if (valid) {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (e < per) {
          if (outf) outf[base + e] = v[e];
          const float t = v[e] * sc;
          const int hi = __float2int_rn(t);
          S.xhi[base + e] = (uint16_t)(int16_t)hi;
          S.xlo[base + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
        }
      if (sl == 0) S.xs[gi] = inv;
    }
  }
  csync();
}

// K bf16 values (K % 8 == 0, read-only data) into shared memory with 16-byte loads
__device__ __forceinline__ void load_ro(uint16_t* dst, const uint16_t* src, int K) {
  for (int i = threadIdx.x; i < (K >> 3); i += NT) ((uint4*)dst)[i] = __ldg(((const uint4*)src) + i);
}

// ---------------------------------------------------------------------------
// int8 rows from shared memory: LPR lanes per row, 16 columns a lane per step, NR rows
// (2NR for gate/up pairs) per lane group at once: sum_k q*s*x exactly as
// gemv_w8_kernel with LO staging and float64 accumulation.  The 16-column dp2a sums
// run as two chains of four so that their latencies overlap.
// ---------------------------------------------------------------------------
template <int G, int NR, int LPR>
__device__ __forceinline__ void rows_dot(const uint8_t* const (&rp)[NR], int K, const Smem& S, double (&out)[NR]) {
  const int sub = threadIdx.x & (LPR - 1);
  double acc[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) acc[i] = 0.0;
#pragma unroll 2
  for (int c = sub; c < (K >> 4); c += LPR) {
    const int g = (c * 16) / G;
    const uint4 xa = *(const uint4*)(S.xhi + c * 16), xb = *(const uint4*)(S.xhi + c * 16 + 8);
    const uint4 la = *(const uint4*)(S.xlo + c * 16), lb = *(const uint4*)(S.xlo + c * 16 + 8);
    const float xsc = S.xs[g];
    uint4 w[NR];
    float sv[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      w[i] = *(const uint4*)(rp[i] + c * 16);
      sv[i] = bf2f(((const uint16_t*)(rp[i] + K))[g]);
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      int a0 = __dp2a_lo((int)xa.x, (int)w[i].x, 0), a1 = __dp2a_hi((int)xa.y, (int)w[i].x, 0);
      a0 = __dp2a_lo((int)xa.z, (int)w[i].y, a0);
      a1 = __dp2a_hi((int)xa.w, (int)w[i].y, a1);
      a0 = __dp2a_lo((int)xb.x, (int)w[i].z, a0);
      a1 = __dp2a_hi((int)xb.y, (int)w[i].z, a1);
      a0 = __dp2a_lo((int)xb.z, (int)w[i].w, a0);
      a1 = __dp2a_hi((int)xb.w, (int)w[i].w, a1);
      int l0 = __dp2a_lo((int)la.x, (int)w[i].x, 0), l1 = __dp2a_hi((int)la.y, (int)w[i].x, 0);
      l0 = __dp2a_lo((int)la.z, (int)w[i].y, l0);
      l1 = __dp2a_hi((int)la.w, (int)w[i].y, l1);
      l0 = __dp2a_lo((int)lb.x, (int)w[i].z, l0);
      l1 = __dp2a_hi((int)lb.y, (int)w[i].z, l1);
      l0 = __dp2a_lo((int)lb.z, (int)w[i].w, l0);
      l1 = __dp2a_hi((int)lb.w, (int)w[i].w, l1);
      const long long t = (long long)(a0 + a1) * 32768 + (l0 + l1);
      acc[i] = fma((double)t, (double)(sv[i] * xsc) * (1.0 / 32768.0), acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    double v = acc[i];
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    out[i] = v;
  }
}

// The n rows of one chunk (rb bytes each; with PAIR the n gate rows, then the n up
// rows).  The NG = NT/LPR lane groups take rows b + rg + i*NG of each block of
// NG*R rows; every lane of a warp runs the same trip count (the shuffles need it).
template <int G, int R, int LPR, bool PAIR, class Epi>
__device__ void chunk_rows(const uint8_t* wb, int n, int rb, int K, const Smem& S, Epi epi) {
  constexpr int NR = PAIR ? 2 * R : R;
  constexpr int NG = NT / LPR;
  const int rg = threadIdx.x / LPR, sub = threadIdx.x & (LPR - 1);
  for (int b = 0; b < n; b += NG * R) {
    const uint8_t* rp[NR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int r = min(b + rg + i * NG, n - 1);
      rp[i] = wb + (size_t)r * rb;
      if (PAIR) rp[R + i] = wb + (size_t)(n + r) * rb;
    }
    double out[NR];
    rows_dot<G, NR, LPR>(rp, K, S, out);  // every lane of the group holds all the sums
#pragma unroll
    for (int i = 0; i < R; ++i)  // lane i of the group finishes row i, the epilogues side by side
      if (sub == i && b + rg + i * NG < n) epi(b + rg + i * NG, out[i], PAIR ? out[R + i] : 0.0);
  }
}

// one row-block width R per call site keeps a single copy of the row loop in the kernel
template <int G, int LPR, int R, bool PAIR, class Epi>
__device__ __forceinline__ void chunk_gemv(const uint8_t* wb, int n, int rb, int K, const Smem& S, Epi epi) {
  chunk_rows<G, R, LPR, PAIR>(wb, n, rb, K, S, epi);
}

// bf16 rows with float32 activations: the lm_head arithmetic of gemv_bf16_kernel
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

// the same with this lane's activations held in registers: xr[k] = xf[(lane + 32k)*8 ..]
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

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// attention: KV head h, split s of ns over the positions; writes the split's
// partial (o, m, l) per query head to the workspace slot [h][s]
// ---------------------------------------------------------------------------
// raw: the flagged q/k/v words of this layer (epoch `ep`); returns false when a wait
// for them gave up
template <int GQ>
__device__ bool attention_split(const Kp& p, const Smem& S, int layer, int h, int s, int ns, int P,
                                const unsigned long long* raw, uint32_t ep) {
  const iron_qwen3_model& m = p.m;
  constexpr int PER = HDIM / 32;
  constexpr int U = 4;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int L = P + 1;
  const int chunk = (L + ns - 1) / ns;
  const int start = min(L, s * chunk), end = min(L, start + chunk);
  float* qf = S.att;                   // [GQ][HD]
  float* kt = qf + GQ * HDIM;          // [HD]
  float* vt = kt + HDIM;               // [HD]
  float* part = vt + HDIM;             // [NWARP][GQ][HD+2]
  uint16_t* head = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
  const uint16_t* ang = m.angles + (size_t)P * HDIM;
  const bool owner = P >= start && P < end;
  // the first K/V positions do not depend on q/k: their loads go out before the norms
  auto load = [&](int j0, uint2 (&kk)[U], uint2 (&vv)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = min(j0 + u, end - 1);
      if (j != P) {
        const uint16_t* kr = head + (size_t)j * 2 * HDIM + lane * PER;
        kk[u] = ldg_stream8(kr);
        vv[u] = ldg_stream8(kr + HDIM);
      }
    }
  };
  uint2 kc[U], vc[U], kn[U], vn[U];
  int j0 = start + wid * U;
  if (j0 < end) load(j0, kc, vc);
  // per-head q/k RMSNorm (golden form) + RoPE and the v copy: qk_norm_rope_kv_kernel's arithmetic
  int bad = 0;
  if (threadIdx.x == 0) S.flag[6] = 0;
  csync();
  for (int t = wid; t < GQ + 2; t += NWARP) {
    if (t == GQ + 1) {
      const unsigned long long* vs = raw + (size_t)(m.Hq + m.Hkv + h) * HDIM + lane * 4;
      uint32_t b[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) b[e] = ll_get(vs + e, ep, m.sync, bad);
      const uint2 v = make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
      vt[lane * 4 + 0] = bf_lo(v.x);
      vt[lane * 4 + 1] = bf_hi(v.x);
      vt[lane * 4 + 2] = bf_lo(v.y);
      vt[lane * 4 + 3] = bf_hi(v.y);
      if (owner) ((uint2*)(head + (size_t)P * 2 * HDIM + HDIM))[lane] = v;
      continue;
    }
    const bool isq = t < GQ;
    const int hh = isq ? h * GQ + t : m.Hq + h;
    const unsigned long long* src = raw + (size_t)hh * HDIM;
    const uint16_t* nw = isq ? S.lay[layer].qn : S.lay[layer].kn;
    float v[PER], wv[PER], cs[PER], sn[PER];
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      const int i = lane + 32 * j;
      v[2 * j] = bf2f(ll_get(src + i, ep, m.sync, bad));
      v[2 * j + 1] = bf2f(ll_get(src + i + HDIM / 2, ep, m.sync, bad));
      wv[2 * j] = bf2f(__ldg(nw + i));
      wv[2 * j + 1] = bf2f(__ldg(nw + i + HDIM / 2));
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
      if (!isq && owner) {
        head[(size_t)P * 2 * HDIM + i] = o1;
        head[(size_t)P * 2 * HDIM + i + HDIM / 2] = o2;
      }
    }
  }
  if (bad) S.flag[6] = 1;
  csync();
  if (S.flag[6]) return false;
  STEP_MARK(layer, 14);
  // flash decoding over [start, end): the online softmax of attn_split_kernel, with the
  // next group of positions loaded while the current one is reduced
  const float scale = 1.4426950408889634f / sqrtf((float)HDIM);
  float q[GQ][PER];
#pragma unroll
  for (int g = 0; g < GQ; ++g)
#pragma unroll
    for (int e = 0; e < PER; ++e) q[g][e] = qf[g * HDIM + lane * PER + e];
  float mm[GQ], ll[GQ], o[GQ][PER];
#pragma unroll
  for (int g = 0; g < GQ; ++g) {
    mm[g] = -INFINITY;
    ll[g] = 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) o[g][e] = 0.f;
  }
  for (; j0 < end; j0 += NWARP * U) {
    const int jn = j0 + NWARP * U;
    if (jn < end) load(jn, kn, vn);
    float kf[U][PER], vf[U][PER];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = min(j0 + u, end - 1);
      if (j == P) {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          kf[u][e] = kt[lane * PER + e];
          vf[u][e] = vt[lane * PER + e];
        }
      } else {
        kf[u][0] = bf_lo(kc[u].x);
        kf[u][1] = bf_hi(kc[u].x);
        kf[u][2] = bf_lo(kc[u].y);
        kf[u][3] = bf_hi(kc[u].y);
        vf[u][0] = bf_lo(vc[u].x);
        vf[u][1] = bf_hi(vc[u].x);
        vf[u][2] = bf_lo(vc[u].y);
        vf[u][3] = bf_hi(vc[u].y);
      }
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      float sv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) d = fmaf(q[g][e], kf[u][e], d);
        sv[u] = warp_sum(d) * scale;
        if (j0 + u >= end) sv[u] = -INFINITY;
      }
      float mn = mm[g];
#pragma unroll
      for (int u = 0; u < U; ++u) mn = fmaxf(mn, sv[u]);
      const float corr = exp2f(mm[g] - mn);
      float ls = ll[g] * corr;
#pragma unroll
      for (int e = 0; e < PER; ++e) o[g][e] *= corr;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pu = exp2f(sv[u] - mn);
        ls += pu;
#pragma unroll
        for (int e = 0; e < PER; ++e) o[g][e] = fmaf(pu, vf[u][e], o[g][e]);
      }
      ll[g] = ls;
      mm[g] = mn;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      kc[u] = kn[u];
      vc[u] = vn[u];
    }
  }
  // merge the warps; write this split's partial per head
#pragma unroll
  for (int g = 0; g < GQ; ++g) {
    float* pw = part + (wid * GQ + g) * (HDIM + 2);
#pragma unroll
    for (int e = 0; e < PER; ++e) pw[lane * PER + e] = o[g][e];
    if (lane == 0) {
      pw[HDIM] = mm[g];
      pw[HDIM + 1] = ll[g];
    }
  }
  csync();
  float* ws = m.attn_ws + ((size_t)(h * GMAX + s) * GQ) * (HDIM + 2);
  for (int t = threadIdx.x; t < GQ * HDIM; t += NT) {
    const int g = t / HDIM, d = t - g * HDIM;
    float M = -INFINITY;
    for (int w = 0; w < NWARP; ++w) M = fmaxf(M, part[(w * GQ + g) * (HDIM + 2) + HDIM]);
    float oo = 0.f, lsum = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NWARP; ++w) {
        const float* pw = part + (w * GQ + g) * (HDIM + 2);
        const float f = exp2f(pw[HDIM] - M);
        oo = fmaf(pw[d], f, oo);
        lsum = fmaf(pw[HDIM + 1], f, lsum);
      }
    }
    ws[g * (HDIM + 2) + d] = oo;
    if (d == 0) {
      ws[g * (HDIM + 2) + HDIM] = M;
      ws[g * (HDIM + 2) + HDIM + 1] = lsum;
    }
  }
  return true;
}

// Merge the ns split partials of KV head h (attn_combine_kernel's arithmetic) into
// bf16 bits in xhi[0, GQ*HD).  The partials are contiguous in the workspace and
// come in with one bulk copy; `use` counts the calls (mbarrier phase).
template <int GQ>
__device__ bool merge_splits(const Kp& p, const Smem& S, int h, int ns, int use) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    const float* base = p.m.attn_ws + (size_t)h * GMAX * GQ * (HDIM + 2);
    const uint32_t bytes = (uint32_t)ns * GQ * (HDIM + 2) * 4;
    // the partials were written through the generic proxy by the group's CTAs
    asm volatile("fence.proxy.async.global;" ::: "memory");
    mbar_expect(&S.mbar[NMB], bytes);
    bulk_g2s(S.mst, base, bytes, &S.mbar[NMB]);
    S.flag[3] = wait_slot(&S.mbar[NMB], p.m.sync, (uint32_t)(use & 1)) ? 1 : 0;
    if (!S.flag[3]) {  // leaving early: let the copy land first (bounded)
      const unsigned long long t0 = gtimer();
      while (!mbar_test(&S.mbar[NMB], (uint32_t)(use & 1)) && gtimer() - t0 < 20ull * 1000 * 1000) {
      }
    }
  }
  csync();
  if (!S.flag[3]) return false;
  for (int t = tid; t < GQ * HDIM; t += NT) {
    const int g = t / HDIM, d = t - g * HDIM;
    const float* ps = S.mst + g * (HDIM + 2);
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, ps[sp * GQ * (HDIM + 2) + HDIM]);
    float oo = 0.f, lsum = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < ns; ++sp) {
        const float* q = ps + sp * GQ * (HDIM + 2);
        const float f = exp2f(q[HDIM] - M);
        oo = fmaf(q[d], f, oo);
        lsum = fmaf(q[HDIM + 1], f, lsum);
      }
    }
    S.xhi[t] = f2bf(lsum > 0.f ? oo / lsum : 0.f);
  }
  return true;
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
  const int tid = threadIdx.x;
  const int N = gridDim.x, D = m.D, NL = m.n_layers;
  const Plan P = make_plan(p);
  const int pos = m.pos[0];
  // a position outside the cache or a token outside the vocabulary: record and leave
  // before touching memory (every CTA takes the same decision)
  if (pos < 0 || pos >= m.max_seq || (p.embed_input && (m.tok[0] < 0 || m.tok[0] >= m.V))) {
    if (tid == 0) atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_INPUT);
    return;
  }
  // projection accumulators: two sets of [NL][O, down][D] float64 that alternate by
  // token; this token zeroes the other set for the next one
  const int parity = __ldcg((const int*)&sync[SYNC_PARITY]) & 1;
  const uint32_t tok_epoch = (uint32_t)__ldcg((const int*)&sync[SYNC_EPOCH]);
  double* acc_base = (double*)((uint8_t*)m.attn_ws + (size_t)m.Hkv * GMAX * GQ * (HDIM + 2) * 4);
  const size_t lstride = (size_t)(1 + XREP) * D;  // accumulator doubles per layer
  double* acc = acc_base + (size_t)parity * NL * lstride;
  // flagged q/k/v words of the current layer, after the accumulators
  unsigned long long* raw_ll = (unsigned long long*)(acc_base + (size_t)2 * NL * lstride);
  if (tid < NT) {
    double* other = acc_base + (size_t)(parity ^ 1) * NL * lstride;
    for (size_t i = (size_t)blockIdx.x * NT + tid; i < NL * lstride; i += (size_t)N * NT) other[i] = 0.0;
    // the layer pointer table, read once
    const int nw = NL * (int)(sizeof(iron_qwen3_layer) / 8);
    for (int i = tid; i < nw; i += NT) ((unsigned long long*)S.lay)[i] = __ldg(((const unsigned long long*)m.layers) + i);
  }
  if (tid == 0) {
    for (int i = 0; i <= NMB; ++i) mbar_init(&S.mbar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    S.rs->tail = 0;
    S.rs->issued = S.rs->consumed = S.rs->abort = 0;
  }
  __syncthreads();  // the last barrier of all NT + 32 threads
  if (tid >= NT) {
    if (tid == NT) producer(p, P, S, sync);
    return;
  }
  // layer-0 input: the token's embedding row, or the hidden state given in x
  load_ro(S.sx, p.embed_input ? m.embed + (size_t)m.tok[0] * D : m.x, D);
  load_ro(S.xlo, S.lay[0].norm1, D);
  csync();  // the prologue reads these rows across threads

  bool ok = true;
  // consume chunk i: fn(buffer) once its copy landed, then release its space
  volatile RingState& vrs = *S.rs;
  auto consume = [&](int i, auto&& fn) -> bool {
    const int sl = i % NMB;
    if (tid == 0) S.flag[2] = wait_slot(&S.mbar[sl], sync, (uint32_t)((i / NMB) & 1)) ? 1 : 0;
    csync();
    if (!S.flag[2]) return false;
    if ((i >> 2) < NL) STEP_MARK(i >> 2, 16 + (i & 3));
    fn(S.ring + vrs.slot[sl]);
    csync();
    if ((i >> 2) < NL) STEP_MARK(i >> 2, 20 + (i & 3));
    if (tid == 0) {
      fence_proxy_async();
      vrs.tail = vrs.end[sl];
      vrs.consumed = i + 1;
    }
    return true;
  };
  auto arrive = [&](int word) {
    csync();
    if (tid == 0) {
      __threadfence();
      atomicAdd((unsigned*)&sync[word], 1u);
    }
  };
  auto wait = [&](int word, unsigned target) -> bool {
    if (tid == 0) S.flag[0] = wait_count(sync, word, target) ? 1 : 0;
    csync();
    return S.flag[0] != 0;
  };

  const int h = P.h, gsz = P.gsz;
  const int k0 = 4 * P.u0, w = 4 * (P.u1 - P.u0);
  for (int layer = 0; layer < NL && ok; ++layer) {
    const iron_qwen3_layer& Lw = S.lay[layer];
    double* oacc = acc + (size_t)layer * lstride;
    double* xacc = oacc + (size_t)D * (1 + h % XREP);  // this KV-head group's replica
    const int c0 = 4 * layer;
    const uint32_t ep = tok_epoch * (uint32_t)NL + (uint32_t)layer + 1u;  // this layer's flag value
    STEP_MARK(layer, 0);
    STEP_CLK(layer, 28);
    // ---- QKV: x = bf16(x1 + bf16(down)), hn = RMSNorm_golden(x, norm1), raw = bf16(Wqkv @ hn) ----
    if (layer > 0) {
      if (!(ok = wait(SYNC_B1, (unsigned)layer * N))) break;
      STEP_MARK(layer, 1);
    }
    prologue<G, XREP>(S, S.sx, S.sx1, layer > 0 ? acc + (size_t)(layer - 1) * lstride + D : nullptr, D, m.eps, 1,
                      nullptr, (m.trace && blockIdx.x == 0) ? m.trace + (size_t)layer * D : nullptr);
    STEP_MARK(layer, 24);
    STEP_MARK(layer, 25);
    STEP_MARK(layer, 2);
    ok = consume(c0 + CK_QKV, [&](const uint8_t* wb) {
      chunk_gemv<G, 32, 4, false>(wb, P.q1 - P.q0, rowb(D, G), D, S, [&](int r, double a, double) {
        ll_put(raw_ll + qkv_src_row(P.q0 + r, h, GQ, m.Hq, m.Hkv), f2bf((float)a), ep);
      });
    });
    if (!ok) break;
    STEP_MARK(layer, 3);
    if (tid == 0) {  // this CTA's KV range of this layer, ahead of the attention
      const int L = pos + 1, chunk = (L + gsz - 1) / gsz;
      const int st = min(L, P.gi * chunk), en = min(min(L, st + chunk), pos);
      if (en > st) {
        const uint16_t* hb = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
        prefetch_l2(hb + (size_t)st * 2 * HDIM, (uint32_t)(en - st) * 4 * HDIM);
      }
    }
    STEP_MARK(layer, 4);
    // ---- attention: KV head h, split gi of gsz (its q/k/v rows arrive as flagged words) ----
    if (!(ok = attention_split<GQ>(p, S, layer, h, P.gi, gsz, pos, raw_ll, ep))) break;
    STEP_MARK(layer, 5);
    arrive(SYNC_G1 + m.Hkv + h);
    if (!(ok = wait(SYNC_G1 + m.Hkv + h, (unsigned)(layer + 1) * gsz))) break;
    STEP_MARK(layer, 6);
    // ---- O (head h's column block): oacc += Wo[:, head h] @ attn[head h] ----
    if (!(ok = merge_splits<GQ>(p, S, h, gsz, layer))) break;
    csync();
    STEP_MARK(layer, 15);
    bfp_stage(S, GQ * HDIM, G);
    csync();
    STEP_MARK(layer, 7);
    ok = consume(c0 + CK_O, [&](const uint8_t* wb) {
      chunk_gemv<G, GQ * HDIM / 16 < 32 ? GQ * HDIM / 16 : 32, 4, false>(wb, P.o1 - P.o0, rowb_heads(GQ, G), GQ * HDIM, S,
                               [&](int r, double a, double) { red_add(oacc + P.o0 + r, a); });
    });
    if (!ok) break;
    STEP_MARK(layer, 8);
    load_ro(S.xlo, Lw.norm2, D);
    arrive(SYNC_B2);
    if (!(ok = wait(SYNC_B2, (unsigned)(layer + 1) * N))) break;
    STEP_MARK(layer, 9);
    // ---- gate/up: x1 = bf16(x + bf16(O)), hf = RMSNorm_kernel(x1, norm2),
    //      gh = bf16(silu_tanh(bf16(Wg@hf)) * bf16(Wu@hf)) for this CTA's slice ----
    prologue<G, 1>(S, S.sx1, S.sx, oacc, D, m.eps, 0, nullptr, nullptr);
    STEP_MARK(layer, 26);
    STEP_MARK(layer, 10);
    ok = consume(c0 + CK_GU, [&](const uint8_t* wb) {
      chunk_gemv<G, 32, 3, true>(wb, w, rowb(D, G), D, S, [&](int r, double g, double u) {
        S.ghv[r] = rbf(silu_tanh_bf16(rbf_d(g)) * rbf_d(u));
      });
    });
    if (!ok) break;
    STEP_MARK(layer, 11);
    // the slice as one exact int16 block (hi + lo words)
    if (tid < 32) {
      float mx = 0.f;
      for (int j = tid; j < w; j += 32) mx = fmaxf(mx, fabsf(S.ghv[j]));
      mx = warp_max(mx);
      float sc, inv;
      bfp_scale(mx, sc, inv);
      for (int j = tid; j < w; j += 32) {
        const float t = S.ghv[j] * sc;
        const int hi = __float2int_rn(t);
        S.dh[j] = (uint16_t)(int16_t)hi;
        S.dl[j] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
      }
      if (tid == 0) S.flag[4] = __float_as_int(inv);
    }
    csync();
    STEP_MARK(layer, 12);
    // ---- down (this CTA's K slice): xacc += Wd[:, k0:k0+w] @ gh[k0:k0+w] ----
    ok = consume(c0 + CK_D, [&](const uint8_t* wb) {
      const uint32_t* wq = (const uint32_t*)wb;
      const uint16_t* wsc = (const uint16_t*)(wb + (size_t)w * D);
      const uint32_t* xh = (const uint32_t*)S.dh;
      const uint32_t* xl = (const uint32_t*)S.dl;
      const float inv = __int_as_float(S.flag[4]);
      // words j < jb1 belong to the slice's first scale group, j < jb2 to its second,
      // the rest to its third (a 32-column slice touches at most two groups of 32)
      const int nw4 = w >> 2;
      const int jb1 = (min(w, (P.ga + 1) * G - k0)) >> 2, jb2 = (min(w, (P.ga + 2) * G - k0)) >> 2;
      constexpr int RPT = 4;  // rows per thread and pass, their loads overlapped
      for (int r0 = tid; r0 < D; r0 += NT * RPT) {
        int ah[RPT][3], al[RPT][3];
#pragma unroll
        for (int q = 0; q < RPT; ++q)
#pragma unroll
          for (int e = 0; e < 3; ++e) ah[q][e] = al[q][e] = 0;
#pragma unroll
        for (int j = 0; j < SLICE_MAX / 4; ++j) {
          if (j < nw4) {
            const int h0 = (int)xh[2 * j], h1 = (int)xh[2 * j + 1], l0 = (int)xl[2 * j], l1 = (int)xl[2 * j + 1];
            const int e = j < jb1 ? 0 : (j < jb2 ? 1 : 2);
#pragma unroll
            for (int q = 0; q < RPT; ++q) {
              const int r = r0 + q * NT;
              const int wv = r < D ? (int)wq[(size_t)j * D + r] : 0;
              const int dh = __dp2a_hi(h1, wv, __dp2a_lo(h0, wv, 0));
              const int dl = __dp2a_hi(l1, wv, __dp2a_lo(l0, wv, 0));
              ah[q][0] += e == 0 ? dh : 0;
              ah[q][1] += e == 1 ? dh : 0;
              ah[q][2] += e == 2 ? dh : 0;
              al[q][0] += e == 0 ? dl : 0;
              al[q][1] += e == 1 ? dl : 0;
              al[q][2] += e == 2 ? dl : 0;
            }
          }
        }
#pragma unroll
        for (int q = 0; q < RPT; ++q) {
          const int r = r0 + q * NT;
          if (r >= D) continue;
          double a = 0.0;
#pragma unroll
          for (int e = 0; e < 3; ++e)
            if (e < P.nsg) {
              const long long t = (long long)ah[q][e] * 32768 + al[q][e];
              a = fma((double)t, (double)(bf2f(wsc[(size_t)e * D + r]) * inv) * (1.0 / 32768.0), a);
            }
          red_add(xacc + r, a);
        }
      }
    });
    if (!ok) break;
    STEP_MARK(layer, 13);
    load_ro(S.xlo, layer + 1 < NL ? S.lay[layer + 1].norm1 : m.final_norm, D);
    arrive(SYNC_B1);
  }

  STEP_MARK(NL, 0);
  if (ok) ok = wait(SYNC_B1, (unsigned)NL * N);
  STEP_MARK(NL, 1);
  STEP_CLK(NL, 29);
  if (ok) {
    // ---- final: x = bf16(x1 + bf16(down)), RMSNorm (golden) + lm_head + greedy argmax ----
    prologue<G, XREP>(S, S.sx, S.sx1, acc + (size_t)(NL - 1) * lstride + D, D, m.eps, 1, S.xf,
                      blockIdx.x == 0 ? m.x : nullptr);
    if (m.trace && blockIdx.x == 0)
      for (int i = tid; i < D; i += NT) m.trace[(size_t)NL * D + i] = S.sx[i];
    const int lane = tid & 31, wid = tid >> 5;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const int rbh = m.lm_w8 ? rowb(D, G) : D * 2;
    auto track = [&](int idx, uint16_t o) {
      if (m.logits) m.logits[idx] = o;
      if (better(bf2f(o), idx, bv, bi)) {
        bv = bf2f(o);
        bi = idx;
      }
    };
    float xr[4][8];  // this lane's activations for the D == 1024 bf16 rows
    if (D == 1024) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) xr[k][e] = S.xf[(lane + 32 * k) * 8 + e];
    }
    for (int j = 0; j < P.hnch && ok; ++j) {
      const int r0 = P.hlo + j * p.lm_rows, n = min(P.hhi, r0 + p.lm_rows) - r0;
      ok = consume(4 * NL + j, [&](const uint8_t* wb) {
        if (m.lm_w8) {
          chunk_gemv<G, 32, 4, false>(wb, n, rbh, D, S, [&](int r, double a, double) { track(r0 + r, f2bf((float)a)); });
        } else {
          constexpr int R = 4;
          for (int rr = wid * R; rr < n; rr += NWARP * R) {
            const uint8_t* rp[R];
#pragma unroll
            for (int i = 0; i < R; ++i) rp[i] = wb + (size_t)min(rr + i, n - 1) * rbh;
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
        }
      });
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
          // every CTA has passed every wait of this token: reset the counters and
          // hand the other accumulator set to the next token
          sync[SYNC_B1] = 0;
          sync[SYNC_B2] = 0;
          for (int k = 0; k < 2 * m.Hkv; ++k) sync[SYNC_G1 + k] = 0;
          sync[SYNC_ARGMAX] = 0;
          sync[SYNC_PARITY] = parity ^ 1;
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
// weight packing for the step kernel
// ---------------------------------------------------------------------------
// wo_heads[h][r] = [wo[r, h*GQ*HD : (h+1)*GQ*HD] int8 | its GQ*HD/G bf16 scales | 0 pad]
__global__ void pack_wo_heads_kernel(const uint8_t* wire, int D, int QD, int Hkv, int G, uint8_t* out) {
  const int GQH = QD / Hkv, rb_in = rowb(QD, G), rb_out = rowb_heads(GQH / HDIM, G);
  const long long total = (long long)Hkv * D * rb_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i % rb_out);
    const long long hr = i / rb_out;
    const int r = (int)(hr % D), h = (int)(hr / D);
    const uint8_t* row = wire + (size_t)r * rb_in;
    uint8_t v = 0;
    if (b < GQH)
      v = row[h * GQH + b];
    else if (b < GQH + 2 * (GQH / G))
      v = row[QD + 2 * (h * (GQH / G)) + (b - GQH)];
    out[i] = v;
  }
}

// wd_cols[k/4][r][k%4] = wd[r, k]; wd_col_scales[g][r] = the scale of wd row r, group g
__global__ void pack_wd_cols_kernel(const uint8_t* wire, int D, int FF, int G, uint8_t* q, uint16_t* s) {
  const int rb = rowb(FF, G);
  const long long nq = (long long)FF * D, ns = (long long)(FF / G) * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nq + ns;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < nq) {
      const int e = (int)(i & 3);
      const long long jr = i >> 2;
      const int r = (int)(jr % D), j = (int)(jr / D);
      q[i] = wire[(size_t)r * rb + 4 * j + e];
    } else {
      const long long k = i - nq;
      const int r = (int)(k % D), g = (int)(k / D);
      s[k] = ((const uint16_t*)(wire + (size_t)r * rb + FF))[g];
    }
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

// host mirror of the per-CTA chunk sizes: the largest chunk of any CTA
static size_t max_chunk(const iron_qwen3_model* m, int N, int lm_rows) {
  const int G = m->group, GQ = m->Hq / m->Hkv, D = m->D;
  size_t mx = (size_t)lm_rows * (m->lm_w8 ? rowb(D, G) : D * 2);
  for (int c = 0; c < N; ++c) {
    int h, c0, c1, lo, hi;
    head_group(c, N, m->Hkv, h, c0, c1);
    part((GQ + 2) * HDIM, c - c0, c1 - c0, lo, hi);
    mx = std::max(mx, (size_t)(hi - lo) * rowb(D, G));
    part(D, c - c0, c1 - c0, lo, hi);
    mx = std::max(mx, (size_t)(hi - lo) * rowb_heads(GQ, G));
    part(m->FF / 4, c, N, lo, hi);
    const int k0 = 4 * lo, k1 = 4 * hi;
    const int nsg = k1 > k0 ? (k1 - 1) / G - k0 / G + 1 : 0;
    mx = std::max(mx, (size_t)2 * (k1 - k0) * rowb(D, G));
    mx = std::max(mx, (size_t)(hi - lo) * D * 4 + (size_t)nsg * D * 2);
  }
  return mx;
}

static int validate(const iron_qwen3_model* m, int grid) {
  IRON_REQUIRE(m != nullptr, IRON_ERR_ARG, "qwen3 step: null model");
  IRON_REQUIRE(m->HD == HDIM, IRON_ERR_UNSUPPORTED, "qwen3 step: head_dim %d (supported: 128)", m->HD);
  IRON_REQUIRE(m->Hkv >= 1 && m->Hq % m->Hkv == 0, IRON_ERR_ARG, "qwen3 step: Hq=%d, Hkv=%d", m->Hq, m->Hkv);
  const int GQ = m->Hq / m->Hkv;
  IRON_REQUIRE(GQ == 1 || GQ == 2 || GQ == 4 || GQ == 8, IRON_ERR_UNSUPPORTED, "qwen3 step: GQA group %d", GQ);
  IRON_REQUIRE(m->group == 32 || m->group == 64 || m->group == 128, IRON_ERR_ARG, "qwen3 step: group %d",
               m->group);
  IRON_REQUIRE(m->D % m->group == 0 && m->FF % m->group == 0 && m->D % 256 == 0 && m->D <= 4096 && m->FF % 4 == 0,
               IRON_ERR_ARG, "qwen3 step: D=%d FF=%d must be multiples of the group and D a multiple of 256 (<= 4096)",
               m->D, m->FF);
  IRON_REQUIRE(grid >= m->Hkv && (grid + m->Hkv - 1) / m->Hkv <= GMAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: %d CTAs cannot form %d KV-head groups of at most %d", grid, m->Hkv, GMAX);
  IRON_REQUIRE(4 * ((m->FF / 4 + grid - 1) / grid) <= SLICE_MAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: down-projection slice wider than %d columns", SLICE_MAX);
  IRON_REQUIRE(m->D <= 4 * NT, IRON_ERR_UNSUPPORTED, "qwen3 step: hidden size %d above %d", m->D, 4 * NT);
  IRON_REQUIRE(grid <= 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: grid %d exceeds the candidate slots", grid);
  IRON_REQUIRE(m->layers && m->final_norm && m->embed && m->angles && m->kv && m->x && m->attn_ws &&
                   m->cand && m->tok && m->pos && m->seq_len && m->kv_off && m->sync,
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

extern "C" int iron_qwen3_sync_words(const iron_qwen3_model* m) { return SYNC_G1 + 2 * (m ? m->Hkv : 64); }
extern "C" int64_t iron_qwen3_cand_bytes(void) { return 1024 * 8; }
extern "C" int iron_qwen3_grid(const iron_qwen3_model* m) { return grid_for(m); }

static int64_t partial_bytes(const iron_qwen3_model* m) {
  return (int64_t)m->Hkv * GMAX * (m->Hq / m->Hkv) * (HDIM + 2) * 4;
}
static int64_t acc_bytes(const iron_qwen3_model* m) { return (int64_t)2 * m->n_layers * (1 + XREP) * m->D * 8; }
static int64_t raw_ll_bytes(const iron_qwen3_model* m) { return (int64_t)(m->Hq + 2 * m->Hkv) * HDIM * 8; }

extern "C" int64_t iron_qwen3_attn_ws_bytes(const iron_qwen3_model* m) {
  if (!m || m->Hkv < 1 || m->Hq % m->Hkv != 0) return 0;
  return partial_bytes(m) + acc_bytes(m) + raw_ll_bytes(m);
}

extern "C" int iron_qwen3_sync_reset(const iron_qwen3_model* m, void* stream) {
  IRON_REQUIRE(m && m->sync && m->attn_ws, IRON_ERR_ARG, "qwen3 sync reset: null");
  cudaError_t e = cudaMemsetAsync(m->sync, 0, (size_t)iron_qwen3_sync_words(m) * 4, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemsetAsync((uint8_t*)m->attn_ws + partial_bytes(m), 0, (size_t)(acc_bytes(m) + raw_ll_bytes(m)),
                        (cudaStream_t)stream);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 sync reset: %s", cudaGetErrorString(e));
  return IRON_OK;
}

extern "C" int64_t iron_qwen3_pack_wo_heads_bytes(int D, int QD, int Hkv, int group) {
  if (D < 1 || Hkv < 1 || group < 1 || QD % (Hkv * HDIM) != 0) return -1;
  return (int64_t)Hkv * D * rowb_heads(QD / Hkv / HDIM, group);
}

extern "C" int iron_qwen3_pack_wo_heads(const void* wo_wire, int D, int QD, int Hkv, int group, void* out,
                                        void* stream) {
  IRON_REQUIRE(wo_wire && out, IRON_ERR_ARG, "pack_wo_heads: null pointer");
  IRON_REQUIRE(D >= 1 && Hkv >= 1 && group >= 16 && QD % (Hkv * HDIM) == 0 && (QD / Hkv) % group == 0,
               IRON_ERR_ARG, "pack_wo_heads: D=%d QD=%d Hkv=%d group=%d", D, QD, Hkv, group);
  const long long total = iron_qwen3_pack_wo_heads_bytes(D, QD, Hkv, group);
  const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
  pack_wo_heads_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)wo_wire, D, QD, Hkv, group,
                                                                  (uint8_t*)out);
  return iron_check_launch("pack_wo_heads_kernel");
}

extern "C" int iron_qwen3_pack_wd_cols(const void* wd_wire, int D, int FF, int group, void* out_q,
                                       uint16_t* out_scales, void* stream) {
  IRON_REQUIRE(wd_wire && out_q && out_scales, IRON_ERR_ARG, "pack_wd_cols: null pointer");
  IRON_REQUIRE(D >= 1 && group >= 4 && FF % 4 == 0 && FF % group == 0, IRON_ERR_ARG,
               "pack_wd_cols: D=%d FF=%d group=%d", D, FF, group);
  const long long total = (long long)FF * D + (long long)(FF / group) * D;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
  pack_wd_cols_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)wd_wire, D, FF, group,
                                                                 (uint8_t*)out_q, out_scales);
  return iron_check_launch("pack_wd_cols_kernel");
}

extern "C" int iron_qwen3_decode_step(const iron_qwen3_model* m, int embed_input, int advance, void* stream) {
  const int grid = grid_for(m);
  int rc = validate(m, grid);
  if (rc) return rc;
  const int GQ = m->Hq / m->Hkv;
  Kp p;
  p.m = *m;
  p.embed_input = embed_input;
  p.advance = advance;
  p.kst = std::max(m->D, GQ * HDIM);
  const size_t fixed = fixed_smem(p.kst, m->D, GQ, m->n_layers);
  IRON_REQUIRE(fixed + 64 * 1024 <= (size_t)SMEM_MAX, IRON_ERR_UNSUPPORTED,
               "qwen3 step: %zu bytes of fixed shared memory leave no room for the weight ring", fixed);
  p.ring = (int)(((size_t)SMEM_MAX - fixed) & ~(size_t)1023);
  p.lm_rows = 4 * NWARP;  // one pass of the lm_head row loop per chunk (64 KB of bf16 rows)
  const size_t mc = max_chunk(m, grid, p.lm_rows);
  IRON_REQUIRE(mc <= (size_t)p.ring, IRON_ERR_UNSUPPORTED,
               "qwen3 step: a %zu-byte weight share exceeds the %d-byte ring (model too large for one launch)", mc,
               p.ring);
  const size_t smem = (size_t)p.ring + fixed;
  cudaStream_t st = (cudaStream_t)stream;
#define IRON_STEP_CASE(g, gq) \
  if (m->group == g && GQ == gq) return launch<g, gq>(p, grid, smem, st);
  IRON_STEP_CASE(32, 2) IRON_STEP_CASE(32, 1) IRON_STEP_CASE(32, 4) IRON_STEP_CASE(32, 8)
  IRON_STEP_CASE(64, 2) IRON_STEP_CASE(64, 4) IRON_STEP_CASE(128, 2) IRON_STEP_CASE(128, 4)
#undef IRON_STEP_CASE
  return iron_set_error(IRON_ERR_UNSUPPORTED, "qwen3 step: group %d with GQA group %d", m->group, GQ);
}
