// One greedy Qwen3 decode token (batch 1) as ONE persistent cooperative kernel.
//
// Layout of the work.  The grid is one CTA per SM.  A token is a sequence of
// phases separated by grid barriers: for every layer QKV -> attention -> O-proj
// -> gate/up -> down, then the lm_head.  In each GEMV phase a CTA owns a
// contiguous range of output rows.  Its weight rows (native wire, tile_m = 1)
// arrive in shared memory by cp.async.bulk (no multicast) into two buffers.
// Copies are issued in a fixed per-CTA chunk order one chunk ahead, so the next
// phase's weights stream in while this phase computes and while the grid waits
// at the barrier; the weights do not depend on the activations.  The attention
// phase's KV range is prefetched to L2 one phase early.
//
// Arithmetic.  Every stage uses the device code of the per-operator entry
// points:
//   - activations staged as exact int16 block floating point (hi + lo words);
//   - dp2a chunk sums with float64 accumulation;
//   - the golden RMSNorm form for the QKV input, q/k and the final norm, and
//     the kernel form for the MLP norm;
//   - the same bf16 stores between stages.
// So the token equals the chained kernels' token up to float64 / float32
// summation order.
//
// Synchronisation.  Grid barriers and the per-KV-head split counters are
// int32 words in global memory.  Every wait is bounded by %globaltimer.  On
// timeout the CTA records an error code and returns; the other CTAs see it and
// return too.  In-flight bulk copies are drained (bounded) before exit.
#include "common.cuh"

namespace iron {
namespace qstep {

constexpr int NT = 256, NWARP = NT / 32;
constexpr int BUF = 48 * 1024;  // bytes per weight buffer (two buffers)
constexpr int HDIM = 128;       // head_dim of the step kernel
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;  // per wait

enum { SYNC_BAR = 0, SYNC_ERR = 1, SYNC_ARGMAX = 2, SYNC_HEAD0 = 3 };
enum { ERR_BARRIER = 1, ERR_COPY = 2, ERR_INPUT = 3 };

constexpr int SMAX = 16;  // most attention splits per KV head

struct Kp {
  iron_qwen3_model m;
  int embed_input, advance, smax, kmax;
};

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
__device__ __forceinline__ unsigned ld_acquire(const int32_t* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ldcg_u16(const uint16_t* p) { return (uint32_t)__ldcg(p); }

// ---------------------------------------------------------------------------
// shared memory
// ---------------------------------------------------------------------------
struct Smem {
  uint8_t* buf[2];
  uint16_t* xhi;  // [kmax] bf16 bits, then int16 hi words
  uint16_t* xlo;  // [kmax]
  float* xs;      // [kmax / 32]
  float* xf;      // [D] lm_head activations (bf16 path)
  float* att;     // attention scratch
  float* mrg;     // split-merge scratch: [Hq][SMAX] weights, [Hq] sums
  iron_qwen3_layer* lay;  // [n_layers] copy of the layer pointer table
  double* red;    // [32]
  uint64_t* mbar; // [2]
  int* flag;      // [4]
};

__device__ Smem carve(uint8_t* base, const Kp& p, int GQ) {
  Smem s;
  size_t o = 0;
  s.buf[0] = base + o;
  o += BUF;
  s.buf[1] = base + o;
  o += BUF;
  s.xhi = (uint16_t*)(base + o);
  o += (size_t)p.kmax * 2;
  s.xlo = (uint16_t*)(base + o);
  o += (size_t)p.kmax * 2;
  s.red = (double*)(base + o);
  o += 32 * 8;
  s.mbar = (uint64_t*)(base + o);
  o += 2 * 8;
  s.flag = (int*)(base + o);
  o += 16;
  s.xs = (float*)(base + o);
  o += (size_t)(p.kmax / 32) * 4;
  s.xf = (float*)(base + o);
  o += (size_t)p.m.D * 4;
  s.att = (float*)(base + o);
  o += (size_t)(GQ * HDIM + 2 * HDIM + NWARP * GQ * (HDIM + 2)) * 4;
  s.mrg = (float*)(base + o);
  o += (size_t)(p.m.Hq * SMAX + p.m.Hq) * 4;
  o = (o + 15) & ~(size_t)15;
  s.lay = (iron_qwen3_layer*)(base + o);
  return s;
}

__host__ __device__ inline size_t smem_bytes(int kmax, int D, int GQ, int Hq, int n_layers) {
  const size_t att = (size_t)(GQ * HDIM + 2 * HDIM + NWARP * GQ * (HDIM + 2)) * 4;
  const size_t mrg = (size_t)(Hq * SMAX + Hq) * 4;
  return 2 * (size_t)BUF + (size_t)kmax * 4 + 32 * 8 + 16 + 16 + (size_t)(kmax / 32) * 4 + (size_t)D * 4 + att + mrg +
         16 + (size_t)n_layers * sizeof(iron_qwen3_layer);
}

// ---------------------------------------------------------------------------
// work partition and the per-CTA chunk sequence
// ---------------------------------------------------------------------------
__device__ __forceinline__ void part(int M, int c, int N, int& lo, int& hi) {
  lo = (int)((long long)M * c / N);
  hi = (int)((long long)M * (c + 1) / N);
}
__device__ __forceinline__ int rowb(int K, int G) { return K + 2 * (K / G); }

enum { PH_QKV = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_D = 4 };

struct Plan {  // identical in every thread of a CTA
  int lo[5], hi[5], rpc[5], nch[5];  // per GEMV phase kind: my rows, rows per chunk, chunks
  int per_layer;                     // chunks per layer
  int hlo, hhi, hrpc, hnch;          // lm_head
  int total;
};

__device__ Plan make_plan(const Kp& p) {
  const iron_qwen3_model& m = p.m;
  Plan P;
  const int G = m.group, N = gridDim.x, c = blockIdx.x;
  const int QKV = (m.Hq + 2 * m.Hkv) * m.HD, QD = m.Hq * m.HD;
  const int Ms[5] = {QKV, 0, m.D, m.FF, m.D};
  const int Ks[5] = {m.D, 0, QD, m.D, m.FF};
  P.per_layer = 0;
  for (int k = 0; k < 5; ++k) {
    if (k == PH_ATT) {
      P.lo[k] = P.hi[k] = P.rpc[k] = P.nch[k] = 0;
      continue;
    }
    part(Ms[k], c, N, P.lo[k], P.hi[k]);
    const int unit = rowb(Ks[k], G) * (k == PH_GU ? 2 : 1);
    P.rpc[k] = BUF / unit;
    P.nch[k] = (P.hi[k] - P.lo[k] + P.rpc[k] - 1) / P.rpc[k];
    P.per_layer += P.nch[k];
  }
  part(m.V, c, N, P.hlo, P.hhi);
  P.hrpc = BUF / (m.lm_w8 ? rowb(m.D, G) : m.D * 2);
  P.hnch = (P.hhi - P.hlo + P.hrpc - 1) / P.hrpc;
  P.total = P.per_layer * m.n_layers + P.hnch;
  return P;
}

struct Chunk {
  int layer, kind, r0, r1;  // kind 5 = lm_head
};

__device__ Chunk chunk_at(const Plan& P, int i, int n_layers) {
  Chunk ch;
  if (i < P.per_layer * n_layers) {
    ch.layer = i / P.per_layer;
    int j = i - ch.layer * P.per_layer;
    int k = 0;
    for (;; ++k) {
      if (k == PH_ATT) continue;
      if (j < P.nch[k]) break;
      j -= P.nch[k];
    }
    ch.kind = k;
    ch.r0 = P.lo[k] + j * P.rpc[k];
    ch.r1 = min(P.hi[k], ch.r0 + P.rpc[k]);
  } else {
    const int j = i - P.per_layer * n_layers;
    ch.layer = n_layers;
    ch.kind = 5;
    ch.r0 = P.hlo + j * P.hrpc;
    ch.r1 = min(P.hhi, ch.r0 + P.hrpc);
  }
  return ch;
}

// thread 0: bulk-copy chunk i into buffer b
__device__ void issue(const Kp& p, const Plan& P, const Smem& S, int i, int b) {
  if (i >= P.total) return;
  const iron_qwen3_model& m = p.m;
  const Chunk ch = chunk_at(P, i, m.n_layers);
  const int G = m.group, n = ch.r1 - ch.r0;
  const uint8_t* src[2] = {nullptr, nullptr};
  uint32_t rb = 0;
  int nsrc = 1;
  if (ch.kind == 5) {
    rb = m.lm_w8 ? rowb(m.D, G) : m.D * 2;
    src[0] = m.lm_w8 ? (const uint8_t*)m.lm_w8 + (size_t)ch.r0 * rb : (const uint8_t*)(m.embed + (size_t)ch.r0 * m.D);
  } else {
    const iron_qwen3_layer& L = S.lay[ch.layer];
    const int QD = m.Hq * m.HD;
    if (ch.kind == PH_QKV) {
      rb = rowb(m.D, G);
      src[0] = (const uint8_t*)L.wqkv + (size_t)ch.r0 * rb;
    } else if (ch.kind == PH_O) {
      rb = rowb(QD, G);
      src[0] = (const uint8_t*)L.wo + (size_t)ch.r0 * rb;
    } else if (ch.kind == PH_GU) {
      rb = rowb(m.D, G);
      src[0] = (const uint8_t*)L.wg + (size_t)ch.r0 * rb;
      src[1] = (const uint8_t*)L.wu + (size_t)ch.r0 * rb;
      nsrc = 2;
    } else {
      rb = rowb(m.FF, G);
      src[0] = (const uint8_t*)L.wd + (size_t)ch.r0 * rb;
    }
  }
  const uint32_t bytes = (uint32_t)n * rb;
  fence_proxy_async();  // generic-proxy use of this buffer happens before the async writes
  mbar_expect(&S.mbar[b], bytes * nsrc);
  for (int s = 0; s < nsrc; ++s) {
    uint8_t* dst = S.buf[b] + (size_t)s * bytes;
    for (uint32_t o = 0; o < bytes; o += 16384u) {
      const uint32_t len = min(16384u, bytes - o);
      bulk_g2s(dst + o, src[s] + o, len, &S.mbar[b]);
    }
  }
}

// L2 prefetch of every weight chunk of `layer` that this CTA will copy
__device__ void prefetch_layer_l2(const Kp& p, const Plan& P, const Smem& S, int layer) {
  if (layer >= p.m.n_layers) return;
  const iron_qwen3_model& m = p.m;
  const iron_qwen3_layer& L = S.lay[layer];
  const int G = m.group, QD = m.Hq * m.HD;
  struct R {
    const void* base;
    int k, K;
  } rs[5] = {{L.wqkv, PH_QKV, m.D}, {L.wo, PH_O, QD}, {L.wg, PH_GU, m.D}, {L.wu, PH_GU, m.D}, {L.wd, PH_D, m.FF}};
  for (int t = 0; t < 5; ++t) {
    const int rb = rowb(rs[t].K, G);
    const int n = P.hi[rs[t].k] - P.lo[rs[t].k];
    if (n <= 0) continue;
    const uint8_t* s = (const uint8_t*)rs[t].base + (size_t)P.lo[rs[t].k] * rb;
    const uint32_t bytes = (uint32_t)n * rb;
    for (uint32_t o = 0; o < bytes; o += 65536u) prefetch_l2(s + o, min(65536u, bytes - o));
  }
}

// ---------------------------------------------------------------------------
// bounded waits (thread 0) and CTA-wide abort
// ---------------------------------------------------------------------------
__device__ bool grid_barrier(int32_t* sync, unsigned target) {
  __threadfence();
  atomicAdd((unsigned*)&sync[SYNC_BAR], 1u);
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    if (ld_acquire(&sync[SYNC_BAR]) >= target) return true;
    if (ld_acquire(&sync[SYNC_ERR]) != 0) return false;
    if ((it & 63) == 63 && gtimer() - t0 > TIMEOUT_NS) {
      atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_BARRIER);
      return false;
    }
  }
}

__device__ bool wait_buf(const Smem& S, int32_t* sync, int b, uint32_t parity) {
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; ++it) {
    if (mbar_test(&S.mbar[b], parity)) return true;
    if ((it & 63) == 63 && gtimer() - t0 > TIMEOUT_NS) {
      atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_COPY);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// activation staging (the arithmetic of gemv_w8_kernel's prologue)
// ---------------------------------------------------------------------------
// K bf16 values (K % 8 == 0) from global memory to shared memory with 16-byte
// loads issued back to back; `copy_to` (global) receives the same bits.
__device__ __forceinline__ void load_bits(uint16_t* dst, const uint16_t* src, int K, bool readonly,
                                          uint16_t* copy_to = nullptr) {
  const int n16 = K >> 3;
#pragma unroll 4
  for (int i = threadIdx.x; i < n16; i += NT) {
    const uint4 v = readonly ? __ldg(((const uint4*)src) + i) : __ldcg(((const uint4*)src) + i);
    ((uint4*)dst)[i] = v;
    if (copy_to) ((uint4*)copy_to)[i] = v;
  }
}

// In place: xhi holds the bf16 bits of K values -> int16 hi words; xlo lo words;
// xs the group factors.  Eight lanes per quant group.
__device__ void bfp_stage(const Smem& S, int K, int G) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane >> 3, sl = lane & 7, per = G / 8;
  const int ng = K / G;
  for (int g0 = wid * 4; g0 < ng; g0 += NWARP * 4) {
    const int gi = g0 + sub;
    const bool valid = gi < ng;
    uint16_t* base = S.xhi + (size_t)(valid ? gi : 0) * G + sl * per;
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
          S.xlo[(base - S.xhi) + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
        }
      if (sl == 0) S.xs[gi] = inv;
    }
  }
}

// RMSNorm(src) * w -> bf16 bits in xhi (mode 0 kernel form, 1 golden form);
// `outf` (shared) receives the values as floats when non-null.  Uses xlo as scratch.
__device__ void stage_rmsnorm(const Smem& S, const uint16_t* src, bool src_readonly, const uint16_t* w, int K,
                              float eps, int mode, float* outf, uint16_t* copy_to) {
  load_bits(S.xhi, src, K, src_readonly, copy_to);
  load_bits(S.xlo, w, K, true);
  __syncthreads();
  double ss = 0.0;
  for (int i = threadIdx.x; i < K; i += NT) ss += rms_sq(bf2f(S.xhi[i]), mode);
  ss = block_sum_d(ss, S.red);
  const RmsCoef rc = rms_coef(ss, K, eps, mode);
  for (int i = threadIdx.x; i < K; i += NT) {
    const uint16_t o = f2bf(rms_apply(bf2f(S.xhi[i]), bf2f(S.xlo[i]), rc));
    S.xhi[i] = o;
    if (outf) outf[i] = bf2f(o);
  }
}

// ---------------------------------------------------------------------------
// int8 rows from shared memory, R (or 2R for gate/up pairs) rows per warp at once:
// sum_k q*s*x exactly as gemv_w8_kernel with LO staging and float64 accumulation
// ---------------------------------------------------------------------------
template <int G, int NR>
__device__ __forceinline__ void rows_dot(const uint8_t* const (&rp)[NR], int K, const Smem& S, double (&out)[NR]) {
  const int lane = threadIdx.x & 31;
  double acc[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) acc[i] = 0.0;
  for (int c = lane; c < (K >> 4); c += 32) {
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
      int a = __dp2a_lo((int)xa.x, (int)w[i].x, 0);
      a = __dp2a_hi((int)xa.y, (int)w[i].x, a);
      a = __dp2a_lo((int)xa.z, (int)w[i].y, a);
      a = __dp2a_hi((int)xa.w, (int)w[i].y, a);
      a = __dp2a_lo((int)xb.x, (int)w[i].z, a);
      a = __dp2a_hi((int)xb.y, (int)w[i].z, a);
      a = __dp2a_lo((int)xb.z, (int)w[i].w, a);
      a = __dp2a_hi((int)xb.w, (int)w[i].w, a);
      int l = __dp2a_lo((int)la.x, (int)w[i].x, 0);
      l = __dp2a_hi((int)la.y, (int)w[i].x, l);
      l = __dp2a_lo((int)la.z, (int)w[i].y, l);
      l = __dp2a_hi((int)la.w, (int)w[i].y, l);
      l = __dp2a_lo((int)lb.x, (int)w[i].z, l);
      l = __dp2a_hi((int)lb.y, (int)w[i].z, l);
      l = __dp2a_lo((int)lb.z, (int)w[i].w, l);
      l = __dp2a_hi((int)lb.w, (int)w[i].w, l);
      const long long t = (long long)a * 32768 + l;
      acc[i] = fma((double)t, (double)(sv[i] * xsc) * (1.0 / 32768.0), acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < NR; ++i) out[i] = warp_sum_d(acc[i]);
}

// the rows of one chunk: n rows (pairs when PAIR: gate rows then up rows) of rb bytes
template <int G, int R, bool PAIR, class Epi>
__device__ void chunk_rows(const uint8_t* wb, int n, int rb, int K, const Smem& S, Epi epi) {
  constexpr int NR = PAIR ? 2 * R : R;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int r0 = wid * R; r0 < n; r0 += NWARP * R) {
    const uint8_t* rp[NR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int r = min(r0 + i, n - 1);
      rp[i] = wb + (size_t)r * rb;
      if (PAIR) rp[R + i] = wb + (size_t)(n + r) * rb;
    }
    double out[NR];
    rows_dot<G, NR>(rp, K, S, out);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < R; ++i)
        if (r0 + i < n) epi(r0 + i, out[i], PAIR ? out[R + i] : 0.0);
    }
  }
}

template <int G, bool PAIR, class Epi>
__device__ void chunk_gemv(const uint8_t* wb, int n, int rb, int K, const Smem& S, Epi epi) {
  const int R = (n + NWARP - 1) / NWARP;
  if (R <= 1)
    chunk_rows<G, 1, PAIR>(wb, n, rb, K, S, epi);
  else if (R == 2)
    chunk_rows<G, 2, PAIR>(wb, n, rb, K, S, epi);
  else if (R == 3)
    chunk_rows<G, 3, PAIR>(wb, n, rb, K, S, epi);
  else
    chunk_rows<G, 4, PAIR>(wb, n, rb, K, S, epi);
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

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// splits per KV head for a context of L positions (about 128 positions each)
__device__ __forceinline__ int att_splits(int L, int smax) {
  const int s = (L + 127) / 128;
  return s < 1 ? 1 : (s > smax ? smax : s);
}

// ---------------------------------------------------------------------------
// attention unit: one KV head, one split of the positions; writes the split's
// partial (o, m, l) per query head.  The merge happens in the O-proj prologue.
// ---------------------------------------------------------------------------
template <int GQ>
__device__ void attention_unit(const Kp& p, const Smem& S, int layer, int h, int s, int ns, int P) {
  const iron_qwen3_model& m = p.m;
  constexpr int PER = HDIM / 32;
  constexpr int U = 4;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int L = P + 1;
  const int chunk = (L + ns - 1) / ns;
  const int start = s * chunk, end = min(L, start + chunk);
  float* qf = S.att;                   // [GQ][HD]
  float* kt = qf + GQ * HDIM;          // [HD]
  float* vt = kt + HDIM;               // [HD]
  float* part = vt + HDIM;             // [NWARP][GQ][HD+2]
  uint16_t* head = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
  const uint16_t* ang = m.angles + (size_t)P * HDIM;
  const bool owner = P >= start && P < end;
  // per-head q/k RMSNorm (golden form) + RoPE and the v copy: qk_norm_rope_kv_kernel's arithmetic
  for (int t = wid; t < GQ + 2; t += NWARP) {
    if (t == GQ + 1) {
      const uint16_t* vs = m.raw + (size_t)(m.Hq + m.Hkv + h) * HDIM;
      const uint2 v = __ldcg(((const uint2*)vs) + lane);
      vt[lane * 4 + 0] = bf_lo(v.x);
      vt[lane * 4 + 1] = bf_hi(v.x);
      vt[lane * 4 + 2] = bf_lo(v.y);
      vt[lane * 4 + 3] = bf_hi(v.y);
      if (owner) ((uint2*)(head + (size_t)P * 2 * HDIM + HDIM))[lane] = v;
      continue;
    }
    const bool isq = t < GQ;
    const int hh = isq ? h * GQ + t : m.Hq + h;
    const uint16_t* src = m.raw + (size_t)hh * HDIM;
    const uint16_t* nw = isq ? S.lay[layer].qn : S.lay[layer].kn;
    float v[PER], wv[PER], cs[PER], sn[PER];
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      const int i = lane + 32 * j;
      v[2 * j] = bf2f(ldcg_u16(src + i));
      v[2 * j + 1] = bf2f(ldcg_u16(src + i + HDIM / 2));
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
  __syncthreads();
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
  __syncthreads();
  float* ws = m.attn_ws + ((size_t)(h * ns + s) * GQ) * (HDIM + 2);
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
}

// Merge the split partials of every head (attn_combine_kernel's arithmetic) into
// bf16 bits in xhi; CTA 0 also stores them to m.attn.
template <int GQ>
__device__ void stage_attention(const Kp& p, const Smem& S, int ns) {
  const iron_qwen3_model& m = p.m;
  const int Hq = m.Hq;
  float* wgt = S.mrg;            // [Hq][SMAX]: m, then 2^(m - M)
  float* lsum = S.mrg + Hq * SMAX;  // [Hq]
  float* lv = (float*)S.xlo;     // [Hq][SMAX] l values (xlo is free until the BFP pass)
  for (int t = threadIdx.x; t < Hq * ns; t += NT) {
    const int hh = t / ns, sp = t - hh * ns;
    const int h = hh / GQ, g = hh - h * GQ;
    const float* ps = m.attn_ws + ((size_t)(h * ns + sp) * GQ + g) * (HDIM + 2);
    wgt[hh * SMAX + sp] = __ldcg(ps + HDIM);
    lv[hh * SMAX + sp] = __ldcg(ps + HDIM + 1);
  }
  __syncthreads();
  for (int hh = threadIdx.x; hh < Hq; hh += NT) {
    float M = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, wgt[hh * SMAX + sp]);
    float l = 0.f;
    for (int sp = 0; sp < ns; ++sp) {
      const float f = M != -INFINITY ? exp2f(wgt[hh * SMAX + sp] - M) : 0.f;
      wgt[hh * SMAX + sp] = f;
      l = fmaf(lv[hh * SMAX + sp], f, l);
    }
    lsum[hh] = l;
  }
  __syncthreads();
  const int QD = Hq * HDIM;
  constexpr int B4 = 4;  // outputs per thread per pass, their partial loads in flight together
  for (int i0 = threadIdx.x; i0 < QD; i0 += NT * B4) {
    float ov[B4][SMAX];
#pragma unroll
    for (int k = 0; k < B4; ++k) {
      const int i = i0 + k * NT;
      const int hh = i / HDIM, d = i - hh * HDIM;
      const int h = hh / GQ, g = hh - h * GQ;
#pragma unroll
      for (int sp = 0; sp < SMAX; ++sp)
        if (i < QD && sp < ns) ov[k][sp] = __ldcg(m.attn_ws + ((size_t)(h * ns + sp) * GQ + g) * (HDIM + 2) + d);
    }
#pragma unroll
    for (int k = 0; k < B4; ++k) {
      const int i = i0 + k * NT;
      if (i >= QD) break;
      const int hh = i / HDIM;
      float oo = 0.f;
#pragma unroll
      for (int sp = 0; sp < SMAX; ++sp)
        if (sp < ns) oo = fmaf(ov[k][sp], wgt[hh * SMAX + sp], oo);
      const float l = lsum[hh];
      const uint16_t b = f2bf(l > 0.f ? oo / l : 0.f);
      S.xhi[i] = b;
      if (blockIdx.x == 0) m.attn[i] = b;
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int G, int GQ>
__global__ void __launch_bounds__(NT, 1) qwen3_step_kernel(const __grid_constant__ Kp p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const iron_qwen3_model& m = p.m;
  const Smem S = carve(smem_raw, p, GQ);
  int32_t* sync = m.sync;
  const int tid = threadIdx.x, lane = tid & 31;
  const int N = gridDim.x;
  const Plan P = make_plan(p);
  const int QD = m.Hq * HDIM;
  const int pos = m.pos[0];
  // a position outside the cache or a token outside the vocabulary: record and leave
  // before touching memory (every CTA takes the same decision)
  if (pos < 0 || pos >= m.max_seq || (p.embed_input && (m.tok[0] < 0 || m.tok[0] >= m.V))) {
    if (tid == 0) atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_INPUT);
    return;
  }
  const int ns = att_splits(pos + 1, p.smax);
  const int unit = blockIdx.x < m.Hkv * ns ? (int)blockIdx.x : -1;

  if (tid == 0) {
    mbar_init(&S.mbar[0]);
    mbar_init(&S.mbar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  {  // the layer pointer table, read once
    const int nw = m.n_layers * (int)(sizeof(iron_qwen3_layer) / 8);
    for (int i = tid; i < nw; i += NT) ((unsigned long long*)S.lay)[i] = __ldg(((const unsigned long long*)m.layers) + i);
  }
  __syncthreads();
  if (tid == 0) {
    issue(p, P, S, 0, 0);
    issue(p, P, S, 1, 1);
    prefetch_layer_l2(p, P, S, 0);
    prefetch_layer_l2(p, P, S, 1);
  }
  int ci = 0;            // next chunk to consume
  unsigned epoch = 0;    // grid barriers passed
  bool ok = true;

  auto barrier = [&]() -> bool {
    __syncthreads();
    if (tid == 0) S.flag[0] = grid_barrier(sync, (++epoch) * (unsigned)N) ? 1 : 0;
    else ++epoch;
    __syncthreads();
    return S.flag[0] != 0;
  };
  // consume my chunks of one phase kind; fn(chunk, buffer) does the math
  auto consume = [&](int kind, auto&& fn) -> bool {
    const int nch = kind == 5 ? P.hnch : P.nch[kind];
    for (int k = 0; k < nch; ++k, ++ci) {
      const int b = ci & 1;
      if (tid == 0) S.flag[2] = wait_buf(S, sync, b, (ci >> 1) & 1) ? 1 : 0;
      __syncthreads();
      if (!S.flag[2]) return false;
      const Chunk ch = chunk_at(P, ci, m.n_layers);
      fn(ch, S.buf[b]);
      __syncthreads();
      if (tid == 0) issue(p, P, S, ci + 2, b);
    }
    return true;
  };

  for (int layer = 0; layer < m.n_layers && ok; ++layer) {
    const iron_qwen3_layer& Lw = S.lay[layer];
    // ---- QKV: hn = RMSNorm_golden(x, norm1); raw = bf16(Wqkv @ hn) ----
    {
      const bool emb = layer == 0 && p.embed_input;
      const uint16_t* xs = emb ? m.embed + (size_t)m.tok[0] * m.D : m.x;
      stage_rmsnorm(S, xs, emb, Lw.norm1, m.D, m.eps, 1, nullptr, (emb && blockIdx.x == 0) ? m.x : nullptr);
      __syncthreads();
      bfp_stage(S, m.D, G);
      __syncthreads();
      const int rbq = rowb(m.D, G);
      ok = consume(PH_QKV, [&](const Chunk& ch, const uint8_t* wb) {
        chunk_gemv<G, false>(wb, ch.r1 - ch.r0, rbq, m.D, S, [&](int r, double a, double) {
          m.raw[ch.r0 + r] = f2bf((float)a);
        });
      });
      if (tid == 0 && ok) {
        prefetch_layer_l2(p, P, S, layer + 2);
        if (unit >= 0) {  // this CTA's KV range of this layer, ahead of the attention phase
          const int L = pos + 1, h = unit / ns, sp = unit - (unit / ns) * ns;
          const int chunk = (L + ns - 1) / ns, st = sp * chunk, en = min(min(L, st + chunk), pos);
          if (en > st) {
            const uint16_t* hb = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
            prefetch_l2(hb + (size_t)st * 2 * HDIM, (uint32_t)(en - st) * 4 * HDIM);
          }
        }
      }
      if (!ok || !barrier()) break;
    }
    // ---- attention: one KV head and one split of the positions per CTA ----
    if (unit >= 0) attention_unit<GQ>(p, S, layer, unit / ns, unit - (unit / ns) * ns, ns, pos);
    if (!barrier()) break;
    // ---- O-proj + residual: x1 = bf16(x + bf16(Wo @ attn)); the split merge first ----
    {
      stage_attention<GQ>(p, S, ns);
      __syncthreads();
      bfp_stage(S, QD, G);
      __syncthreads();
      const int rbo = rowb(QD, G);
      ok = consume(PH_O, [&](const Chunk& ch, const uint8_t* wb) {
        chunk_gemv<G, false>(wb, ch.r1 - ch.r0, rbo, QD, S, [&](int r, double a, double) {
          const int row = ch.r0 + r;
          m.x1[row] = f2bf(bf2f(ldcg_u16(m.x + row)) + rbf_d(a));
        });
      });
      if (!ok || !barrier()) break;
    }
    // ---- gate/up: gh = bf16(silu_tanh(bf16(Wg@hf)) * bf16(Wu@hf)), hf = RMSNorm_kernel(x1) ----
    {
      stage_rmsnorm(S, m.x1, false, Lw.norm2, m.D, m.eps, 0, nullptr, nullptr);
      __syncthreads();
      bfp_stage(S, m.D, G);
      __syncthreads();
      const int rbg = rowb(m.D, G);
      ok = consume(PH_GU, [&](const Chunk& ch, const uint8_t* wb) {
        chunk_gemv<G, true>(wb, ch.r1 - ch.r0, rbg, m.D, S, [&](int r, double g, double u) {
          m.gh[ch.r0 + r] = f2bf(silu_tanh_bf16(rbf_d(g)) * rbf_d(u));
        });
      });
      if (!ok || !barrier()) break;
    }
    // ---- down + residual: x = bf16(x1 + bf16(Wd @ gh)) ----
    {
      load_bits(S.xhi, m.gh, m.FF, false);
      __syncthreads();
      bfp_stage(S, m.FF, G);
      __syncthreads();
      const int rbd = rowb(m.FF, G);
      ok = consume(PH_D, [&](const Chunk& ch, const uint8_t* wb) {
        chunk_gemv<G, false>(wb, ch.r1 - ch.r0, rbd, m.FF, S, [&](int r, double a, double) {
          const int row = ch.r0 + r;
          m.x[row] = f2bf(bf2f(ldcg_u16(m.x1 + row)) + rbf_d(a));
        });
      });
      if (!ok || !barrier()) break;
    }
  }

  if (ok && S.flag[0]) {
    // ---- final RMSNorm (golden form) + lm_head + greedy argmax ----
    stage_rmsnorm(S, m.x, false, m.final_norm, m.D, m.eps, 1, S.xf, nullptr);
    __syncthreads();
    if (m.lm_w8) bfp_stage(S, m.D, G);
    __syncthreads();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const int rbh = m.lm_w8 ? rowb(m.D, G) : m.D * 2;
    auto track = [&](int idx, uint16_t o) {
      if (m.logits) m.logits[idx] = o;
      if (better(bf2f(o), idx, bv, bi)) {
        bv = bf2f(o);
        bi = idx;
      }
    };
    ok = consume(5, [&](const Chunk& ch, const uint8_t* wb) {
      const int n = ch.r1 - ch.r0;
      if (m.lm_w8) {
        chunk_gemv<G, false>(wb, n, rbh, m.D, S, [&](int r, double a, double) { track(ch.r0 + r, f2bf((float)a)); });
      } else {
        constexpr int R = 3;
        const int wid = tid >> 5;
        for (int r0 = wid * R; r0 < n; r0 += NWARP * R) {
          const uint8_t* rp[R];
#pragma unroll
          for (int i = 0; i < R; ++i) rp[i] = wb + (size_t)min(r0 + i, n - 1) * rbh;
          float out[R];
          rows_dot_bf16<R>(rp, m.D, S.xf, out);
          if (lane == 0) {
#pragma unroll
            for (int i = 0; i < R; ++i)
              if (r0 + i < n) track(ch.r0 + r0 + i, f2bf(out[i]));
          }
        }
      }
    });
    if (ok) {
      // CTA-best over the warps' lane 0, then publish and let the last CTA reduce
      const int wid = tid >> 5;
      if (lane == 0) {
        S.att[wid] = bv;
        ((int*)S.att)[NWARP + wid] = bi;
      }
      __syncthreads();
      if (tid == 0) {
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int w = 0; w < NWARP; ++w)
          if (better(S.att[w], ((int*)S.att)[NWARP + w], v, i)) {
            v = S.att[w];
            i = ((int*)S.att)[NWARP + w];
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
          sync[SYNC_ARGMAX] = 0;
          sync[SYNC_BAR] = 0;
          __threadfence();
        }
      }
    }
  }
  // drain bulk copies still in flight (only after an early exit) before leaving
  if (tid == 0 && ci < P.total) {
    for (int k = ci; k < min(ci + 2, P.total); ++k) {
      const unsigned long long t0 = gtimer();
      while (!mbar_test(&S.mbar[k & 1], (k >> 1) & 1) && gtimer() - t0 < 20ull * 1000 * 1000) {
      }
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
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr[dev] = true;
  }
  void* args[] = {(void*)&p};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)fn, dim3(grid), dim3(NT), args, smem, st);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 step launch: %s", cudaGetErrorString(e));
  return IRON_OK;
}

static int kmax_of(const iron_qwen3_model* m) {
  int k = m->D;
  if (m->Hq * m->HD > k) k = m->Hq * m->HD;
  if (m->FF > k) k = m->FF;
  return k;
}

static int validate(const iron_qwen3_model* m) {
  IRON_REQUIRE(m != nullptr, IRON_ERR_ARG, "qwen3 step: null model");
  IRON_REQUIRE(m->HD == HDIM, IRON_ERR_UNSUPPORTED, "qwen3 step: head_dim %d (supported: 128)", m->HD);
  IRON_REQUIRE(m->Hkv >= 1 && m->Hq % m->Hkv == 0, IRON_ERR_ARG, "qwen3 step: Hq=%d, Hkv=%d", m->Hq, m->Hkv);
  const int GQ = m->Hq / m->Hkv;
  IRON_REQUIRE(GQ == 1 || GQ == 2 || GQ == 4 || GQ == 8, IRON_ERR_UNSUPPORTED, "qwen3 step: GQA group %d", GQ);
  IRON_REQUIRE(m->group == 32 || m->group == 64 || m->group == 128, IRON_ERR_ARG, "qwen3 step: group %d",
               m->group);
  IRON_REQUIRE(m->D % m->group == 0 && m->FF % m->group == 0 && m->D % 256 == 0 && m->D <= 4096, IRON_ERR_ARG,
               "qwen3 step: D=%d FF=%d must be multiples of the group and D a multiple of 256 (<= 4096)", m->D,
               m->FF);
  IRON_REQUIRE(kmax_of(m) <= 16 * NT * 4, IRON_ERR_UNSUPPORTED, "qwen3 step: reduction length too large");
  IRON_REQUIRE(2 * (m->D + 2 * (m->D / m->group)) <= BUF && m->FF + 2 * (m->FF / m->group) <= BUF, IRON_ERR_UNSUPPORTED,
               "qwen3 step: rows larger than the %d-byte weight buffers", BUF);
  IRON_REQUIRE(m->layers && m->final_norm && m->embed && m->angles && m->kv && m->x && m->raw && m->attn && m->x1 &&
                   m->gh && m->attn_ws && m->cand && m->tok && m->pos && m->seq_len && m->kv_off && m->sync,
               IRON_ERR_ARG, "qwen3 step: null buffer in the model descriptor");
  return IRON_OK;
}

static int grid_for(const iron_qwen3_model* m, size_t smem) {
  (void)m;
  (void)smem;
  return iron_num_sms();
}

}  // namespace qstep
}  // namespace iron

using namespace iron::qstep;

extern "C" int iron_qwen3_sync_words(const iron_qwen3_model* m) { return SYNC_HEAD0 + (m ? m->Hkv : 64); }
extern "C" int64_t iron_qwen3_cand_bytes(void) { return 1024 * 8; }
extern "C" int iron_qwen3_grid(const iron_qwen3_model* m) { return grid_for(m, 0); }
static int smax_for(const iron_qwen3_model* m, int grid) {
  int s = grid / m->Hkv;
  return s < 1 ? 1 : (s > SMAX ? SMAX : s);
}

extern "C" int64_t iron_qwen3_attn_ws_bytes(const iron_qwen3_model* m) {
  if (!m || m->Hkv < 1) return 0;
  return (int64_t)m->Hkv * smax_for(m, grid_for(m, 0)) * (m->Hq / m->Hkv) * (HDIM + 2) * 4;
}

extern "C" int iron_qwen3_sync_reset(const iron_qwen3_model* m, void* stream) {
  IRON_REQUIRE(m && m->sync, IRON_ERR_ARG, "qwen3 sync reset: null");
  cudaError_t e = cudaMemsetAsync(m->sync, 0, (size_t)iron_qwen3_sync_words(m) * 4, (cudaStream_t)stream);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "qwen3 sync reset: %s", cudaGetErrorString(e));
  return IRON_OK;
}

extern "C" int iron_qwen3_decode_step(const iron_qwen3_model* m, int embed_input, int advance, void* stream) {
  int rc = validate(m);
  if (rc) return rc;
  Kp p;
  p.m = *m;
  p.embed_input = embed_input;
  p.advance = advance;
  p.kmax = kmax_of(m);
  const int GQ = m->Hq / m->Hkv;
  const size_t smem = smem_bytes(p.kmax, m->D, GQ, m->Hq, m->n_layers);
  IRON_REQUIRE(smem <= 227 * 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: %zu bytes of shared memory", smem);
  const int grid = grid_for(m, smem);
  IRON_REQUIRE(grid <= 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: grid %d exceeds the candidate slots", grid);
  p.smax = smax_for(m, grid);
  cudaStream_t st = (cudaStream_t)stream;
#define IRON_STEP_CASE(g, gq) \
  if (m->group == g && GQ == gq) return launch<g, gq>(p, grid, smem, st);
  IRON_STEP_CASE(32, 2) IRON_STEP_CASE(32, 4) IRON_STEP_CASE(32, 1) IRON_STEP_CASE(32, 8)
  IRON_STEP_CASE(64, 2) IRON_STEP_CASE(64, 4) IRON_STEP_CASE(128, 2) IRON_STEP_CASE(128, 4)
#undef IRON_STEP_CASE
  return iron_set_error(IRON_ERR_UNSUPPORTED, "qwen3 step: group %d with GQA group %d", m->group, GQ);
}
