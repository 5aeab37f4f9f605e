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

struct Kp {
  iron_qwen3_model m;
  int embed_input, advance, nsplit, kmax;
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
  return s;
}

__host__ __device__ inline size_t smem_bytes(int kmax, int D, int GQ) {
  const size_t att = (size_t)(GQ * HDIM + 2 * HDIM + NWARP * GQ * (HDIM + 2)) * 4;
  return 2 * (size_t)BUF + (size_t)kmax * 4 + 32 * 8 + 16 + 16 + (size_t)(kmax / 32) * 4 + (size_t)D * 4 + att;
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
    const iron_qwen3_layer& L = m.layers[ch.layer];
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
__device__ void prefetch_layer_l2(const Kp& p, const Plan& P, int layer) {
  if (layer >= p.m.n_layers) return;
  const iron_qwen3_model& m = p.m;
  const iron_qwen3_layer& L = m.layers[layer];
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
// activation staging (identical arithmetic to gemv_w8_kernel's prologue)
// ---------------------------------------------------------------------------
// in-place: xhi holds bf16 bits of K values -> int16 hi words, xlo lo words, xs factors
__device__ void bfp_stage(const Smem& S, int K, int G) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int per = G / 32;
  for (int gi = wid; gi < K / G; gi += NWARP) {
    uint16_t* base = S.xhi + gi * G + lane * per;
    float v[4];
    float mx = 0.f;
    for (int e = 0; e < per; ++e) {
      v[e] = bf2f(base[e]);
      mx = fmaxf(mx, fabsf(v[e]));
    }
    mx = warp_max(mx);
    float sc, inv;
    bfp_scale(mx, sc, inv);
    for (int e = 0; e < per; ++e) {
      const float t = v[e] * sc;
      const int hi = __float2int_rn(t);
      base[e] = (uint16_t)(int16_t)hi;
      S.xlo[(base - S.xhi) + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
    }
    if (lane == 0) S.xs[gi] = inv;
  }
}

// RMSNorm(src) * w -> bf16 bits in xhi (mode 0 kernel form, 1 golden form); also
// returns the normalised values as floats in `outf` when non-null
__device__ void stage_rmsnorm(const Smem& S, const uint16_t* src, bool src_readonly, const uint16_t* w, int K,
                              float eps, int mode, float* outf, uint16_t* copy_to) {
  constexpr int MAXV = 16;  // K <= NT * MAXV
  float v[MAXV];
  double ss = 0.0;
  int n = 0;
  for (int i = threadIdx.x; i < K; i += NT, ++n) {
    v[n] = bf2f(src_readonly ? __ldg(src + i) : ldcg_u16(src + i));
    ss += rms_sq(v[n], mode);
  }
  ss = block_sum_d(ss, S.red);
  const RmsCoef rc = rms_coef(ss, K, eps, mode);
  n = 0;
  for (int i = threadIdx.x; i < K; i += NT, ++n) {
    const uint16_t o = f2bf(rms_apply(v[n], bf2f(__ldg(w + i)), rc));
    S.xhi[i] = o;
    if (outf) outf[i] = bf2f(o);
    if (copy_to) copy_to[i] = f2bf(v[n]);
  }
}

__device__ void stage_copy(const Smem& S, const uint16_t* src, int K) {
  for (int i = threadIdx.x; i < K; i += NT) S.xhi[i] = (uint16_t)ldcg_u16(src + i);
}

// ---------------------------------------------------------------------------
// int8 row dot product from shared memory: sum_k q*s*x as in gemv_w8_kernel (LO)
// ---------------------------------------------------------------------------
template <int G>
__device__ __forceinline__ double row_dot(const uint8_t* row, int K, const Smem& S) {
  const int lane = threadIdx.x & 31;
  const uint16_t* sc = (const uint16_t*)(row + K);
  double acc = 0.0;
  for (int c = lane; c < (K >> 4); c += 32) {
    const uint4 w = *(const uint4*)(row + c * 16);
    const int g = (c * 16) / G;
    const float sv = bf2f(sc[g]);
    const uint4 xa = *(const uint4*)(S.xhi + c * 16), xb = *(const uint4*)(S.xhi + c * 16 + 8);
    const uint4 la = *(const uint4*)(S.xlo + c * 16), lb = *(const uint4*)(S.xlo + c * 16 + 8);
    int a = __dp2a_lo((int)xa.x, (int)w.x, 0);
    a = __dp2a_hi((int)xa.y, (int)w.x, a);
    a = __dp2a_lo((int)xa.z, (int)w.y, a);
    a = __dp2a_hi((int)xa.w, (int)w.y, a);
    a = __dp2a_lo((int)xb.x, (int)w.z, a);
    a = __dp2a_hi((int)xb.y, (int)w.z, a);
    a = __dp2a_lo((int)xb.z, (int)w.w, a);
    a = __dp2a_hi((int)xb.w, (int)w.w, a);
    int l = __dp2a_lo((int)la.x, (int)w.x, 0);
    l = __dp2a_hi((int)la.y, (int)w.x, l);
    l = __dp2a_lo((int)la.z, (int)w.y, l);
    l = __dp2a_hi((int)la.w, (int)w.y, l);
    l = __dp2a_lo((int)lb.x, (int)w.z, l);
    l = __dp2a_hi((int)lb.y, (int)w.z, l);
    l = __dp2a_lo((int)lb.z, (int)w.w, l);
    l = __dp2a_hi((int)lb.w, (int)w.w, l);
    const long long t = (long long)a * 32768 + l;
    acc = fma((double)t, (double)(sv * S.xs[g]) * (1.0 / 32768.0), acc);
  }
  return warp_sum_d(acc);
}

// bf16 row dot with float32 activations (the lm_head of gemv_bf16_kernel)
__device__ __forceinline__ float row_dot_bf16(const uint8_t* row, int K, const float* xf) {
  const int lane = threadIdx.x & 31;
  float a = 0.f;
  for (int c = lane; c < (K >> 3); c += 32) {
    const uint4 w = *(const uint4*)(row + c * 16);
    const float4 x0 = *(const float4*)(xf + c * 8), x1 = *(const float4*)(xf + c * 8 + 4);
    a = fmaf(bf_lo(w.x), x0.x, a);
    a = fmaf(bf_hi(w.x), x0.y, a);
    a = fmaf(bf_lo(w.y), x0.z, a);
    a = fmaf(bf_hi(w.y), x0.w, a);
    a = fmaf(bf_lo(w.z), x1.x, a);
    a = fmaf(bf_hi(w.z), x1.y, a);
    a = fmaf(bf_lo(w.w), x1.z, a);
    a = fmaf(bf_hi(w.w), x1.w, a);
  }
  return warp_sum(a);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// attention unit: one KV head, one split of the positions
// ---------------------------------------------------------------------------
template <int GQ>
__device__ void attention_unit(const Kp& p, const Smem& S, int layer, int unit, int P, int32_t* sync) {
  const iron_qwen3_model& m = p.m;
  constexpr int PER = HDIM / 32;
  constexpr int U = 4;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int ns = p.nsplit;
  const int h = unit / ns, s = unit - h * ns;
  const int L = P + 1;
  const int chunk = (L + ns - 1) / ns;
  const int start = s * chunk, end = min(L, start + chunk);
  float* qf = S.att;                   // [GQ][HD]
  float* kt = qf + GQ * HDIM;          // [HD]
  float* vt = kt + HDIM;               // [HD]
  float* part = vt + HDIM;             // [NWARP][GQ][HD+2]
  uint16_t* head = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
  const uint16_t* ang = m.angles + (size_t)P * HDIM;
  const int QKV = (m.Hq + 2 * m.Hkv) * HDIM;
  (void)QKV;
  // per-head q/k RMSNorm (golden form) + RoPE, v copy: the arithmetic of qk_norm_rope_kv_kernel
  for (int t = wid; t < GQ + 2; t += NWARP) {
    if (t == GQ + 1) {
      const uint16_t* vs = m.raw + (size_t)(m.Hq + m.Hkv + h) * HDIM;
      for (int i = lane; i < HDIM; i += 32) {
        const uint16_t v = (uint16_t)ldcg_u16(vs + i);
        vt[i] = bf2f(v);
        if (P >= start && P < end) head[(size_t)P * 2 * HDIM + HDIM + i] = v;
      }
      continue;
    }
    const bool isq = t < GQ;
    const int hh = isq ? h * GQ + t : m.Hq + h;
    const uint16_t* src = m.raw + (size_t)hh * HDIM;
    const uint16_t* nw = isq ? m.layers[layer].qn : m.layers[layer].kn;
    float v[PER];
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      const int i = lane + 32 * j;
      v[2 * j] = bf2f(ldcg_u16(src + i));
      v[2 * j + 1] = bf2f(ldcg_u16(src + i + HDIM / 2));
      ss += rms_sq(v[2 * j], 1);
      ss += rms_sq(v[2 * j + 1], 1);
    }
    ss = warp_sum_d(ss);
    const RmsCoef rc = rms_coef(ss, HDIM, m.eps, 1);
    float* dst = isq ? qf + t * HDIM : kt;
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      const int i = lane + 32 * j;
      const float x1 = rbf(rms_apply(v[2 * j], bf2f(__ldg(nw + i)), rc));
      const float x2 = rbf(rms_apply(v[2 * j + 1], bf2f(__ldg(nw + i + HDIM / 2)), rc));
      const float c = bf2f(__ldg(ang + 2 * i)), sn = bf2f(__ldg(ang + 2 * i + 1));
      const uint16_t o1 = f2bf(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn)));
      const uint16_t o2 = f2bf(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn)));
      dst[i] = bf2f(o1);
      dst[i + HDIM / 2] = bf2f(o2);
      if (!isq && P >= start && P < end) {
        head[(size_t)P * 2 * HDIM + i] = o1;
        head[(size_t)P * 2 * HDIM + i + HDIM / 2] = o2;
      }
    }
  }
  __syncthreads();
  // flash decoding over [start, end): the online softmax of attn_split_kernel
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
  for (int j0 = start + wid * U; j0 < end; j0 += NWARP * U) {
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
        const uint16_t* kr = head + (size_t)j * 2 * HDIM + lane * PER;
        const uint2 kk = ldg_stream8(kr), vv = ldg_stream8(kr + HDIM);
        kf[u][0] = bf_lo(kk.x);
        kf[u][1] = bf_hi(kk.x);
        kf[u][2] = bf_lo(kk.y);
        kf[u][3] = bf_hi(kk.y);
        vf[u][0] = bf_lo(vv.x);
        vf[u][1] = bf_hi(vv.x);
        vf[u][2] = bf_lo(vv.y);
        vf[u][3] = bf_hi(vv.y);
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
  }
  // merge the warps, write this split's partial (o, m, l) per head
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
  // the last split of this KV head merges all splits (attn_combine_kernel's arithmetic)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd((int*)&sync[SYNC_HEAD0 + h], 1);
    S.flag[1] = (old == ns - 1);
  }
  __syncthreads();
  if (S.flag[1]) {
    __threadfence();
    for (int t = threadIdx.x; t < GQ * HDIM; t += NT) {
      const int g = t / HDIM, d = t - g * HDIM;
      const float* base = m.attn_ws + ((size_t)h * ns * GQ + g) * (HDIM + 2);
      const size_t stride = (size_t)GQ * (HDIM + 2);
      float M = -INFINITY;
      for (int q2 = 0; q2 < ns; ++q2) M = fmaxf(M, __ldcg(base + q2 * stride + HDIM));
      float oo = 0.f, lsum = 0.f;
      if (M != -INFINITY) {
        for (int q2 = 0; q2 < ns; ++q2) {
          const float* ps = base + q2 * stride;
          const float f = exp2f(__ldcg(ps + HDIM) - M);
          oo = fmaf(__ldcg(ps + d), f, oo);
          lsum = fmaf(__ldcg(ps + HDIM + 1), f, lsum);
        }
      }
      m.attn[(size_t)(h * GQ + g) * HDIM + d] = f2bf(lsum > 0.f ? oo / lsum : 0.f);
    }
    if (threadIdx.x == 0) atomicExch((int*)&sync[SYNC_HEAD0 + h], 0);
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
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int N = gridDim.x;
  const Plan P = make_plan(p);
  const int QD = m.Hq * HDIM, QKV = (m.Hq + 2 * m.Hkv) * HDIM;
  const int pos = m.pos[0];
  const int unit = blockIdx.x < m.Hkv * p.nsplit ? (int)blockIdx.x : -1;
  // a position outside the cache or a token outside the vocabulary: record and leave
  // before touching memory (every CTA takes the same decision)
  if (pos < 0 || pos >= m.max_seq || (p.embed_input && (m.tok[0] < 0 || m.tok[0] >= m.V))) {
    if (tid == 0) atomicCAS((int*)&sync[SYNC_ERR], 0, ERR_INPUT);
    return;
  }

  if (tid == 0) {
    mbar_init(&S.mbar[0]);
    mbar_init(&S.mbar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    issue(p, P, S, 0, 0);
    issue(p, P, S, 1, 1);
    prefetch_layer_l2(p, P, 1);
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
    const iron_qwen3_layer& Lw = m.layers[layer];
    // ---- QKV: hn = RMSNorm_golden(x, norm1); raw = bf16(Wqkv @ hn) ----
    {
      const bool emb = layer == 0 && p.embed_input;
      const uint16_t* xs = emb ? m.embed + (size_t)m.tok[0] * m.D : m.x;
      stage_rmsnorm(S, xs, emb, Lw.norm1, m.D, m.eps, 1, nullptr, (emb && blockIdx.x == 0) ? m.x : nullptr);
      __syncthreads();
      bfp_stage(S, m.D, G);
      if (tid == 0) {
        prefetch_layer_l2(p, P, layer + 2);
        if (unit >= 0) {  // this CTA's KV range of this layer, one phase ahead
          const int L = pos + 1, ns = p.nsplit, h = unit / ns, s = unit - (unit / ns) * ns;
          const int chunk = (L + ns - 1) / ns, st = s * chunk, en = min(min(L, st + chunk), pos);
          if (en > st) {
            const uint16_t* hb = m.kv + ((size_t)layer * m.Hkv + h) * 2 * (size_t)m.max_seq * HDIM;
            prefetch_l2(hb + (size_t)st * 2 * HDIM, (uint32_t)(en - st) * 4 * HDIM);
          }
        }
      }
      __syncthreads();
      const int rbq = rowb(m.D, G);
      ok = consume(PH_QKV, [&](const Chunk& ch, const uint8_t* wb) {
        for (int r = wid; r < ch.r1 - ch.r0; r += NWARP) {
          const double a = row_dot<G>(wb + (size_t)r * rbq, m.D, S);
          if (lane == 0) m.raw[ch.r0 + r] = f2bf((float)a);
        }
      });
      if (!ok || !barrier()) break;
    }
    // ---- attention (per KV head and split) + merge by the last split ----
    if (unit >= 0) attention_unit<GQ>(p, S, layer, unit, pos, sync);
    if (!barrier()) break;
    // ---- O-proj + residual: x1 = bf16(x + bf16(Wo @ attn)) ----
    {
      stage_copy(S, m.attn, QD);
      __syncthreads();
      bfp_stage(S, QD, G);
      __syncthreads();
      const int rbo = rowb(QD, G);
      ok = consume(PH_O, [&](const Chunk& ch, const uint8_t* wb) {
        for (int r = wid; r < ch.r1 - ch.r0; r += NWARP) {
          const double a = row_dot<G>(wb + (size_t)r * rbo, QD, S);
          if (lane == 0) {
            const int row = ch.r0 + r;
            m.x1[row] = f2bf(bf2f(ldcg_u16(m.x + row)) + rbf_d(a));
          }
        }
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
        const int n = ch.r1 - ch.r0;
        for (int r = wid; r < n; r += NWARP) {
          const double g = row_dot<G>(wb + (size_t)r * rbg, m.D, S);
          const double u = row_dot<G>(wb + (size_t)(n + r) * rbg, m.D, S);
          if (lane == 0) m.gh[ch.r0 + r] = f2bf(silu_tanh_bf16(rbf_d(g)) * rbf_d(u));
        }
      });
      if (!ok || !barrier()) break;
    }
    // ---- down + residual: x = bf16(x1 + bf16(Wd @ gh)) ----
    {
      stage_copy(S, m.gh, m.FF);
      __syncthreads();
      bfp_stage(S, m.FF, G);
      __syncthreads();
      const int rbd = rowb(m.FF, G);
      ok = consume(PH_D, [&](const Chunk& ch, const uint8_t* wb) {
        for (int r = wid; r < ch.r1 - ch.r0; r += NWARP) {
          const double a = row_dot<G>(wb + (size_t)r * rbd, m.FF, S);
          if (lane == 0) {
            const int row = ch.r0 + r;
            m.x[row] = f2bf(bf2f(ldcg_u16(m.x1 + row)) + rbf_d(a));
          }
        }
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
    ok = consume(5, [&](const Chunk& ch, const uint8_t* wb) {
      for (int r = wid; r < ch.r1 - ch.r0; r += NWARP) {
        const uint8_t* row = wb + (size_t)r * rbh;
        const uint16_t o = m.lm_w8 ? f2bf((float)row_dot<G>(row, m.D, S)) : f2bf(row_dot_bf16(row, m.D, S.xf));
        const int idx = ch.r0 + r;
        if (m.logits && lane == 0) m.logits[idx] = o;
        if (better(bf2f(o), idx, bv, bi)) {
          bv = bf2f(o);
          bi = idx;
        }
      }
    });
    if (ok) {
      // CTA-best (all lanes of a warp agree), then publish and let the last CTA reduce
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
extern "C" int64_t iron_qwen3_attn_ws_bytes(const iron_qwen3_model* m) {
  if (!m || m->Hkv < 1) return 0;
  const int grid = grid_for(m, 0);
  const int ns = grid / m->Hkv < 1 ? 1 : grid / m->Hkv;
  return (int64_t)m->Hkv * ns * (m->Hq / m->Hkv) * (HDIM + 2) * 4;
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
  const size_t smem = smem_bytes(p.kmax, m->D, GQ);
  IRON_REQUIRE(smem <= 227 * 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: %zu bytes of shared memory", smem);
  const int grid = grid_for(m, smem);
  IRON_REQUIRE(grid <= 1024, IRON_ERR_UNSUPPORTED, "qwen3 step: grid %d exceeds the candidate slots", grid);
  p.nsplit = grid / m->Hkv < 1 ? 1 : grid / m->Hkv;
  cudaStream_t st = (cudaStream_t)stream;
#define IRON_STEP_CASE(g, gq) \
  if (m->group == g && GQ == gq) return launch<g, gq>(p, grid, smem, st);
  IRON_STEP_CASE(32, 2) IRON_STEP_CASE(32, 4) IRON_STEP_CASE(32, 1) IRON_STEP_CASE(32, 8)
  IRON_STEP_CASE(64, 2) IRON_STEP_CASE(64, 4) IRON_STEP_CASE(128, 2) IRON_STEP_CASE(128, 4)
#undef IRON_STEP_CASE
  return iron_set_error(IRON_ERR_UNSUPPORTED, "qwen3 step: group %d with GQA group %d", m->group, GQ);
}
