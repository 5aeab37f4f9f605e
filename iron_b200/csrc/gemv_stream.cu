// Streaming int8 group-quantised GEMV (W8A16) for plain wires (tile_m = 1, rows
// contiguous): the same arithmetic as gemv_w8_kernel, with the weight brought in
// by bulk copies instead of per-lane loads.
//
// Why.  A decode GEMV is a single pass over the weight; it reaches HBM bandwidth
// only with enough bytes in flight per SM.  Per-lane 16-byte loads keep a few
// hundred bytes in flight per warp and wait out the memory latency every
// iteration.  Here one CTA per SM owns a contiguous block of rows; a producer warp
// copies that block, chunk by chunk, into a ~190 KB shared-memory ring with
// cp.async.bulk (no multicast) as fast as ring slots free up, while eight compute
// warps work on the chunks already landed.
//
// Numerics.  Identical to gemv_w8_kernel: activations (optionally RMS-normalised)
// staged once per CTA as exact int16 block floating point (hi words, plus lo words
// at batch 1), dp2a over 16-byte weight chunks, the group scale applied per chunk,
// float64 accumulation, one bf16 rounding.
//
// Waits are bounded by %globaltimer; on a timeout the CTA stops and the outputs
// of its rows are undefined.
#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {
namespace gstream {

constexpr int NT = 256, NWARP = NT / 32;
constexpr int NMB = 8;  // ring slots
constexpr int PIECE = 32768;
constexpr int SMEM_MAX = 227 * 1024;
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;

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
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

struct RingState {  // producer lane <-> compute thread 0
  unsigned long long tail;
  int issued, consumed, abort, bad;
  uint32_t slot[NMB];             // ring offset of each slot's chunk
  unsigned long long end[NMB];    // allocation count after it (monotonic)
};

__host__ __device__ inline int rowb(int K, int G) { return K + 2 * (K / G); }
__host__ __device__ inline void part(int M, int c, int N, int& lo, int& hi) {
  lo = (int)((long long)M * c / N);
  hi = (int)((long long)M * (c + 1) / N);
}
// bytes of x staging for NB rows of K (hi words, lo words at batch 1, block factors)
__host__ __device__ inline size_t stage_bytes(int NB, bool LO, int K, int G) {
  return (size_t)(LO ? 2 : 1) * NB * K * 2 + (size_t)NB * (K / G) * 4;
}

template <int G, int NB, bool PAIR, bool LO, int R>
__global__ void __launch_bounds__(NT + 32, 1) gemv_stream_kernel(const __grid_constant__ GemvW8Params p, int ring) {
  constexpr int RPC = NWARP * R;  // rows per chunk (each warp R rows)
  constexpr int NRW = PAIR ? 2 * R : R;
  extern __shared__ __align__(128) uint8_t sm[];
  const int K = p.K, KG = K / G, RB = rowb(K, G);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  size_t o = (size_t)ring;
  uint16_t* xq = (uint16_t*)(sm + o);  // [NB][K] hi words
  o += (size_t)NB * K * 2;
  uint16_t* xl = (uint16_t*)(sm + o);  // [NB][K] lo words (LO)
  o += LO ? (size_t)NB * K * 2 : 0;
  float* xs = (float*)(sm + o);        // [NB][KG]
  o += ((size_t)NB * KG * 4 + 15) & ~(size_t)15;
  double* red = (double*)(sm + o);     // [32]
  o += 32 * 8;
  uint64_t* mbar = (uint64_t*)(sm + o);
  o += NMB * 8;
  volatile RingState& rs = *(RingState*)(sm + o);

  int r0, r1;
  part(p.M, blockIdx.x, gridDim.x, r0, r1);
  const int nch = (r1 - r0 + RPC - 1) / RPC;
  auto chunk_rows = [&](int j) { return min(RPC, r1 - r0 - j * RPC); };
  if (tid == 0) {
    for (int i = 0; i < NMB; ++i) mbar_init(&mbar[i]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    rs.tail = 0;
    rs.issued = rs.consumed = rs.abort = rs.bad = 0;
  }
  __syncthreads();  // the last barrier of all NT + 32 threads

  if (tid >= NT) {  // ---- producer lane ----
    if (tid != NT) return;
    const uint32_t Rb = (uint32_t)ring;
    unsigned long long head = 0;
    bool stop = false;
    for (int j = 0; j < nch && !stop; ++j) {
      const int n = chunk_rows(j);
      const uint32_t seg = (uint32_t)n * RB, bytes = seg * (PAIR ? 2u : 1u);
      unsigned long long start = head;
      const uint32_t off = (uint32_t)(start % Rb);
      if (off + bytes > Rb) start += Rb - off;
      const unsigned long long t0 = gtimer();
      for (unsigned it = 0;; ++it) {
        if (start + bytes - rs.tail <= Rb && j - rs.consumed < NMB) break;
        if (rs.abort || ((it & 15) == 15 && gtimer() - t0 > TIMEOUT_NS)) {
          stop = true;
          break;
        }
        __nanosleep(32);
      }
      if (stop) break;
      const int sl = j % NMB;
      uint8_t* dst = sm + (uint32_t)(start % Rb);
      rs.slot[sl] = (uint32_t)(start % Rb);
      rs.end[sl] = start + bytes;
      head = start + bytes;
      const int row = r0 + j * RPC;
      fence_proxy_async();
      mbar_expect(&mbar[sl], bytes);
#pragma unroll
      for (int s = 0; s < (PAIR ? 2 : 1); ++s) {
        const uint8_t* src = (s == 0 ? p.wa.base : p.wb.base) + (size_t)row * RB;
        for (uint32_t q = 0; q < seg; q += PIECE) bulk_g2s(dst + q, src + q, min((uint32_t)PIECE, seg - q), &mbar[sl]);
        dst += seg;
      }
      rs.issued = j + 1;
    }
    if (stop) {  // let the copies in flight land before the CTA may exit
      for (int k = rs.consumed; k < rs.issued; ++k) {
        const unsigned long long t0 = gtimer();
        while (!mbar_test(&mbar[k % NMB], (uint32_t)((k / NMB) & 1)) && gtimer() - t0 < 20ull * 1000 * 1000) {
        }
      }
    }
    return;
  }

  // ---- prologue: activations -> (optionally RMS-normalised) bf16 -> int16 BFP ----
  for (int b = 0; b < NB; ++b) {
    const uint16_t* xr = p.x + (size_t)b * p.ld_x;
    if (b >= p.nb) {
      for (int i = tid; i < K; i += NT) xq[b * K + i] = 0;
      continue;
    }
    if (p.rms_w) {
      double ss = 0.0;
      for (int i = tid; i < K; i += NT) ss += rms_sq(bf2f(xr[i]), p.rms_mode);
      ss = warp_sum_d(ss);
      csync();
      if (lane == 0) red[wid] = ss;
      csync();
      ss = warp_sum_d(lane < NWARP ? red[lane] : 0.0);
      const RmsCoef rc = rms_coef(ss, K, p.eps, p.rms_mode);
      for (int i = tid; i < K; i += NT) xq[b * K + i] = f2bf(rms_apply(bf2f(xr[i]), bf2f(p.rms_w[i]), rc));
      csync();  // red is reused by the next row
    } else {
      for (int i = tid; i < K; i += NT) xq[b * K + i] = xr[i];
    }
  }
  csync();
  {
    constexpr int PER = G / 32;
    for (int gi = wid; gi < NB * KG; gi += NWARP) {
      const int b = gi / KG, g = gi - b * KG;
      uint16_t* base = xq + b * K + g * G + lane * PER;
      float v[PER];
      float mx = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        v[e] = bf2f(base[e]);
        mx = fmaxf(mx, fabsf(v[e]));
      }
      mx = warp_max(mx);
      float sc, inv;
      bfp_scale(mx, sc, inv);
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const float t = v[e] * sc;
        const int hi = __float2int_rn(t);
        base[e] = (uint16_t)(int16_t)hi;
        if (LO) xl[(base - xq) + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
      }
      if (lane == 0) xs[b * KG + g] = inv;
    }
  }
  csync();

  // ---- the chunks ----
  const uint32_t xm = p.xor_mask;
  for (int j = 0; j < nch; ++j) {
    const int sl = j % NMB;
    if (tid == 0) {
      const unsigned long long t0 = gtimer();
      bool landed = true;
      for (unsigned it = 0; !mbar_test(&mbar[sl], (uint32_t)((j / NMB) & 1)); ++it)
        if ((it & 63) == 63 && gtimer() - t0 > TIMEOUT_NS) {
          landed = false;
          break;
        }
      rs.bad = landed ? 0 : 1;
    }
    csync();
    if (rs.bad) break;
    const int n = chunk_rows(j);
    const uint8_t* buf = sm + rs.slot[sl];
    const uint8_t* wp[NRW];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int r = min(wid + NWARP * i, n - 1);
      wp[i] = buf + (size_t)r * RB;
      if (PAIR) wp[R + i] = buf + (size_t)(n + r) * RB;
    }
    double acc[NRW][NB];
#pragma unroll
    for (int r = 0; r < NRW; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.0;
    for (int c = lane; c < (K >> 4); c += 32) {
      const int g = (c * 16) / G;
      uint4 wv[NRW];
      float sv[NRW];
#pragma unroll
      for (int r = 0; r < NRW; ++r) {
        wv[r] = *(const uint4*)(wp[r] + c * 16);
        sv[r] = bf2f(((const uint16_t*)(wp[r] + K))[g]);
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const uint4 xa = *(const uint4*)(xq + b * K + c * 16), xb = *(const uint4*)(xq + b * K + c * 16 + 8);
        uint4 la = make_uint4(0, 0, 0, 0), lb = la;
        if (LO) {
          la = *(const uint4*)(xl + b * K + c * 16);
          lb = *(const uint4*)(xl + b * K + c * 16 + 8);
        }
        const float xsc = xs[b * KG + g];
#pragma unroll
        for (int r = 0; r < NRW; ++r) {
          const uint32_t w0 = wv[r].x ^ xm, w1 = wv[r].y ^ xm, w2 = wv[r].z ^ xm, w3 = wv[r].w ^ xm;
          int a = __dp2a_lo((int)xa.x, (int)w0, 0);
          a = __dp2a_hi((int)xa.y, (int)w0, a);
          a = __dp2a_lo((int)xa.z, (int)w1, a);
          a = __dp2a_hi((int)xa.w, (int)w1, a);
          a = __dp2a_lo((int)xb.x, (int)w2, a);
          a = __dp2a_hi((int)xb.y, (int)w2, a);
          a = __dp2a_lo((int)xb.z, (int)w3, a);
          a = __dp2a_hi((int)xb.w, (int)w3, a);
          long long t = a;
          if (LO) {
            int l = __dp2a_lo((int)la.x, (int)w0, 0);
            l = __dp2a_hi((int)la.y, (int)w0, l);
            l = __dp2a_lo((int)la.z, (int)w1, l);
            l = __dp2a_hi((int)la.w, (int)w1, l);
            l = __dp2a_lo((int)lb.x, (int)w2, l);
            l = __dp2a_hi((int)lb.y, (int)w2, l);
            l = __dp2a_lo((int)lb.z, (int)w3, l);
            l = __dp2a_hi((int)lb.w, (int)w3, l);
            t = t * 32768 + l;
          }
          const double sc = LO ? (double)(sv[r] * xsc) * (1.0 / 32768.0) : (double)(sv[r] * xsc);
          acc[r][b] = fma((double)t, sc, acc[r][b]);
        }
      }
    }
    // every lane holds the sums after the butterfly; lane r*NB + b stores output (r, b)
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const double s0 = warp_sum_d(acc[r][b]);
        const double s1 = PAIR ? warp_sum_d(acc[R + r][b]) : 0.0;
        const int lr = wid + NWARP * r;
        if (lane == r * NB + b && lr < n && b < p.nb) {
          const int row = r0 + j * RPC + lr;
          uint16_t* yo = p.y + (size_t)b * p.ld_y + row;
          if (PAIR) {
            *yo = f2bf(silu_tanh_bf16(rbf_d(s0)) * rbf_d(s1));
          } else if (p.epi == EPI_RESID) {
            *yo = f2bf(bf2f(p.res[(size_t)b * p.ld_y + row]) + rbf_d(s0));
          } else if (p.epi == EPI_F32) {
            ((float*)p.y)[(size_t)b * p.ld_y + row] = (float)s0;
          } else {
            *yo = f2bf((float)s0);
          }
        }
      }
    csync();
    if (tid == 0) {  // release the chunk's ring space
      fence_proxy_async();
      rs.tail = rs.end[sl];
      rs.consumed = j + 1;
    }
  }
  if (tid == 0 && rs.consumed < nch) rs.abort = 1;  // the producer stops and drains
}

}  // namespace gstream

// Bytes of shared memory the streaming kernel needs besides its ring, or 0 if the
// shape does not suit it (the caller then uses gemv_w8_kernel).
static size_t stream_fixed(int NB, bool LO, int K, int G) {
  return gstream::stage_bytes(NB, LO, K, G) + 16 + 32 * 8 + gstream::NMB * 8 + sizeof(gstream::RingState) + 64;
}

template <int G, int NB, bool PAIR, bool LO, int R>
static int stream_launch_r(const GemvW8Params& p, cudaStream_t st, size_t fixed) {
  using namespace gstream;
  auto fn = gemv_stream_kernel<G, NB, PAIR, LO, R>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
    attr[dev] = true;
  }
  const int ring = (int)(((size_t)SMEM_MAX - fixed) & ~(size_t)1023);
  int grid = iron_num_sms();
  if (grid > p.M) grid = p.M;
  fn<<<grid, NT + 32, (size_t)ring + fixed, st>>>(p, ring);
  return iron_check_launch("gemv_stream_kernel");
}

// Streaming launch for a plain wire when the staging and a ring of at least two
// chunks fit; returns 1 when the shape is not handled here.
template <int G, int NB, bool PAIR>
static int stream_launch(const GemvW8Params& p, cudaStream_t st) {
  constexpr bool LO = NB == 1;
  const size_t fixed = stream_fixed(NB, LO, p.K, G);
  const size_t rb = (size_t)gstream::rowb(p.K, G) * (PAIR ? 2 : 1);
  if (fixed > 64 * 1024) return 1;
  const size_t ring = (size_t)gstream::SMEM_MAX - fixed;
  // four rows per warp and chunk while a chunk stays near 40 KB and the float64 sums fit
  // in registers; otherwise one; the ring must hold three chunks
  if constexpr (4 * (PAIR ? 2 : 1) * NB <= 16) {
    if (rb * gstream::NWARP * 4 <= 40 * 1024) return stream_launch_r<G, NB, PAIR, LO, 4>(p, st, fixed);
  }
  if (3 * rb * gstream::NWARP > ring) return 1;
  return stream_launch_r<G, NB, PAIR, LO, 1>(p, st, fixed);
}

template <int G>
int stream_launch_g(const GemvW8Params& p, bool pair, cudaStream_t st) {
  const int nb = p.nb;  // 2..3 rows run in the 4-row kernel, 5..7 in the 8-row one
  if (pair) {
    if (nb <= 1) return stream_launch<G, 1, true>(p, st);
    if (nb <= 4) return stream_launch<G, 4, true>(p, st);
    return stream_launch<G, 8, true>(p, st);
  }
  if (nb <= 1) return stream_launch<G, 1, false>(p, st);
  if (nb <= 4) return stream_launch<G, 4, false>(p, st);
  return stream_launch<G, 8, false>(p, st);
}

// 0: launched (or a launch error code < 0); 1: not a shape for the streaming kernel
int gemv_stream_launch(const GemvW8Params& p, bool pair, cudaStream_t st) {
  if (!p.wa.plain1 || (pair && !p.wb.plain1) || p.K > 4096) return 1;
  switch (p.wa.G) {
    case 32: return stream_launch_g<32>(p, pair, st);
    case 64: return stream_launch_g<64>(p, pair, st);
    case 128: return stream_launch_g<128>(p, pair, st);
  }
  return 1;
}

}  // namespace iron
