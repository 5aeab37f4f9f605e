// int8 group-quantised GEMV (W8A16) for decode: batch 1..8 activation rows.
//
// Numerics.  The weight stays int8 in registers.  The activations are staged
// once per CTA in shared memory as int16 block floating point per quant group
// (see bfp_scale), so the inner product of one 16-byte weight chunk is 8 dp2a
// instructions with exact int32 accumulation; the group scale
// s[m,g] * 2^(e_g - 15) is applied once per chunk in float32.  With LO (used at
// batch 1) each activation also carries a second int16 word holding the next 15
// bits, X = X_hi + X_lo 2^-15, which makes the staging exact for every bf16
// value within 22 binades of its group maximum; a second dp2a pass adds it.
// The result is the exact dequantised product sum_k q*s*x (GEMVInt8.reference,
// gemv_int8/op.py:173-178) up to float32 accumulation; the kernel-faithful
// golden (gemv_int8/reference.py:25-40) approximates the same sum with its
// premultiplied bf16(x*s) activations.
//
// Work split.  A CTA is 8 warps.  `ks` warps share one group of NR rows along K
// (split-K inside the CTA, reduced through shared memory) so small-M GEMVs
// still spread over every SM; each warp streams 16-byte weight chunks of its NR
// rows with no L1 allocation.
#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {

template <int G, int NB, bool PAIR, bool LO>
__global__ void __launch_bounds__(256) gemv_w8_kernel(GemvW8Params p) {
  constexpr int NR = 4;                      // output rows per job
  constexpr int NRW = PAIR ? 2 * NR : NR;    // weight rows per job
  constexpr int NW = LO ? 2 : 1;             // int16 words per activation
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.K;
  const int KG = K / G;
  uint16_t* xq = (uint16_t*)smem;                                   // [NB][K] (hi words)
  uint16_t* xl = xq + (size_t)NB * K;                               // [NB][K] (lo words, LO only)
  double* red = (double*)(smem + (size_t)NW * NB * K * 2);          // [8][NRW][NB]
  double* misc = red + 8 * NRW * NB;                                // [32]
  float* xs = (float*)(misc + 32);                                  // [NB][KG]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nb = p.nb;

  // ---- prologue: activations -> (optionally RMS-normalised) bf16 -> int16 BFP ----
  for (int b = 0; b < NB; ++b) {
    const uint16_t* xr = p.x + (size_t)b * p.ld_x;
    if (b >= nb) {
      for (int i = tid; i < K; i += blockDim.x) xq[b * K + i] = 0;
      continue;
    }
    if (p.rms_w) {
      double ss = 0.0;
      for (int i = tid; i < K; i += blockDim.x) ss += rms_sq(bf2f(xr[i]), p.rms_mode);
      ss = block_sum_d(ss, misc);
      const RmsCoef rc = rms_coef(ss, K, p.eps, p.rms_mode);
      for (int i = tid; i < K; i += blockDim.x)
        xq[b * K + i] = f2bf(rms_apply(bf2f(xr[i]), bf2f(p.rms_w[i]), rc));
    } else {
      for (int i = tid; i < K; i += blockDim.x) xq[b * K + i] = xr[i];
    }
  }
  __syncthreads();
  {
    constexpr int PER = G / 32;  // elements per lane in one group
    for (int gi = wid; gi < NB * KG; gi += 8) {
      const int b = gi / KG, g = gi - b * KG;
      uint16_t* base = xq + b * K + g * G + lane * PER;
      float v[PER];
      float m = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        v[e] = bf2f(base[e]);
        m = fmaxf(m, fabsf(v[e]));
      }
      m = warp_max(m);
      float sc, inv;
      bfp_scale(m, sc, inv);
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const float t = v[e] * sc;  // exact: v is bf16, sc a power of two
        const int hi = __float2int_rn(t);
        base[e] = (uint16_t)(int16_t)hi;
        if (LO) xl[(base - xq) + e] = (uint16_t)(int16_t)__float2int_rn((t - (float)hi) * 32768.0f);
      }
      if (lane == 0) xs[b * KG + g] = inv;
    }
  }
  __syncthreads();

  // ---- main loop ----
  const int KS = p.ksplit, RG = 8 / KS;
  const int rg = wid / KS, ks = wid - rg * KS;
  const int nchunk = K >> 4;
  const int njobs = (p.M + NR - 1) / NR;
  const uint32_t xm = p.xor_mask;
  for (int job0 = blockIdx.x * RG; job0 < njobs; job0 += gridDim.x * RG) {
    const int job = job0 + rg;
    double acc[NRW][NB];  // float64: the integer chunk sums are exact, so is their sum
#pragma unroll
    for (int r = 0; r < NRW; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.0;
    if (job < njobs) {
      const uint8_t* pw[NRW];
      const uint16_t* ps[NRW];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        int row = job * NR + r;
        row = row < p.M ? row : p.M - 1;
        wire_row(p.wa, row, pw[r], ps[r]);
        if (PAIR) wire_row(p.wb, row, pw[NR + r], ps[NR + r]);
      }
      for (int c = ks * 32 + lane; c < nchunk; c += 32 * KS) {
        uint4 wv[NRW];
#pragma unroll
        for (int r = 0; r < NRW; ++r) wv[r] = ldg_stream(pw[r] + (size_t)c * 16);
        const int g = (c * 16) / G;
        float sv[NRW];
#pragma unroll
        for (int r = 0; r < NRW; ++r) sv[r] = bf2f(__ldg(ps[r] + g));
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const uint4 xa = *(const uint4*)(xq + b * K + c * 16);
          const uint4 xb = *(const uint4*)(xq + b * K + c * 16 + 8);
          const float xsc = xs[b * KG + g];
          uint4 la = make_uint4(0, 0, 0, 0), lb = la;
          if (LO) {
            la = *(const uint4*)(xl + b * K + c * 16);
            lb = *(const uint4*)(xl + b * K + c * 16 + 8);
          }
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
              t = t * 32768 + l;  // X_hi 2^15 + X_lo, exact in int64
            }
            // sv * xsc is exact (bf16 times a power of two); so is the float64 product
            const double sc = LO ? (double)(sv[r] * xsc) * (1.0 / 32768.0) : (double)(sv[r] * xsc);
            acc[r][b] = fma((double)t, sc, acc[r][b]);
          }
        }
      }
    }
    // ---- reduce across lanes, then across the K-split warps ----
#pragma unroll
    for (int r = 0; r < NRW; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const double v = warp_sum_d(acc[r][b]);
        if (lane == 0) red[(wid * NRW + r) * NB + b] = v;
      }
    __syncthreads();
    if (ks == 0 && job < njobs && lane < NR * NB) {
      const int r = lane / NB, b = lane - (lane / NB) * NB;
      const int row = job * NR + r;
      if (row < p.M && b < nb) {
        double s0 = 0.0, s1 = 0.0;
        for (int s = 0; s < KS; ++s) {
          s0 += red[((rg * KS + s) * NRW + r) * NB + b];
          if (PAIR) s1 += red[((rg * KS + s) * NRW + NR + r) * NB + b];
        }
        uint16_t* yo = p.y + (size_t)b * p.ld_y + row;
        if (PAIR) {
          // gh = bf16(silu_tanh(bf16(g)) * bf16(u))  (swiglu_mlp_dp/test.py:87-89)
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
    __syncthreads();
  }
}

template <int G, int NB, bool PAIR, bool LO = (NB == 1)>
static int launch_t(const GemvW8Params& p, cudaStream_t st) {
  constexpr int NRW = PAIR ? 8 : 4;
  const size_t smem = (size_t)(LO ? 2 : 1) * NB * p.K * 2 + 8 * NRW * NB * 8 + 32 * 8 + (size_t)NB * (p.K / G) * 4;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(gemv_w8_kernel<G, NB, PAIR, LO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         227 * 1024);
    attr_set[dev] = true;
  }
  if (smem > 227 * 1024)
    return iron_set_error(IRON_ERR_UNSUPPORTED, "gemv_w8: K=%d x batch=%d needs %zu B of shared memory",
                          p.K, p.nb, smem);
  const int njobs = (p.M + 3) / 4;
  const int RG = 8 / p.ksplit;
  int grid = (njobs + RG - 1) / RG;
  const int per_sm = smem > 100 * 1024 ? 1 : (smem > 64 * 1024 ? 2 : 4);
  const int maxgrid = iron_num_sms() * per_sm;
  if (grid > maxgrid) grid = maxgrid;
  gemv_w8_kernel<G, NB, PAIR, LO><<<grid, 256, smem, st>>>(p);
  return iron_check_launch("gemv_w8_kernel");
}

template <int G>
static int launch_g(const GemvW8Params& p, bool pair, cudaStream_t st) {
  const int nb = p.nb;
  if (pair) {
    if (nb <= 1) return launch_t<G, 1, true>(p, st);
    if (nb <= 2) return launch_t<G, 2, true>(p, st);
    if (nb <= 4) return launch_t<G, 4, true>(p, st);
    return launch_t<G, 8, true>(p, st);
  }
  if (nb <= 1) return launch_t<G, 1, false>(p, st);
  if (nb <= 2) return launch_t<G, 2, false>(p, st);
  if (nb <= 4) return launch_t<G, 4, false>(p, st);
  return launch_t<G, 8, false>(p, st);
}

int make_wire(Wire& w, const void* base, int M, int K, int group, int tile_m, int rows_per_core,
              int tiles_per_core, int domain) {
  IRON_REQUIRE(base != nullptr, IRON_ERR_ARG, "wire: null pointer");
  IRON_REQUIRE(group == 32 || group == 64 || group == 128, IRON_ERR_ARG,
               "wire: group must be 32, 64 or 128 (got %d)", group);
  IRON_REQUIRE(K > 0 && K % group == 0 && K % 16 == 0, IRON_ERR_ARG,
               "wire: K=%d must be a positive multiple of group=%d and of 16", K, group);
  IRON_REQUIRE(M > 0 && tile_m > 0, IRON_ERR_ARG, "wire: M=%d, tile_m=%d must be positive", M, tile_m);
  if (rows_per_core <= 0) rows_per_core = M;
  if (tiles_per_core <= 0) tiles_per_core = (rows_per_core + tile_m - 1) / tile_m;
  IRON_REQUIRE(rows_per_core % tile_m == 0 || tiles_per_core * tile_m >= rows_per_core, IRON_ERR_ARG,
               "wire: %d tiles of %d rows cannot hold a %d-row window", tiles_per_core, tile_m,
               rows_per_core);
  IRON_REQUIRE(domain == 0 || domain == 1, IRON_ERR_ARG, "wire: domain must be 0 (signed) or 1 (biased)");
  const long long tile_bytes = (long long)tile_m * (K + 2 * (K / group));
  IRON_REQUIRE(tile_bytes % 16 == 0 && iron_aligned(base, 16), IRON_ERR_ALIGN,
               "wire: tiles of %lld bytes / base %p are not 16-byte aligned", tile_bytes, base);
  w.base = (const uint8_t*)base;
  w.K = K;
  w.G = group;
  w.tile_m = tile_m;
  w.rows_per_core = rows_per_core;
  w.tiles_per_core = tiles_per_core;
  w.tile_bytes = tile_bytes;
  w.plain1 = (tile_m == 1 && rows_per_core >= M) ? 1 : 0;
  w.xor_mask = domain == 1 ? 0x80808080u : 0u;
  return IRON_OK;
}

static int gemv_w8_launch_rows(GemvW8Params p, bool pair, cudaStream_t st);
int gemv_mma_launch(const GemvW8Params& p, bool pair, cudaStream_t st);

// Batches of 9..15 (and larger ones the tensor-core kernel does not take) run as
// successive launches over 8 activation rows each (the weight streams once per
// launch): the batch-8 kernel's arithmetic for every row.
int gemm_tc_launch(const GemvW8Params& p, bool pair, cudaStream_t st);

int gemv_w8_launch(GemvW8Params p, bool pair, cudaStream_t st) {
  IRON_REQUIRE(p.nb >= 1, IRON_ERR_UNSUPPORTED, "gemv_w8: batch %d below 1", p.nb);
  if (p.nb <= 8) return gemv_w8_launch_rows(p, pair, st);
  // 16 streams and more: one tensor-core contraction that streams the weight once (gemm_tc.cu)
  if (p.nb >= 16 && (!pair || p.wa.xor_mask == p.wb.xor_mask)) {
    const int rc = gemm_tc_launch(p, pair, st);
    if (rc <= 0) return rc;
  }
  for (int b0 = 0; b0 < p.nb; b0 += 8) {
    const int rc = gemv_w8_launch_rows(gemv_rows(p, b0, p.nb - b0 < 8 ? p.nb - b0 : 8), pair, st);
    if (rc) return rc;
  }
  return IRON_OK;
}

static int gemv_w8_launch_rows(GemvW8Params p, bool pair, cudaStream_t st) {
  IRON_REQUIRE(p.nb >= 1 && p.nb <= 8, IRON_ERR_UNSUPPORTED, "gemv_w8: batch %d not in 1..8", p.nb);
  IRON_REQUIRE(p.M > 0 && p.K > 0, IRON_ERR_ARG, "gemv_w8: empty shape M=%d K=%d", p.M, p.K);
  IRON_REQUIRE(p.x && p.y, IRON_ERR_ARG, "gemv_w8: null x / y");
  IRON_REQUIRE(iron_aligned(p.x, 4) && p.ld_x % 2 == 0, IRON_ERR_ALIGN, "gemv_w8: x must be 4-byte aligned");
  if (pair && p.wa.xor_mask != p.wb.xor_mask)
    return iron_set_error(IRON_ERR_ARG, "gemv_w8: paired wires must share a payload domain");
  p.xor_mask = p.wa.xor_mask;
  // plain wires: exact integer tensor-core dot products over a bulk-copy ring (gemv_mma.cu)
  const int mrc = gemv_mma_launch(p, pair, st);
  if (mrc <= 0) return mrc;
  // split K inside the CTA until the grid covers the GPU (at least one chunk per lane)
  const int njobs = (p.M + 3) / 4;
  int ks = 1;
  while (ks < 8 && ((njobs + (8 / ks) - 1) / (8 / ks)) < 2 * iron_num_sms() && (p.K / 16) >= 64 * ks)
    ks *= 2;
  p.ksplit = ks;
  switch (p.wa.G) {
    case 32: return launch_g<32>(p, pair, st);
    case 64: return launch_g<64>(p, pair, st);
    case 128: return launch_g<128>(p, pair, st);
  }
  return iron_set_error(IRON_ERR_ARG, "gemv_w8: bad group %d", p.wa.G);
}

// ---------------------------------------------------------------------------
// dequantise / quantise (bit-exact helpers for the wire format)
// ---------------------------------------------------------------------------
__global__ void dequant_w8_kernel(Wire w, int M, float* out) {
  const int row = blockIdx.x;
  if (row >= M) return;
  const uint8_t* pw;
  const uint16_t* ps;
  wire_row(w, row, pw, ps);
  for (int k = threadIdx.x; k < w.K; k += blockDim.x) {
    const int8_t q = (int8_t)(pw[k] ^ (uint8_t)(w.xor_mask & 0xffu));
    out[(size_t)row * w.K + k] = (float)q * bf2f(ps[k / w.G]);
  }
}

// one warp per (row, group); torch semantics of Qwen3NPU._set_int8_rtn
__global__ void quantize_rtn_kernel(const uint16_t* wsrc, int M, int K, int G, Wire w) {
  const int lane = threadIdx.x & 31;
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int KG = K / G;
  if (gid >= (long long)M * KG) return;
  const int row = (int)(gid / KG), g = (int)(gid - (long long)row * KG);
  const uint16_t* src = wsrc + (size_t)row * K + (size_t)g * G;
  float m = 0.f;
  for (int i = lane; i < G; i += 32) m = fmaxf(m, fabsf(bf2f(src[i])));
  m = warp_max(m);
  float s = m / 127.0f;
  if (!(s > 0.f)) s = 1.0f;
  const uint16_t sb = f2bf(s);
  const float sw = bf2f(sb);
  uint8_t* pw;
  uint16_t* ps;
  {
    const uint8_t* cpw;
    const uint16_t* cps;
    wire_row(w, row, cpw, cps);
    pw = (uint8_t*)cpw;
    ps = (uint16_t*)cps;
  }
  for (int i = lane; i < G; i += 32) {
    float q = rintf(bf2f(src[i]) / sw);
    q = fminf(fmaxf(q, -127.f), 127.f);
    pw[g * G + i] = (uint8_t)((int8_t)(int)q) ^ (uint8_t)(w.xor_mask & 0xffu);
  }
  if (lane == 0) ps[g] = sb;
}

}  // namespace iron

using namespace iron;

extern "C" int iron_gemv_w8a16(const void* wire, int M, int K, int group, int tile_m,
                               int rows_per_core, int tiles_per_core, int domain,
                               const uint16_t* x, int batch, const uint16_t* residual,
                               uint16_t* y, void* workspace, int64_t workspace_bytes, void* stream) {
  GemvW8Params p = {};
  p.tc_ws = workspace;
  p.tc_ws_bytes = workspace_bytes;
  int rc = make_wire(p.wa, wire, M, K, group, tile_m, rows_per_core, tiles_per_core, domain);
  if (rc) return rc;
  p.wb = p.wa;
  p.M = M;
  p.K = K;
  p.x = x;
  p.ld_x = K;
  p.nb = batch;
  p.res = residual;
  p.y = y;
  p.ld_y = M;
  p.epi = residual ? EPI_RESID : EPI_STORE;
  return gemv_w8_launch(p, false, (cudaStream_t)stream);
}

extern "C" int iron_dequant_w8(const void* wire, int M, int K, int group, int tile_m,
                               int rows_per_core, int tiles_per_core, int domain, float* out,
                               void* stream) {
  Wire w;
  int rc = make_wire(w, wire, M, K, group, tile_m, rows_per_core, tiles_per_core, domain);
  if (rc) return rc;
  IRON_REQUIRE(out != nullptr, IRON_ERR_ARG, "dequant: null output");
  dequant_w8_kernel<<<M, 256, 0, (cudaStream_t)stream>>>(w, M, out);
  return iron_check_launch("dequant_w8_kernel");
}

extern "C" int iron_quantize_rtn(const uint16_t* wsrc, int M, int K, int group, int tile_m,
                                 int domain, void* wire_out, void* stream) {
  Wire w;
  IRON_REQUIRE(wsrc != nullptr, IRON_ERR_ARG, "quantize: null input");
  IRON_REQUIRE(M % tile_m == 0, IRON_ERR_ARG, "quantize: tile_m=%d must divide M=%d", tile_m, M);
  int rc = make_wire(w, wire_out, M, K, group, tile_m, 0, 0, domain);
  if (rc) return rc;
  const long long groups = (long long)M * (K / group);
  const int wpb = 8;
  const long long blocks = (groups + wpb - 1) / wpb;
  quantize_rtn_kernel<<<(unsigned)blocks, wpb * 32, 0, (cudaStream_t)stream>>>(wsrc, M, K, group, w);
  return iron_check_launch("quantize_rtn_kernel");
}
