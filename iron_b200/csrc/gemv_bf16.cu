// bf16 GEMV (lm_head, Llama-shape projections) and greedy argmax.
//
// Each warp streams NR=4 weight rows as 16-byte chunks (8 bf16) with no L1
// allocation; the activations sit in shared memory as float32.  The optional
// argmax epilogue keeps, per CTA, the best (bf16-rounded logit, lowest index)
// pair per batch row and writes it to a candidate list that a one-CTA pass
// reduces -- the same tie rule as numpy.argmax over the bf16 logits the
// reference's host argmax sees (qwen3_npu_int8.py:615-620).
#include "common.cuh"

namespace iron {

struct GemvBf16Params {
  const uint16_t* A;
  int M, K;
  const uint16_t* x;
  int nb;
  int independent;     // x row b multiplies its own matrix A + b*M*K
  uint16_t* y;         // may be null (argmax only)
  float* cand_val;     // [nb][gridDim.x] or null
  int* cand_idx;
  int ksplit;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <int NB>
__global__ void __launch_bounds__(256) gemv_bf16_kernel(GemvBf16Params p) {
  constexpr int NR = 4;
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = p.K;
  float* xf = (float*)smem;                 // [NB][K]
  float* red = xf + NB * K;                 // [8][NR][NB]
  float* bestv = red + 8 * NR * NB;         // [8][NB]
  int* besti = (int*)(bestv + 8 * NB);      // [8][NB]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nb = p.independent ? 1 : p.nb;
  const int bsel = p.independent ? blockIdx.y : 0;
  const uint16_t* A = p.A + (p.independent ? (size_t)bsel * p.M * K : 0);
  const uint16_t* xsrc = p.x + (size_t)bsel * K;
  for (int i = tid; i < NB * K; i += blockDim.x) {
    const int b = i / K;
    xf[i] = b < nb ? bf2f(xsrc[i]) : 0.f;
  }
  float myv[NB];
  int myi[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    myv[b] = -INFINITY;
    myi[b] = 0x7fffffff;
  }
  __syncthreads();

  const int KS = p.ksplit, RG = 8 / KS;
  const int rg = wid / KS, ks = wid - rg * KS;
  const int nchunk = K >> 3;
  const int njobs = (p.M + NR - 1) / NR;
  for (int job0 = blockIdx.x * RG; job0 < njobs; job0 += gridDim.x * RG) {
    const int job = job0 + rg;
    float acc[NR][NB];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
    if (job < njobs) {
      const uint16_t* pr[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        int row = job * NR + r;
        row = row < p.M ? row : p.M - 1;
        pr[r] = A + (size_t)row * K;
      }
      for (int c = ks * 32 + lane; c < nchunk; c += 32 * KS) {
        uint4 wv[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) wv[r] = ldg_stream(pr[r] + (size_t)c * 8);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float4 x0 = *(const float4*)(xf + b * K + c * 8);
          const float4 x1 = *(const float4*)(xf + b * K + c * 8 + 4);
#pragma unroll
          for (int r = 0; r < NR; ++r) {
            float a = acc[r][b];
            a = fmaf(bf_lo(wv[r].x), x0.x, a);
            a = fmaf(bf_hi(wv[r].x), x0.y, a);
            a = fmaf(bf_lo(wv[r].y), x0.z, a);
            a = fmaf(bf_hi(wv[r].y), x0.w, a);
            a = fmaf(bf_lo(wv[r].z), x1.x, a);
            a = fmaf(bf_hi(wv[r].z), x1.y, a);
            a = fmaf(bf_lo(wv[r].w), x1.z, a);
            a = fmaf(bf_hi(wv[r].w), x1.w, a);
            acc[r][b] = a;
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float v = warp_sum(acc[r][b]);
        if (lane == 0) red[(wid * NR + r) * NB + b] = v;
      }
    __syncthreads();
    if (ks == 0 && job < njobs && lane < NR * NB) {
      const int r = lane / NB, b = lane - (lane / NB) * NB;
      const int row = job * NR + r;
      if (row < p.M && b < nb) {
        float s = 0.f;
        for (int q = 0; q < KS; ++q) s += red[((rg * KS + q) * NR + r) * NB + b];
        const uint16_t o = f2bf(s);
        const int ob = p.independent ? bsel : b;
        if (p.y) p.y[(size_t)ob * p.M + row] = o;
        const float v = bf2f(o);
#pragma unroll
        for (int bb = 0; bb < NB; ++bb)
          if (bb == b && better(v, row, myv[bb], myi[bb])) {
            myv[bb] = v;
            myi[bb] = row;
          }
      }
    }
    __syncthreads();
  }
  if (p.cand_val) {
    // per-warp best (lanes hold disjoint rows), then per-CTA best
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = myv[b];
      int i = myi[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, v, o);
        int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
          v = ov;
          i = oi;
        }
      }
      if (lane == 0) {
        bestv[wid * NB + b] = v;
        besti[wid * NB + b] = i;
      }
    }
    __syncthreads();
    if (tid < NB && tid < nb) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int w = 0; w < 8; ++w)
        if (better(bestv[w * NB + tid], besti[w * NB + tid], v, i)) {
          v = bestv[w * NB + tid];
          i = besti[w * NB + tid];
        }
      p.cand_val[tid * gridDim.x + blockIdx.x] = v;
      p.cand_idx[tid * gridDim.x + blockIdx.x] = i;
    }
  }
}

// one CTA per batch row: reduce n candidates to the final token
__global__ void argmax_reduce_kernel(const float* cv, const int* ci, int n, int32_t* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  float v = -INFINITY;
  int i = 0x7fffffff;
  for (int k = threadIdx.x; k < n; k += blockDim.x)
    if (better(cv[b * n + k], ci[b * n + k], v, i)) {
      v = cv[b * n + k];
      i = ci[b * n + k];
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sv[wid] = v;
    si[wid] = i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], v, i)) {
        v = sv[w];
        i = si[w];
      }
    out[b] = i;
  }
}

// argmax over existing bf16 logits: grid-stride candidate pass
__global__ void argmax_bf16_kernel(const uint16_t* lg, int M, int nb, float* cv, int* ci) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int b = 0; b < nb; ++b) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
      const float x = bf2f(lg[(size_t)b * M + m]);
      if (better(x, m, v, i)) {
        v = x;
        i = m;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, v, o);
      int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) {
      sv[wid] = v;
      si[wid] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (better(sv[w], si[w], v, i)) {
          v = sv[w];
          i = si[w];
        }
      cv[b * gridDim.x + blockIdx.x] = v;
      ci[b * gridDim.x + blockIdx.x] = i;
    }
    __syncthreads();
  }
}

static const int kMaxCand = 1024;  // candidate slots per batch row

template <int NB>
static int launch_bf16(GemvBf16Params p, cudaStream_t st, int gridy) {
  const size_t smem = (size_t)NB * p.K * 4 + 8 * 4 * NB * 4 + 8 * NB * 8;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(gemv_bf16_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr[dev] = true;
  }
  if (smem > 227 * 1024)
    return iron_set_error(IRON_ERR_UNSUPPORTED, "gemv_bf16: K=%d x batch=%d exceeds shared memory", p.K, p.nb);
  const int njobs = (p.M + 3) / 4;
  int ks = 1;
  while (ks < 8 && ((njobs + (8 / ks) - 1) / (8 / ks)) < 2 * iron_num_sms() && (p.K / 8) >= 64 * ks) ks *= 2;
  p.ksplit = ks;
  const int RG = 8 / ks;
  int grid = (njobs + RG - 1) / RG;
  const int per_sm = smem > 100 * 1024 ? 1 : (smem > 48 * 1024 ? 2 : 4);
  int maxgrid = iron_num_sms() * per_sm;
  if (maxgrid > kMaxCand) maxgrid = kMaxCand;
  if (grid > maxgrid) grid = maxgrid;
  dim3 g(grid, gridy);
  gemv_bf16_kernel<NB><<<g, 256, smem, st>>>(p);
  return grid;
}

static int gemv_bf16_dispatch(GemvBf16Params p, cudaStream_t st) {
  IRON_REQUIRE(p.A && p.x && p.M > 0 && p.K > 0, IRON_ERR_ARG, "gemv_bf16: bad arguments");
  IRON_REQUIRE(p.K % 8 == 0 && iron_aligned(p.A, 16) && iron_aligned(p.x, 4), IRON_ERR_ALIGN,
               "gemv_bf16: K=%d must be a multiple of 8 and A 16-byte aligned", p.K);
  IRON_REQUIRE(p.nb >= 1 && (p.independent || p.nb <= 8), IRON_ERR_UNSUPPORTED,
               "gemv_bf16: batch %d (shared weight) not in 1..8", p.nb);
  int grid;
  if (p.independent) {
    grid = launch_bf16<1>(p, st, p.nb);
  } else if (p.nb <= 1) {
    grid = launch_bf16<1>(p, st, 1);
  } else if (p.nb <= 2) {
    grid = launch_bf16<2>(p, st, 1);
  } else if (p.nb <= 4) {
    grid = launch_bf16<4>(p, st, 1);
  } else {
    grid = launch_bf16<8>(p, st, 1);
  }
  if (grid < 0) return grid;
  int rc = iron_check_launch("gemv_bf16_kernel");
  return rc ? rc : grid;
}

int gemm_tc_bf16_launch(const uint16_t* A, int M, int K, const uint16_t* x, int ld_x, int nb, uint16_t* y,
                        int ld_y, void* workspace, int64_t workspace_bytes, cudaStream_t st);

}  // namespace iron

using namespace iron;

extern "C" int64_t iron_argmax_workspace_bytes(int batch) {
  return (int64_t)batch * kMaxCand * 8;
}

extern "C" int64_t iron_tc_workspace_bytes(int M, int K, int batch);

// Batch 16+ with iron_lm_head_workspace_bytes: [tensor-core scratch (its status word
// first) | argmax candidates | logits when the caller keeps none]; smaller workspaces
// and batch 1..15: the argmax candidates from offset 0.
extern "C" int64_t iron_lm_head_workspace_bytes(int M, int K, int batch) {
  const int64_t am = (iron_argmax_workspace_bytes(batch) + 255) & ~(int64_t)255;
  if (batch < 16) return am;
  return iron_tc_workspace_bytes(M, K, batch) + am + (((int64_t)batch * M * 2 + 255) & ~(int64_t)255);
}

extern "C" int iron_gemv_bf16(const uint16_t* A, int M, int K, const uint16_t* x, int batch,
                              int independent, uint16_t* y, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  IRON_REQUIRE(y != nullptr, IRON_ERR_ARG, "gemv_bf16: null output");
  IRON_REQUIRE(batch >= 1, IRON_ERR_UNSUPPORTED, "gemv_bf16: batch %d below 1", batch);
  // 16+ rows of a shared weight: one tensor-core contraction (gemm_tc.cu)
  if (!independent && batch >= 16) {
    const int rc = gemm_tc_bf16_launch(A, M, K, x, K, batch, y, M, workspace, workspace_bytes, (cudaStream_t)stream);
    if (rc <= 0) return rc;
  }
  // a shared weight with more than 8 activation rows: launches over 8 rows each
  const int step = independent ? batch : 8;
  for (int b0 = 0; b0 < batch; b0 += step) {
    GemvBf16Params p = {};
    p.A = A;
    p.M = M;
    p.K = K;
    p.x = x + (size_t)b0 * K;
    p.nb = batch - b0 < step ? batch - b0 : step;
    p.independent = independent;
    p.y = y + (size_t)b0 * M;
    int g = gemv_bf16_dispatch(p, (cudaStream_t)stream);
    if (g < 0) return g;
  }
  return IRON_OK;
}

extern "C" int iron_lm_head_bf16_argmax(const uint16_t* A, int M, int K, const uint16_t* x,
                                        int batch, uint16_t* logits, int32_t* token_out,
                                        void* workspace, int64_t workspace_bytes, void* stream) {
  IRON_REQUIRE(workspace && token_out, IRON_ERR_ARG, "lm_head_argmax: null workspace/token_out");
  IRON_REQUIRE(workspace_bytes >= iron_argmax_workspace_bytes(batch), IRON_ERR_ARG,
               "lm_head_argmax: workspace below iron_lm_head_workspace_bytes");
  IRON_REQUIRE(batch >= 1, IRON_ERR_UNSUPPORTED, "lm_head_argmax: batch %d below 1", batch);
  cudaStream_t st = (cudaStream_t)stream;
  // 16+ rows: the logits from one tensor-core contraction, then the argmax passes
  if (batch >= 16 && workspace_bytes >= iron_lm_head_workspace_bytes(M, K, batch)) {
    const int64_t tcb = iron_tc_workspace_bytes(M, K, batch);
    const int64_t am = (iron_argmax_workspace_bytes(batch) + 255) & ~(int64_t)255;
    uint8_t* cand = (uint8_t*)workspace + tcb;
    uint16_t* L = logits ? logits : (uint16_t*)(cand + am);
    const int rc = gemm_tc_bf16_launch(A, M, K, x, K, batch, L, M, workspace, tcb, st);
    if (rc < 0) return rc;
    if (rc == 0) return iron_argmax_bf16(L, M, batch, token_out, cand, stream);
  }
  // up to 8 activation rows per launch; rows b0.. use the workspace's candidate slots
  // from b0 * kMaxCand on
  for (int b0 = 0; b0 < batch; b0 += 8) {
    const int nb = batch - b0 < 8 ? batch - b0 : 8;
    GemvBf16Params p = {};
    p.A = A;
    p.M = M;
    p.K = K;
    p.x = x + (size_t)b0 * K;
    p.nb = nb;
    p.y = logits ? logits + (size_t)b0 * M : nullptr;
    p.cand_val = (float*)workspace + (size_t)b0 * kMaxCand;
    p.cand_idx = (int*)((char*)workspace + (size_t)batch * kMaxCand * 4) + (size_t)b0 * kMaxCand;
    int grid = gemv_bf16_dispatch(p, st);
    if (grid < 0) return grid;
    argmax_reduce_kernel<<<nb, 256, 0, st>>>(p.cand_val, p.cand_idx, grid, token_out + b0);
    int rc = iron_check_launch("argmax_reduce_kernel");
    if (rc) return rc;
  }
  return IRON_OK;
}

extern "C" int iron_argmax_bf16(const uint16_t* logits, int M, int batch, int32_t* token_out,
                                void* workspace, void* stream) {
  IRON_REQUIRE(logits && workspace && token_out && M > 0 && batch >= 1, IRON_ERR_ARG,
               "argmax: bad arguments");
  cudaStream_t st = (cudaStream_t)stream;
  float* cv = (float*)workspace;
  int* ci = (int*)((char*)workspace + (size_t)batch * kMaxCand * 4);
  int grid = iron_num_sms() * 2;
  if (grid > kMaxCand) grid = kMaxCand;
  argmax_bf16_kernel<<<grid, 256, 0, st>>>(logits, M, batch, cv, ci);
  int rc = iron_check_launch("argmax_bf16_kernel");
  if (rc) return rc;
  argmax_reduce_kernel<<<batch, 256, 0, st>>>(cv, ci, grid, token_out);
  return iron_check_launch("argmax_reduce_kernel");
}
