// Building blocks of tensor-parallel decode (Qwen3-8B over 1/2/4/8 GPUs).
//
// The reference runs one NPU and has no tensor parallelism; these entry points
// split its fused blocks at the points where a rank's partial result must be summed
// over the ranks (the O and down projections, row-parallel along K) or compared
// across them (the vocabulary-parallel greedy argmax):
//   - iron_gemv_w8a16_ex: the int8 GEMV with every epilogue exposed (float32
//     partial sums, residual, RMS-normalised gate/up pair);
//   - iron_resid_add_f32: y = bf16(res + bf16(sum)), the residual add of a summed
//     partial (the same roundings as the GEMV's residual epilogue);
//   - iron_argmax_pair / iron_argmax_merge: a rank's (value, global index) of its
//     local argmax, and the greedy token over all ranks' pairs (ties -> lowest
//     index, as numpy.argmax).
#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {

__global__ void resid_add_f32_kernel(const uint16_t* res, const float* sum, uint16_t* y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = f2bf(bf2f(res[i]) + rbf(sum[i]));
}

__global__ void argmax_pair_kernel(const uint16_t* logits, int M, int batch, const int32_t* tok, int offset,
                                   int32_t* pairs) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  int t = tok[b];
  t = t < 0 ? 0 : (t >= M ? M - 1 : t);
  pairs[2 * b] = __float_as_int(bf2f(logits[(size_t)b * M + t]));
  pairs[2 * b + 1] = t + offset;
}

__global__ void argmax_merge_kernel(const int32_t* pairs, int n, int batch, int32_t* tok_out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float best = -INFINITY;
  int idx = -1;
  for (int r = 0; r < n; ++r) {
    const float v = __int_as_float(pairs[((size_t)r * batch + b) * 2]);
    const int i = pairs[((size_t)r * batch + b) * 2 + 1];
    if (idx < 0 || v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  tok_out[b] = idx;
}

}  // namespace iron

using namespace iron;

extern "C" int iron_gemv_w8a16_ex(const void* wire_a, const void* wire_b, int M, int K, int group, int domain,
                                  const uint16_t* x, int ld_x, int batch, const uint16_t* rms_w, float eps,
                                  int rms_mode, const uint16_t* residual, int epi, void* y, int ld_y,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  IRON_REQUIRE(wire_a && x && y, IRON_ERR_ARG, "gemv_ex: null pointer");
  IRON_REQUIRE(epi >= 0 && epi <= 2, IRON_ERR_ARG, "gemv_ex: epilogue %d not in 0..2", epi);
  IRON_REQUIRE(epi != 1 || residual, IRON_ERR_ARG, "gemv_ex: the residual epilogue needs a residual");
  IRON_REQUIRE(!wire_b || epi == 0, IRON_ERR_ARG, "gemv_ex: a gate/up pair stores bf16 (epilogue 0)");
  IRON_REQUIRE(rms_mode == 0 || rms_mode == 1, IRON_ERR_ARG, "gemv_ex: rms_mode must be 0 or 1");
  IRON_REQUIRE(ld_x >= K && ld_y >= M, IRON_ERR_ARG, "gemv_ex: ld_x %d < K %d or ld_y %d < M %d", ld_x, K, ld_y, M);
  IRON_REQUIRE(!rms_w || iron_aligned(rms_w, 2), IRON_ERR_ALIGN, "gemv_ex: rms_w misaligned");
  GemvW8Params p = {};
  int rc = make_wire(p.wa, wire_a, M, K, group, 1, 0, 0, domain);
  if (rc) return rc;
  if (wire_b) {
    rc = make_wire(p.wb, wire_b, M, K, group, 1, 0, 0, domain);
    if (rc) return rc;
  } else {
    p.wb = p.wa;
  }
  p.M = M;
  p.K = K;
  p.x = x;
  p.ld_x = ld_x;
  p.rms_w = rms_w;
  p.eps = eps;
  p.rms_mode = rms_mode;
  p.res = residual;
  p.y = (uint16_t*)y;
  p.ld_y = ld_y;
  p.nb = batch;
  p.epi = epi;
  p.tc_ws = workspace;
  p.tc_ws_bytes = workspace_bytes;
  return gemv_w8_launch(p, wire_b != nullptr, (cudaStream_t)stream);
}

extern "C" int iron_resid_add_f32(const uint16_t* res, const float* sum, uint16_t* y, int64_t n, void* stream) {
  IRON_REQUIRE(res && sum && y && n >= 0, IRON_ERR_ARG, "resid_add_f32: bad arguments");
  if (n == 0) return IRON_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 4 * iron_num_sms()) grid = 4 * iron_num_sms();
  resid_add_f32_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(res, sum, y, n);
  return iron_check_launch("resid_add_f32_kernel");
}

extern "C" int iron_argmax_pair(const uint16_t* logits, int M, int batch, const int32_t* tok, int offset,
                                int32_t* pairs, void* stream) {
  IRON_REQUIRE(logits && tok && pairs && M > 0 && batch >= 1, IRON_ERR_ARG, "argmax_pair: bad arguments");
  argmax_pair_kernel<<<(batch + 127) / 128, 128, 0, (cudaStream_t)stream>>>(logits, M, batch, tok, offset, pairs);
  return iron_check_launch("argmax_pair_kernel");
}

extern "C" int iron_argmax_merge(const int32_t* pairs, int n, int batch, int32_t* tok_out, void* stream) {
  IRON_REQUIRE(pairs && tok_out && n >= 1 && batch >= 1, IRON_ERR_ARG, "argmax_merge: bad arguments");
  argmax_merge_kernel<<<(batch + 127) / 128, 128, 0, (cudaStream_t)stream>>>(pairs, n, batch, tok_out);
  return iron_check_launch("argmax_merge_kernel");
}
