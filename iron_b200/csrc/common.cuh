// Shared device/host helpers for the iron_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/iron_b200.h"

// ---------------------------------------------------------------------------
// host-side error reporting (thread-local message, negative status codes)
// ---------------------------------------------------------------------------
int iron_set_error(int code, const char* fmt, ...);
// cudaGetLastError after a launch: a negative code on failure, else counts the launch
int iron_check_launch(const char* what);
// counts a launch whose status was checked another way (iron_launch_count)
void iron_count_launch();

#define IRON_REQUIRE(cond, code, ...)                                  \
  do {                                                                 \
    if (!(cond)) return iron_set_error((code), __VA_ARGS__);           \
  } while (0)

static inline bool iron_aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

// number of SMs of the current device (cached per device)
int iron_num_sms();

// ---------------------------------------------------------------------------
// bf16 <-> f32
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(uint32_t b16) { return __uint_as_float(b16 << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// round a float to the nearest bf16 value (returned as float)
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }
// round a double to the nearest bf16 value through float32 (the f64 -> f32 -> bf16
// path of a float64 result stored by a float32 program)
__device__ __forceinline__ float rbf_d(double d) { return rbf((float)d); }
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
// Streaming 16-byte load for data read exactly once (weights, KV): read-only
// path, no L1 allocation, 256-byte L2 prefetch.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------
// warp reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// block-wide double sum for blockDim.x <= 1024; `red` holds >= 32 doubles
__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  double t = lane < nw ? red[lane] : 0.0;
  return warp_sum_d(t);
}

// block-wide sum for blockDim.x <= 1024; `red` holds >= 32 floats
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ---------------------------------------------------------------------------
// block floating point for activations
// ---------------------------------------------------------------------------
// A group of bf16 values with max magnitude m (2^(e-1) <= m < 2^e) is stored as
// int16 X_i = x_i * 2^(15-e), exact for every element within 7 binades of m
// (bf16 carries 8 significant bits) and |X_i| <= 32640.  The group factor
// 2^(e-15) is kept as a float.  Returns the factor and the scale to apply.
__device__ __forceinline__ void bfp_scale(float m, float& sc, float& inv) {
  uint32_t eb = (__float_as_uint(m) >> 23) & 0xffu;  // biased exponent of m
  if (eb == 0u) {  // zero or subnormal group -> all zero
    sc = 0.f;
    inv = 0.f;
    return;
  }
  int e = (int)eb - 126;           // m < 2^e
  int se = 127 + 15 - e;           // biased exponent of 2^(15-e)
  int ie = 127 + e - 15;           // biased exponent of 2^(e-15)
  se = se < 1 ? 1 : (se > 254 ? 254 : se);
  ie = ie < 1 ? 1 : (ie > 254 ? 254 : ie);
  sc = __uint_as_float((uint32_t)se << 23);
  inv = __uint_as_float((uint32_t)ie << 23);
}

// Weighted RMSNorm in two numerical forms.  The sum of squares is kept in
// float64 in both, so it does not depend on the reduction order.
//  mode 0 (kernel form, aie_kernels/aie2p/rms_norm.cc:9-53): x * w / sqrt(mean(x^2)
//    + eps) evaluated in float64 and rounded once (through float32) to bf16.
//  mode 1 (golden form, rms_norm/reference.py:8-17 on bf16 tensors): every
//    torch op rounds to bf16 -- x^2, mean, + eps, sqrt, x / rms, * w.
//  mode 2 (Llama form, llama_cpu.py:41-46 on bf16 tensors): x^2, mean, + eps,
//    rsqrt (correctly rounded), x * r, w * . each rounded to bf16.
struct RmsCoef {
  double inv;
  float rms;
  int mode;
};
__device__ __forceinline__ double rms_sq(float v, int mode) {
  const float s = v * v;  // exact in float64; rounded to float32 by mode 1 only
  return mode ? (double)rbf(s) : (double)v * (double)v;
}
__device__ __forceinline__ RmsCoef rms_coef(double sum_sq, int n, float eps, int mode) {
  RmsCoef c;
  c.mode = mode;
  // the mean: a multiply when n is a power of two (1/n exact, the same value as the divide)
  const double mean_sq = (n & (n - 1)) == 0 ? sum_sq * (1.0 / (double)n) : sum_sq / (double)n;
  if (mode == 0) {
    c.inv = 1.0 / sqrt(mean_sq + (double)eps);
    c.rms = 0.f;
  } else if (mode == 1) {
    const float mean = rbf((float)mean_sq);
    const float ms = rbf(mean + eps);
    c.rms = rbf(sqrtf(ms));
    c.inv = 0.0;
  } else {  // mode 2: c.rms holds r = bf16(rsqrt(bf16(mean + eps)))
    const float mean = rbf((float)mean_sq);
    const float ms = rbf(mean + eps);
    c.rms = rbf((float)(1.0 / sqrt((double)ms)));
    c.inv = 0.0;
  }
  return c;
}
// normalised, weighted value before the final bf16 rounding
__device__ __forceinline__ float rms_apply(float v, float w, const RmsCoef& c) {
  if (c.mode == 0) return (float)((double)v * c.inv * (double)w);
  return c.mode == 1 ? rbf(v / c.rms) * w : w * rbf(v * c.rms);
}

// sigmoid via tanh with bf16 rounding after every vector op, the arithmetic of
// aie_kernels/aie2p/silu.cc (golden: swiglu_mlp_dp/test.py:70-76)
__device__ __forceinline__ float silu_tanh_bf16(float g /* bf16 value */) {
  float th = rbf((float)tanh((double)(g * 0.5f)));
  float op = rbf(th + 1.0f);
  float sg = rbf(op * 0.5f);
  return rbf(g * sg);
}
