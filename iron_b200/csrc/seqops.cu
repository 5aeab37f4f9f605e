// The data-movement and softmax operators of IRON's Llama decode runlist
// (iron/applications/llama_3.2_1b/llama_npu.py:279-557) on the B200:
//   iron_rope_rows      RoPE over (rows, cols) with a row-repeated angle table
//                       (iron/operators/rope/op.py, rope/reference.py:118-154);
//   iron_strided_copy   gather by one access pattern, scatter by another, with runtime
//                       offset addends (strided_copy/op.py, strided_copy/reference.py);
//   iron_repeat_rows    repeat-interleave of rows (repeat/op.py, repeat/reference.py);
//   iron_softmax_rows   row softmax over the first `vector_size` entries, the rest
//                       masked (softmax/op.py, softmax/design.py:86-103);
//   iron_transpose      batched (M, N) -> (N, M) transposes (transpose/op.py).
// They move bytes (or a few flops per byte): each is bound by HBM or by its launch.
#include "common.cuh"

namespace iron {

// ---------------------------------------------------------------------------
// RoPE: y1 = x1*c - x2*s, y2 = x2*c + x1*s in float32 with every product and sum
// rounded separately (no fused multiply-add, as the reference's float32 tensor ops),
// one bf16 rounding.  Method 0 (two halves) pairs columns j and j + cols/2, method 1
// (interleaved) columns 2j and 2j + 1; (c, s) is pair j of the interleaved angle row
// r / rep.  One thread owns one pair of a row, so y may alias x.
// ---------------------------------------------------------------------------
__global__ void rope_rows_kernel(const uint16_t* x, const uint16_t* ang, uint16_t* y, int rows, int cols,
                                 int rep, int method) {
  const int half = cols >> 1;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * half) return;
  const int r = (int)(i / half), j = (int)(i - (long long)r * half);
  const uint16_t* a = ang + (size_t)(r / rep) * cols;
  const float c = bf2f(a[2 * j]), s = bf2f(a[2 * j + 1]);
  const size_t o = (size_t)r * cols;
  const size_t i1 = o + (method == 0 ? j : 2 * j), i2 = o + (method == 0 ? half + j : 2 * j + 1);
  const float x1 = bf2f(x[i1]), x2 = bf2f(x[i2]);
  const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  y[i1] = f2bf(y1);
  y[i2] = f2bf(y2);
}

// ---------------------------------------------------------------------------
// Strided copy.  An access pattern is 4 (size, stride) pairs, outermost first, and an
// element offset; its elements are visited with the innermost index fastest.  The
// pattern's innermost non-empty dimension is cut into `channels` equal parts and part c
// of the input pairs with part c of the output, element by element (the channel split
// of the reference's DMA taps).  Runtime addends (elements) come from device slots.
// Elements whose source or destination falls outside its buffer are skipped and
// recorded in the error word.
// ---------------------------------------------------------------------------
struct Tap {
  long long size[4], stride[4];  // the per-channel split, outermost first
  long long offset, chan_step;   // first element; element distance between channels
};

struct CopyArgs {
  Tap in, out;
  long long per_channel, total, in_elems, out_elems;
  int elem_bytes;
  const int32_t* in_add;
  const int32_t* out_add;
  int32_t* err;
};

__device__ __forceinline__ long long tap_at(const Tap& t, long long c, long long e) {
  long long off = t.offset + c * t.chan_step;
#pragma unroll
  for (int d = 3; d >= 0; --d) {
    const long long sz = t.size[d] > 0 ? t.size[d] : 1;
    off += (e % sz) * t.stride[d];
    e /= sz;
  }
  return off;
}

__global__ void strided_copy_kernel(const uint8_t* in, uint8_t* out, CopyArgs a) {
  const long long ia = a.in_add ? (long long)*a.in_add : 0, oa = a.out_add ? (long long)*a.out_add : 0;
  for (long long f = (long long)blockIdx.x * blockDim.x + threadIdx.x; f < a.total;
       f += (long long)gridDim.x * blockDim.x) {
    const long long c = f / a.per_channel, e = f - c * a.per_channel;
    const long long s = tap_at(a.in, c, e) + ia, d = tap_at(a.out, c, e) + oa;
    if (s < 0 || s >= a.in_elems || d < 0 || d >= a.out_elems) {
      if (a.err) atomicExch(a.err, 1);
      continue;
    }
    switch (a.elem_bytes) {
      case 1: out[d] = in[s]; break;
      case 2: ((uint16_t*)out)[d] = ((const uint16_t*)in)[s]; break;
      case 4: ((uint32_t*)out)[d] = ((const uint32_t*)in)[s]; break;
      default: ((unsigned long long*)out)[d] = ((const unsigned long long*)in)[s]; break;
    }
  }
}

// ---------------------------------------------------------------------------
// Repeat-interleave of rows: out row r * repeat + k = in row r, in 16-byte words when
// the row length and both pointers allow it, else in 2-byte words.
// ---------------------------------------------------------------------------
template <class W>
__global__ void repeat_rows_kernel(const W* in, W* out, long long rows, long long row_words, int repeat) {
  const long long total = rows * repeat * row_words;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long orow = i / row_words, w = i - orow * row_words;
    out[i] = in[(orow / repeat) * row_words + w];
  }
}

// ---------------------------------------------------------------------------
// Row softmax (float32, bf16 out): n = the runtime vector size clamped to [0, cols];
// entries [0, n) get exp(x - max) * (1 / sum), entries [n, cols) are masked (zero).
// One CTA per row.
// ---------------------------------------------------------------------------
constexpr int SMX_T = 256;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  for (int o = 16; o; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();  // red is reused by consecutive reductions
  if (lane == 0) red[wid] = v;
  __syncthreads();
  v = red[0];
  for (int i = 1; i < SMX_T / 32; ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
  return v;
}

__global__ void __launch_bounds__(SMX_T) softmax_rows_kernel(const uint16_t* x, uint16_t* y, int cols, int vsize,
                                                             const int32_t* vsize_dev) {
  __shared__ float red[SMX_T / 32];
  int n = vsize_dev ? *vsize_dev : vsize;
  n = n < 0 ? 0 : (n > cols ? cols : n);
  const size_t o = (size_t)blockIdx.x * cols;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += SMX_T) m = fmaxf(m, bf2f(x[o + j]));
  m = block_reduce(m, red, true);
  float s = 0.f;
  for (int j = threadIdx.x; j < n; j += SMX_T) s += expf(bf2f(x[o + j]) - m);
  s = block_reduce(s, red, false);
  const float inv = 1.0f / s;
  for (int j = threadIdx.x; j < cols; j += SMX_T)
    y[o + j] = j < n ? f2bf(expf(bf2f(x[o + j]) - m) * inv) : (uint16_t)0;
}

// ---------------------------------------------------------------------------
// Batched transpose of bf16 (M, N) matrices through 32 x 33 shared-memory tiles.
// ---------------------------------------------------------------------------
__global__ void transpose_kernel(const uint16_t* in, uint16_t* out, int M, int N) {
  __shared__ uint16_t t[32][33];
  const size_t mat = (size_t)blockIdx.z * M * N;
  const int n0 = blockIdx.x * 32, m0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int m = m0 + i, n = n0 + threadIdx.x;
    if (m < M && n < N) t[i][threadIdx.x] = in[mat + (size_t)m * N + n];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int n = n0 + i, m = m0 + threadIdx.x;
    if (m < M && n < N) out[mat + (size_t)n * M + m] = t[threadIdx.x][i];
  }
}

static int grid_for(long long work, int threads) {
  const long long b = (work + threads - 1) / threads;
  const long long cap = (long long)iron_num_sms() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// The reference's per-channel split of a pattern padded to 4 dimensions.
static bool make_tap(int ndim, const int64_t* sizes, const int64_t* strides, int64_t offset, int channels,
                     Tap& t, long long& count) {
  long long sz[4], st[4];
  for (int d = 0; d < 4; ++d) {
    const int k = d - (4 - ndim);
    sz[d] = k >= 0 ? sizes[k] : 1;
    st[d] = k >= 0 ? strides[k] : 0;
    if (sz[d] < 0) return false;
  }
  int hi = -1;
  for (int d = 0; d < 4; ++d)
    if (sz[d] >= 1) hi = d;
  count = 0;
  for (int d = 0; d < 4; ++d) {
    t.size[d] = sz[d];
    t.stride[d] = st[d];
  }
  t.offset = offset;
  t.chan_step = 0;
  if (hi < 0) return true;
  const long long per = sz[hi] / channels;
  t.size[hi] = per;
  t.chan_step = per * st[hi];
  count = 1;
  for (int d = 0; d < 4; ++d) count *= t.size[d];
  return true;
}

}  // namespace iron

using namespace iron;

extern "C" int iron_rope_rows(const uint16_t* x, const uint16_t* angles, uint16_t* y, int rows, int cols,
                              int angle_rows, int method, void* stream) {
  IRON_REQUIRE(x && angles && y, IRON_ERR_ARG, "rope_rows: null pointer");
  IRON_REQUIRE(rows >= 1 && cols >= 2 && cols % 2 == 0, IRON_ERR_ARG, "rope_rows: %d x %d (cols must be even)", rows,
               cols);
  IRON_REQUIRE(angle_rows >= 1 && angle_rows <= rows && rows % angle_rows == 0, IRON_ERR_ARG,
               "rope_rows: angle_rows %d must divide rows %d", angle_rows, rows);
  IRON_REQUIRE(method == 0 || method == 1, IRON_ERR_ARG, "rope_rows: method %d (0 two halves, 1 interleaved)",
               method);
  const long long n = (long long)rows * (cols / 2);
  rope_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, angles, y, rows, cols,
                                                                                   rows / angle_rows, method);
  return iron_check_launch("rope_rows_kernel");
}

extern "C" int iron_strided_copy(const void* in, int64_t in_elems, void* out, int64_t out_elems, int elem_bytes,
                                 int in_ndim, const int64_t* in_sizes, const int64_t* in_strides, int64_t in_offset,
                                 int out_ndim, const int64_t* out_sizes, const int64_t* out_strides,
                                 int64_t out_offset, int channels, const int32_t* in_addend_dev,
                                 const int32_t* out_addend_dev, int32_t* err_dev, void* stream) {
  IRON_REQUIRE(in && out && in_sizes && in_strides && out_sizes && out_strides, IRON_ERR_ARG,
               "strided_copy: null pointer");
  IRON_REQUIRE(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8, IRON_ERR_ARG,
               "strided_copy: element size %d (1, 2, 4 or 8)", elem_bytes);
  IRON_REQUIRE(in_ndim >= 1 && in_ndim <= 4 && out_ndim >= 1 && out_ndim <= 4 && channels >= 1, IRON_ERR_ARG,
               "strided_copy: %d / %d dimensions (1-4), %d channels", in_ndim, out_ndim, channels);
  IRON_REQUIRE(in_elems >= 0 && out_elems >= 0, IRON_ERR_ARG, "strided_copy: negative buffer size");
  CopyArgs a;
  long long ci = 0, co = 0;
  IRON_REQUIRE(make_tap(in_ndim, in_sizes, in_strides, in_offset, channels, a.in, ci) &&
                   make_tap(out_ndim, out_sizes, out_strides, out_offset, channels, a.out, co),
               IRON_ERR_ARG, "strided_copy: negative size");
  IRON_REQUIRE(ci == co, IRON_ERR_ARG,
               "strided_copy: tap element counts differ (%lld vs %lld per channel); the input and output "
               "access patterns must move the same number of elements", ci, co);
  a.per_channel = ci;
  a.total = ci * channels;
  a.in_elems = in_elems;
  a.out_elems = out_elems;
  a.elem_bytes = elem_bytes;
  a.in_add = in_addend_dev;
  a.out_add = out_addend_dev;
  a.err = err_dev;
  if (a.total == 0) return IRON_OK;
  strided_copy_kernel<<<grid_for(a.total, 256), 256, 0, (cudaStream_t)stream>>>((const uint8_t*)in, (uint8_t*)out,
                                                                                 a);
  return iron_check_launch("strided_copy_kernel");
}

extern "C" int iron_repeat_rows(const void* in, void* out, int64_t rows, int64_t row_bytes, int repeat,
                                void* stream) {
  IRON_REQUIRE(in && out && rows >= 0 && row_bytes >= 0 && repeat >= 1, IRON_ERR_ARG, "repeat_rows: bad arguments");
  IRON_REQUIRE(row_bytes % 2 == 0, IRON_ERR_ARG, "repeat_rows: row of %lld bytes (2-byte elements)",
               (long long)row_bytes);
  if (rows == 0 || row_bytes == 0) return IRON_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (row_bytes % 16 == 0 && iron_aligned(in, 16) && iron_aligned(out, 16)) {
    const long long w = row_bytes / 16;
    repeat_rows_kernel<uint4><<<grid_for(rows * repeat * w, 256), 256, 0, st>>>((const uint4*)in, (uint4*)out, rows,
                                                                                 w, repeat);
  } else {
    const long long w = row_bytes / 2;
    repeat_rows_kernel<uint16_t><<<grid_for(rows * repeat * w, 256), 256, 0, st>>>((const uint16_t*)in,
                                                                                   (uint16_t*)out, rows, w, repeat);
  }
  return iron_check_launch("repeat_rows_kernel");
}

extern "C" int iron_softmax_rows(const uint16_t* x, uint16_t* y, int rows, int cols, int vector_size,
                                 const int32_t* vector_size_dev, void* stream) {
  IRON_REQUIRE(x && y && rows >= 1 && cols >= 1, IRON_ERR_ARG, "softmax_rows: bad arguments");
  softmax_rows_kernel<<<rows, SMX_T, 0, (cudaStream_t)stream>>>(x, y, cols, vector_size, vector_size_dev);
  return iron_check_launch("softmax_rows_kernel");
}

extern "C" int iron_transpose(const uint16_t* in, uint16_t* out, int M, int N, int batches, void* stream) {
  IRON_REQUIRE(in && out && M >= 1 && N >= 1 && batches >= 1 && batches <= 65535, IRON_ERR_ARG,
               "transpose: bad arguments");
  IRON_REQUIRE(in != out, IRON_ERR_ARG, "transpose: in place is not supported");
  const dim3 grid((N + 31) / 32, (M + 31) / 32, batches);
  transpose_kernel<<<grid, dim3(32, 8), 0, (cudaStream_t)stream>>>(in, out, M, N);
  return iron_check_launch("transpose_kernel");
}
