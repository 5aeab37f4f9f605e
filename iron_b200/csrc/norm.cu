// RMSNorm, elementwise ops, embedding gather and the per-head q/k-norm + RoPE +
// KV-cache epilogue of the fused QKV head.
#include "common.cuh"

namespace iron {

// one CTA per row; float32 math, one bf16 rounding (aie_kernels/aie2p/rms_norm.cc:9-53)
__global__ void rmsnorm_kernel(const uint16_t* x, const uint16_t* w, uint16_t* y, int cols, float eps,
                               int mode) {
  __shared__ double red[32];
  const uint16_t* xr = x + (size_t)blockIdx.x * cols;
  uint16_t* yr = y + (size_t)blockIdx.x * cols;
  double ss = 0.0;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) ss += rms_sq(bf2f(xr[i]), mode);
  ss = block_sum_d(ss, red);
  const RmsCoef rc = rms_coef(ss, cols, eps, mode);
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    yr[i] = f2bf(rms_apply(bf2f(xr[i]), w ? bf2f(w[i]) : 1.0f, rc));
  }
}

__global__ void eltwise_kernel(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, int op) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = bf2f(a[i]);
    float r;
    if (op == 0) {
      r = x + bf2f(b[i]);
    } else if (op == 1) {
      r = x * bf2f(b[i]);
    } else if (op == 2) {
      r = x / (1.0f + expf(-x));
    } else {
      r = silu_tanh_bf16(x);
    }
    c[i] = f2bf(r);
  }
}

// ids outside [0, vocab) produce a zero row instead of an out-of-range read
__global__ void embedding_kernel(const uint16_t* table, const int32_t* ids, int vocab, int D, uint16_t* out) {
  const int i = blockIdx.x;
  const int id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  const uint16_t* src = table + (size_t)(ok ? id : 0) * D;
  for (int k = threadIdx.x; k < D; k += blockDim.x) out[(size_t)i * D + k] = ok ? src[k] : (uint16_t)0;
}

// Per-head epilogue of the fused QKV head (qkv_head_dp/reference.py:29-33).
// grid (Hq + Hkv, batch), one warp per head.  q heads: RMSNorm_w(n_qn) -> RoPE ->
// q_out.  kv heads: RMSNorm_w(n_kn) -> RoPE -> K_t, and V_t = raw v, both written
// to the cache at the stream's position.  pos0 >= 0: the rows are consecutive tokens
// of ONE stream (a prompt), row b at position pos0 + b of that stream's cache.
template <int HD>
__global__ void qk_norm_rope_kv_kernel(const uint16_t* raw, const uint16_t* n_qn, const uint16_t* n_kn,
                                       const uint16_t* ang, int ang_is_table, uint16_t* q_out,
                                       uint16_t* kv, int Hq, int Hkv, int max_seq, int kv_off,
                                       const int32_t* kv_off_dev, float eps, int norm_mode, int pos0, int batch) {
  constexpr int PER = HD / 32;
  // one warp per (head, row): warp threadIdx.y of the block takes row blockIdx.y * blockDim.y + threadIdx.y
  const int head = blockIdx.x, b = blockIdx.y * blockDim.y + threadIdx.y, lane = threadIdx.x;
  if (b >= batch) return;
  const int QKV = (Hq + 2 * Hkv) * HD;
  // element offset of K_t in a head region
  const int off = pos0 >= 0 ? (pos0 + b) * 2 * HD : (kv_off_dev ? kv_off_dev[b] : kv_off);
  const int stream = pos0 >= 0 ? 0 : b;
  // an offset outside the cache (e.g. a stale runtime parameter) writes nothing
  if (off < 0 || off % (2 * HD) != 0 || off / (2 * HD) >= max_seq) return;
  const bool isq = head < Hq;
  const uint16_t* src = raw + (size_t)b * QKV + (size_t)head * HD;
  const uint16_t* nw = isq ? n_qn : n_kn;
  const uint16_t* a = ang + (size_t)(ang_is_table ? off / (2 * HD) : b) * HD;
  // lane owns element pairs (i, i + HD/2) for i = lane + 32*j, j < PER/2
  float v[PER];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < PER / 2; ++j) {
    const int i = lane + 32 * j;
    v[2 * j] = bf2f(src[i]);
    v[2 * j + 1] = bf2f(src[i + HD / 2]);
    ss += rms_sq(v[2 * j], norm_mode);
    ss += rms_sq(v[2 * j + 1], norm_mode);
  }
  ss = warp_sum_d(ss);
  const RmsCoef rc = rms_coef(ss, HD, eps, norm_mode);
  uint16_t o[PER];
#pragma unroll
  for (int j = 0; j < PER / 2; ++j) {
    const int i = lane + 32 * j;
    // no norm weights: RoPE alone (Llama: llama_cpu.py:14-38)
    const float x1 = nw ? rbf(rms_apply(v[2 * j], bf2f(nw[i]), rc)) : v[2 * j];
    const float x2 = nw ? rbf(rms_apply(v[2 * j + 1], bf2f(nw[i + HD / 2]), rc)) : v[2 * j + 1];
    const float c = bf2f(a[2 * i]), s = bf2f(a[2 * i + 1]);
    // rope/reference.py:150-154: y1 = x1*c - x2*s, y2 = x2*c + x1*s (float32)
    o[2 * j] = f2bf(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    o[2 * j + 1] = f2bf(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
  }
  if (isq) {
    uint16_t* dst = q_out + ((size_t)b * Hq + head) * HD;
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      dst[lane + 32 * j] = o[2 * j];
      dst[lane + 32 * j + HD / 2] = o[2 * j + 1];
    }
  } else {
    const int kh = head - Hq;
    uint16_t* dst = kv + ((size_t)stream * Hkv + kh) * max_seq * 2 * HD + off;
    const uint16_t* vsrc = raw + (size_t)b * QKV + (size_t)(Hq + Hkv + kh) * HD;
#pragma unroll
    for (int j = 0; j < PER / 2; ++j) {
      dst[lane + 32 * j] = o[2 * j];
      dst[lane + 32 * j + HD / 2] = o[2 * j + 1];
    }
    for (int i = lane; i < HD; i += 32) dst[HD + i] = vsrc[i];
  }
}

int qk_norm_rope_kv_launch(const uint16_t* raw, const uint16_t* n_qn, const uint16_t* n_kn,
                           const uint16_t* ang, int ang_is_table, uint16_t* q_out, uint16_t* kv,
                           int HD, int Hq, int Hkv, int max_seq, int batch, int kv_off,
                           const int32_t* kv_off_dev, float eps, int norm_mode, cudaStream_t st, int pos0) {
  // a warp per (head, row), up to 8 rows per block
  const int rpb = batch >= 64 ? 8 : 1;
  const dim3 g(Hq + Hkv, (batch + rpb - 1) / rpb), blk(32, rpb);
  if (HD == 128) {
    qk_norm_rope_kv_kernel<128><<<g, blk, 0, st>>>(raw, n_qn, n_kn, ang, ang_is_table, q_out, kv, Hq, Hkv,
                                                    max_seq, kv_off, kv_off_dev, eps, norm_mode, pos0, batch);
  } else if (HD == 64) {
    qk_norm_rope_kv_kernel<64><<<g, blk, 0, st>>>(raw, n_qn, n_kn, ang, ang_is_table, q_out, kv, Hq, Hkv,
                                                   max_seq, kv_off, kv_off_dev, eps, norm_mode, pos0, batch);
  } else {
    return iron_set_error(IRON_ERR_UNSUPPORTED, "qkv head: head_dim %d (supported: 64, 128)", HD);
  }
  return iron_check_launch("qk_norm_rope_kv_kernel");
}

__global__ void decode_advance_kernel(int32_t* pos, int32_t* len, int32_t* off, int batch, int HD) {
  const int b = threadIdx.x;
  if (b < batch) {
    const int p = pos[b] + 1;
    pos[b] = p;
    len[b] = p + 1;
    off[b] = p * 2 * HD;
  }
}

static int elt_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)iron_num_sms() * 8;
  return (int)(g < cap ? (g < 1 ? 1 : g) : cap);
}

}  // namespace iron

using namespace iron;

extern "C" int iron_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int cols,
                            float eps, int mode, void* stream) {
  IRON_REQUIRE(x && y && rows > 0 && cols > 0 && mode >= 0 && mode <= 2, IRON_ERR_ARG,
               "rmsnorm: bad arguments");
  rmsnorm_kernel<<<rows, cols >= 1024 ? 512 : 128, 0, (cudaStream_t)stream>>>(x, w, y, cols, eps, mode);
  return iron_check_launch("rmsnorm_kernel");
}

static int elt(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, int op, void* stream) {
  IRON_REQUIRE(a && c && n >= 0 && (b || op >= 2), IRON_ERR_ARG, "eltwise: bad arguments");
  if (n == 0) return IRON_OK;
  eltwise_kernel<<<elt_grid(n), 256, 0, (cudaStream_t)stream>>>(a, b, c, n, op);
  return iron_check_launch("eltwise_kernel");
}

extern "C" int iron_add(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, void* stream) {
  return elt(a, b, c, n, 0, stream);
}
extern "C" int iron_mul(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n, void* stream) {
  return elt(a, b, c, n, 1, stream);
}
// RoPE of q and k heads of a raw (batch, (Hq + 2 Hkv) HD) projection and the K/V cache
// write at each stream's offset, without per-head norms.
extern "C" int iron_rope_kv(const uint16_t* raw, const uint16_t* ang_table, uint16_t* q_out, uint16_t* kv_cache,
                            int HD, int Hq, int Hkv, int max_seq, int batch, const int32_t* kv_off_dev,
                            void* stream) {
  IRON_REQUIRE(raw && ang_table && q_out && kv_cache && kv_off_dev && batch >= 1 && Hq >= 1 && Hkv >= 1,
               IRON_ERR_ARG, "rope_kv: bad arguments");
  return qk_norm_rope_kv_launch(raw, nullptr, nullptr, ang_table, 1, q_out, kv_cache, HD, Hq, Hkv, max_seq, batch,
                                0, kv_off_dev, 0.f, 0, (cudaStream_t)stream, -1);
}

// The QKV head epilogue over the consecutive tokens of one prompt: row r of raw is the
// token at position pos0 + r of the single stream whose cache is kv_cache.
extern "C" int iron_qkv_rows(const uint16_t* raw, int rows, const uint16_t* n_qn, const uint16_t* n_kn,
                             const uint16_t* ang_table, uint16_t* q_out, uint16_t* kv_cache, int HD, int Hq,
                             int Hkv, int max_seq, int pos0, float eps, int norm_mode, void* stream) {
  IRON_REQUIRE(raw && ang_table && q_out && kv_cache && rows >= 1 && Hq >= 1 && Hkv >= 1, IRON_ERR_ARG,
               "qkv_rows: bad arguments");
  IRON_REQUIRE(pos0 >= 0 && pos0 + rows <= max_seq, IRON_ERR_ARG,
               "qkv_rows: positions %d..%d outside a %d-token cache", pos0, pos0 + rows - 1, max_seq);
  IRON_REQUIRE(norm_mode >= 0 && norm_mode <= 2, IRON_ERR_ARG, "qkv_rows: norm_mode must be 0, 1 or 2");
  return qk_norm_rope_kv_launch(raw, n_qn, n_kn, ang_table, 1, q_out, kv_cache, HD, Hq, Hkv, max_seq, rows, 0,
                                nullptr, eps, norm_mode, (cudaStream_t)stream, pos0);
}

extern "C" int iron_silu(const uint16_t* x, uint16_t* y, int64_t n, int mode, void* stream) {
  IRON_REQUIRE(mode == 0 || mode == 1, IRON_ERR_ARG, "silu: mode must be 0 or 1");
  return elt(x, nullptr, y, n, 2 + mode, stream);
}
extern "C" int iron_embedding(const uint16_t* table, int vocab, const int32_t* ids, int n, int D,
                              uint16_t* out, void* stream) {
  IRON_REQUIRE(table && ids && out && n >= 0 && D > 0 && vocab > 0, IRON_ERR_ARG, "embedding: bad arguments");
  if (n == 0) return IRON_OK;
  embedding_kernel<<<n, 256, 0, (cudaStream_t)stream>>>(table, ids, vocab, D, out);
  return iron_check_launch("embedding_kernel");
}

extern "C" int iron_decode_advance(int32_t* pos, int32_t* seq_len, int32_t* kv_off, int batch, int HD,
                                   void* stream) {
  IRON_REQUIRE(pos && seq_len && kv_off && batch >= 1 && batch <= 1024, IRON_ERR_ARG,
               "decode_advance: bad arguments");
  decode_advance_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(pos, seq_len, kv_off, batch, HD);
  return iron_check_launch("decode_advance_kernel");
}
