// Decode attention: split-KV flash decoding over a GQA KV cache.
//
// Pass 1: grid (split, kv_head, stream).  Each CTA owns one KV head of one
// stream and a contiguous slice of its positions; its 4 warps take blocks of
// positions round-robin.  HD/8 lanes share a K or V row, 16 bytes (8 dims) each,
// so one warp-wide load covers 32*8/HD positions and a warp keeps U such loads of
// K and of V in flight.  A lane holds its 8 dims of every query head of the GQA
// group; q.k is a butterfly over the row's lanes, and each row group keeps a
// base-2 online softmax state (m, l, o) per head -- the streaming form of
// decode_attn.cc:208-279.  Row groups merge by shuffles, warps in shared memory,
// and the CTA writes one partial per head.
// Pass 2: grid (head, stream) merges the splits: M = max m_s,
// o = sum o_s 2^(m_s-M) / sum l_s 2^(m_s-M)  (decode_attn/reference.py:26-38).
#include "common.cuh"

namespace iron {

struct AttnParams {
  const uint16_t* q;     // [batch][H][HD]
  const uint16_t* kv;    // per stream, per kv head: 2*max_seq*HD
  float* ws;             // [batch][H][nsplit][HD + 2]
  int H, KV, max_seq, layout, block_kv, seq_len, nsplit;
  const int32_t* seq_lens;
  float scale;           // log2(e)/sqrt(HD)
};

template <int HD, int GQ>
__global__ void __launch_bounds__(128) attn_split_kernel(AttnParams p) {
  constexpr int RL = HD / 8;          // lanes per K / V row, 16 bytes each
  constexpr int RPW = 32 / RL;        // rows per warp-wide load
  constexpr int U = GQ >= 8 ? 2 : 4;  // loads per iteration
  constexpr int PW = U * RPW;         // positions per warp iteration
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane % RL, rg = lane / RL;  // dims [8 sub, 8 sub + 8) of row group rg
  int L = p.seq_lens ? p.seq_lens[b] : p.seq_len;
  L = L < 0 ? 0 : (L > p.max_seq ? p.max_seq : L);
  const int chunk = (L + p.nsplit - 1) / p.nsplit;
  const int start = split * chunk;
  const int end = min(L, start + chunk);

  // the group's queries in shared memory (float32), not registers: the freed
  // registers let more CTAs (more K/V bytes in flight) share an SM
  __shared__ __align__(16) float sq[GQ][HD];
  for (int i = threadIdx.x; i < GQ * HD; i += blockDim.x)
    sq[i / HD][i % HD] = bf2f(p.q[((size_t)b * p.H + kvh * GQ) * HD + i]);
  __syncthreads();
  const uint16_t* head = p.kv + ((size_t)b * p.KV + kvh) * 2 * (size_t)p.max_seq * HD;
  // element offsets of K_j / V_j inside the head region for the three layouts
  auto koff = [&](int j) -> size_t {
    if (p.layout == 0) return (size_t)j * 2 * HD;
    if (p.layout == 1) return (size_t)j * HD;
    const int bk = j / p.block_kv, jj = j - bk * p.block_kv;
    return ((size_t)bk * 2 * p.block_kv + jj) * HD;
  };
  const size_t voff = p.layout == 0 ? HD : (p.layout == 1 ? (size_t)p.max_seq * HD : (size_t)p.block_kv * HD);

  // online softmax state of this lane's row group
  float m[GQ], l[GQ], o[GQ][8];
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] = 0.f;
  }

  for (int j0 = start + wid * PW; j0 < end; j0 += 4 * PW) {
    uint4 kr[U], vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = min(j0 + u * RPW + rg, end - 1);
      const uint16_t* kp = head + koff(j) + sub * 8;
      kr[u] = ldg_stream(kp);
      vr[u] = ldg_stream(kp + voff);
    }
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      float s[U];
      float mn = m[h];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t kw[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
        const float4 qa = *(const float4*)&sq[h][sub * 8], qb = *(const float4*)&sq[h][sub * 8 + 4];
        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          d = fmaf(qv[2 * e], bf_lo(kw[e]), d);
          d = fmaf(qv[2 * e + 1], bf_hi(kw[e]), d);
        }
#pragma unroll
        for (int x = 1; x < RL; x <<= 1) d += __shfl_xor_sync(~0u, d, x);
        s[u] = j0 + u * RPW + rg < end ? d * p.scale : -INFINITY;
        mn = fmaxf(mn, s[u]);
      }
      if (mn == -INFINITY) continue;  // this row group has seen only masked positions
      const float corr = exp2f(m[h] - mn);
      float ls = l[h] * corr;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[h][e] *= corr;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pu = exp2f(s[u] - mn);
        const uint32_t vw[4] = {vr[u].x, vr[u].y, vr[u].z, vr[u].w};
        ls += pu;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[h][2 * e] = fmaf(pu, bf_lo(vw[e]), o[h][2 * e]);
          o[h][2 * e + 1] = fmaf(pu, bf_hi(vw[e]), o[h][2 * e + 1]);
        }
      }
      l[h] = ls;
      m[h] = mn;
    }
  }
  // merge the row groups of the warp (lanes RL apart hold the same dims)
#pragma unroll
  for (int x = RL; x < 32; x <<= 1) {
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
      const float m2 = __shfl_xor_sync(~0u, m[h], x), l2 = __shfl_xor_sync(~0u, l[h], x);
      const float M = fmaxf(m[h], m2);
      const float f1 = M == -INFINITY ? 0.f : exp2f(m[h] - M), f2 = M == -INFINITY ? 0.f : exp2f(m2 - M);
      l[h] = l[h] * f1 + l2 * f2;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[h][e] = o[h][e] * f1 + __shfl_xor_sync(~0u, o[h][e], x) * f2;
      m[h] = M;
    }
  }

  // merge the 4 warps
  __shared__ float sm_m[4][GQ], sm_l[4][GQ];
  __shared__ float sm_o[4][GQ][HD];
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    if (lane == 0) {
      sm_m[wid][h] = m[h];
      sm_l[wid][h] = l[h];
    }
    if (rg == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_o[wid][h][sub * 8 + e] = o[h][e];
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < GQ * HD; t += blockDim.x) {
    const int h = t / HD, d = t - h * HD;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w][h]);
    float oo = 0.f, ll = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_m[w][h] - M);
        oo = fmaf(sm_o[w][h][d], f, oo);
        ll = fmaf(sm_l[w][h], f, ll);
      }
    }
    float* dst = p.ws + (((size_t)b * p.H + kvh * GQ + h) * p.nsplit + split) * (HD + 2);
    dst[d] = oo;
    if (d == 0) {
      dst[HD] = M;
      dst[HD + 1] = ll;
    }
  }
}

template <int HD>
__global__ void attn_combine_kernel(const float* ws, int H, int nsplit, uint16_t* out) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* src = ws + ((size_t)b * H + h) * nsplit * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, src[s * (HD + 2) + HD]);
  float oo = 0.f, ll = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < nsplit; ++s) {
      const float* ps = src + s * (HD + 2);
      const float f = exp2f(ps[HD] - M);
      oo = fmaf(ps[d], f, oo);
      ll = fmaf(ps[HD + 1], f, ll);
    }
  }
  out[((size_t)b * H + h) * HD + d] = f2bf(ll > 0.f ? oo / ll : 0.f);
}

static int nsplit_cap(int max_seq) {
  int n = (max_seq + 63) / 64;
  return n < 1 ? 1 : (n > 256 ? 256 : n);
}

// Resident split CTAs per SM (registers bound them), cached per device.
template <int HD, int GQ>
static int split_ctas_per_sm() {
  static int occ[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && occ[dev]) return occ[dev];
  int n = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_split_kernel<HD, GQ>, 128, 0);
  if (n < 1) n = 1;
  if (dev < 64) occ[dev] = n;
  return n;
}

// Split count: with few (stream, KV head) pairs, one resident wave of CTAs (the
// longest chunk per CTA that still fills the GPU); once the pairs alone come near a
// wave, three waves, so that the SMs stay full while the last CTAs finish.
// Returns the split count.
template <int HD, int GQ>
static int launch_split(AttnParams p, int batch, int cap, cudaStream_t st) {
  const int wave = split_ctas_per_sm<HD, GQ>() * iron_num_sms(), pairs = batch * p.KV;
  const int target = 4 * pairs >= wave ? 3 * wave : wave;
  int ns = target / pairs;  // rounded down: a few CTAs past the last wave would run alone
  ns = ns < 1 ? 1 : (ns > cap ? cap : ns);
  p.nsplit = ns;
  dim3 g(ns, p.KV, batch);
  attn_split_kernel<HD, GQ><<<g, 128, 0, st>>>(p);
  return ns;
}

}  // namespace iron

using namespace iron;

extern "C" int64_t iron_decode_attn_workspace_bytes(int batch, int H, int HD, int max_seq) {
  return (int64_t)batch * H * nsplit_cap(max_seq) * (HD + 2) * 4;
}

extern "C" int iron_decode_attn(const uint16_t* q, const uint16_t* kv, uint16_t* out, int batch, int H,
                                int KV, int HD, int max_seq, int kv_layout, int block_kv, int seq_len,
                                const int32_t* seq_lens_dev, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  IRON_REQUIRE(q && kv && out && workspace, IRON_ERR_ARG, "decode_attn: null pointer");
  IRON_REQUIRE(batch >= 1 && KV >= 1 && H % KV == 0 && max_seq >= 1, IRON_ERR_ARG,
               "decode_attn: bad shape batch=%d H=%d KV=%d max_seq=%d", batch, H, KV, max_seq);
  IRON_REQUIRE(kv_layout >= 0 && kv_layout <= 2, IRON_ERR_ARG, "decode_attn: kv_layout must be 0, 1 or 2");
  IRON_REQUIRE(kv_layout != 2 || (block_kv > 0 && max_seq % block_kv == 0), IRON_ERR_ARG,
               "decode_attn: block layout needs block_kv dividing max_seq");
  IRON_REQUIRE(seq_lens_dev || (seq_len >= 1 && seq_len <= max_seq), IRON_ERR_ARG,
               "decode_attn: seq_len %d not in [1, %d]", seq_len, max_seq);
  IRON_REQUIRE(workspace_bytes >= iron_decode_attn_workspace_bytes(batch, H, HD, max_seq), IRON_ERR_ARG,
               "decode_attn: workspace of %lld bytes is too small", (long long)workspace_bytes);
  IRON_REQUIRE(iron_aligned(kv, 16) && iron_aligned(q, 4), IRON_ERR_ALIGN, "decode_attn: kv must be 16-byte aligned");
  AttnParams p;
  p.q = q;
  p.kv = kv;
  p.ws = (float*)workspace;
  p.H = H;
  p.KV = KV;
  p.max_seq = max_seq;
  p.layout = kv_layout;
  p.block_kv = block_kv;
  p.seq_len = seq_len;
  p.seq_lens = seq_lens_dev;
  p.scale = 1.4426950408889634f / sqrtf((float)HD);
  const int cap = nsplit_cap(seq_lens_dev ? max_seq : seq_len);
  int ns = 0;
  const int GQ = H / KV;
  cudaStream_t st = (cudaStream_t)stream;
#define IRON_ATTN_CASE(hd, gq) \
  if (HD == hd && GQ == gq) { ns = launch_split<hd, gq>(p, batch, cap, st); goto combine; }
  IRON_ATTN_CASE(128, 1) IRON_ATTN_CASE(128, 2) IRON_ATTN_CASE(128, 4) IRON_ATTN_CASE(128, 8)
  IRON_ATTN_CASE(64, 1) IRON_ATTN_CASE(64, 2) IRON_ATTN_CASE(64, 4) IRON_ATTN_CASE(64, 8)
#undef IRON_ATTN_CASE
  return iron_set_error(IRON_ERR_UNSUPPORTED, "decode_attn: head_dim %d / GQA group %d unsupported", HD, GQ);
combine : {
  int rc = iron_check_launch("attn_split_kernel");
  if (rc) return rc;
  dim3 g(H, batch);
  if (HD == 128)
    attn_combine_kernel<128><<<g, 128, 0, st>>>(p.ws, H, ns, out);
  else
    attn_combine_kernel<64><<<g, 64, 0, st>>>(p.ws, H, ns, out);
  return iron_check_launch("attn_combine_kernel");
}
}

// ---------------------------------------------------------------------------
// Decode attention without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they call in:
// a plugin host that owns no allocator and may not call cudaMalloc, an
// embedding runtime that forbids allocation on its decode path, or code
// running under a memory pool that rejects ad-hoc requests.  For them the
// split-KV partials live in one fixed-size array that every GPU loading this
// library reserves until the process exits.  Each call writes every partial
// slot it later reads, so nothing has to start at zero and the array keeps
// whatever the last call left.  All calls on a device share the one array:
// two calls that run at the same time on the GPU (different streams, or
// different host threads) overwrite each other's partials.
// ---------------------------------------------------------------------------
#include <mutex>

#define IRON_ATTN_STATIC_SCRATCH_BYTES (8ll << 20)  // 8 MiB per device

static __device__ __align__(256) float g_attn_static_scratch[IRON_ATTN_STATIC_SCRATCH_BYTES / 4];

// Device address of the array for the current device.  The host-side name of
// a __device__ array is not a device address, so it is looked up once per
// device with that device current, then cached.
static int attn_static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return iron_set_error(IRON_ERR_CUDA, "decode_attn_static: cudaGetDevice: %s",
                                              cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return iron_set_error(IRON_ERR_UNSUPPORTED, "decode_attn_static: device %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return iron_set_error(IRON_ERR_CUDA, "decode_attn_static: cudaGetSymbolAddress: %s",
                            cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return IRON_OK;
}

extern "C" int64_t iron_decode_attn_static_capacity_bytes(void) { return IRON_ATTN_STATIC_SCRATCH_BYTES; }

extern "C" int iron_decode_attn_static(const uint16_t* q, const uint16_t* kv, uint16_t* out, int batch, int H,
                                       int KV, int HD, int max_seq, int kv_layout, int block_kv, int seq_len,
                                       const int32_t* seq_lens_dev, void* stream) {
  IRON_REQUIRE(batch >= 1 && H >= 1 && HD >= 1 && max_seq >= 1, IRON_ERR_ARG,
               "decode_attn_static: bad shape batch=%d H=%d HD=%d max_seq=%d", batch, H, HD, max_seq);
  const int64_t need = iron_decode_attn_workspace_bytes(batch, H, HD, max_seq);
  IRON_REQUIRE(need <= IRON_ATTN_STATIC_SCRATCH_BYTES, IRON_ERR_UNSUPPORTED,
               "decode_attn_static: batch=%d H=%d HD=%d max_seq=%d needs %lld bytes of scratch, more than "
               "the built-in %lld bytes; use iron_decode_attn with a caller workspace",
               batch, H, HD, max_seq, (long long)need, (long long)IRON_ATTN_STATIC_SCRATCH_BYTES);
  void* ws = nullptr;
  int rc = attn_static_scratch(&ws);
  if (rc) return rc;
  return iron_decode_attn(q, kv, out, batch, H, KV, HD, max_seq, kv_layout, block_kv, seq_len, seq_lens_dev,
                          ws, IRON_ATTN_STATIC_SCRATCH_BYTES, stream);
}
