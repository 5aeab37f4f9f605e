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
#include <cstdlib>
#include <cstring>

#include "attn_tc.cuh"
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

// ---------------------------------------------------------------------------
// The same pass 1 on the tensor pipe.  Grid, work split and partials are those of
// attn_split_kernel (one (o, m, l) per query head and split, merged by
// attn_combine_kernel).  The GQ query heads of the KV head are rows 0..GQ-1 of one
// 16-row MMA tile (the other rows are zero).  K/V tiles of 64 positions stream
// through a two-stage cp.async ring (16-byte chunks XOR-swizzled by row, so ldmatrix
// reads are conflict-free); warp w takes positions 16w..16w+15 of every tile:
// S = Q K^T on bf16 mma.sync m16n8k16 with float32 accumulation (products of bf16
// values are exact in float32), a base-2 online softmax per row, and O += P V with P
// as a bf16 high part plus a bf16 remainder (two MMAs: the probabilities enter at
// about float32 precision).  The four warps' states merge in shared memory.  About
// 12 warp instructions per cached position (against ~64 for the lane-load form at
// GQA group 4) leave the kernel bound by the bytes in flight.
// ---------------------------------------------------------------------------
constexpr int TC_KEYS = 64;  // positions per K/V tile
constexpr int TC_THREADS = 128;

template <int HD>
constexpr int tc_smem_bytes() {
  return 16 * HD * 2 + 4 * TC_KEYS * HD * 2;  // Q tile, two stages of K and of V
}

template <int HD>
__global__ void __launch_bounds__(TC_THREADS, 3) attn_split_tc_kernel(AttnParams p) {
  constexpr int CH = HD / 8;   // 16-byte chunks per row
  constexpr int KS = HD / 16;  // k-steps of Q K^T
  constexpr int ND = HD / 8;   // n-tiles of the output
  constexpr int TILE = TC_KEYS * HD * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                // [16][HD]
  uint8_t* sK = smem + 16 * HD * 2;  // [2][64][HD]
  uint8_t* sV = sK + 2 * TILE;       // [2][64][HD]

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int GQ = p.H / p.KV;
  int L = p.seq_lens ? p.seq_lens[b] : p.seq_len;
  L = L < 0 ? 0 : (L > p.max_seq ? p.max_seq : L);
  const int nblk = (L + TC_KEYS - 1) / TC_KEYS;
  const int bps = (nblk + p.nsplit - 1) / p.nsplit;
  const int b_begin = split * bps;
  const int b_end = min(nblk, b_begin + bps);

  // the GQ query rows of this KV head (zeros below them)
  for (int i = tid; i < 16 * CH; i += TC_THREADS) {
    const int r = i / CH, c = i - r * CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < GQ) v = *(const uint4*)(p.q + ((size_t)b * p.H + kvh * GQ + r) * HD + c * 8);
    *(uint4*)(sQ + swz<HD>(r, c)) = v;
  }
  const uint16_t* head = p.kv + ((size_t)b * p.KV + kvh) * 2 * (size_t)p.max_seq * HD;
  const size_t voff = p.layout == 0 ? HD : (p.layout == 1 ? (size_t)p.max_seq * HD : (size_t)p.block_kv * HD);
  auto koff = [&](int j) -> size_t {
    if (p.layout == 0) return (size_t)j * 2 * HD;
    if (p.layout == 1) return (size_t)j * HD;
    const int bk = j / p.block_kv, jj = j - bk * p.block_kv;
    return ((size_t)bk * 2 * p.block_kv + jj) * HD;
  };
  // K/V tile of block blk into stage s; rows past the last position repeat it (masked
  // below), so every copy reads inside the stream's cache
  auto load_tile = [&](int blk, int s) {
    const int jmax = L - 1;
    for (int i = tid; i < TC_KEYS * CH; i += TC_THREADS) {
      const int r = i / CH, c = i - r * CH;
      const int j = min(blk * TC_KEYS + r, jmax);
      const uint16_t* src = head + koff(j) + c * 8;
      cp_async16(smem_u32(sK + s * TILE + swz<HD>(r, c)), src);
      cp_async16(smem_u32(sV + s * TILE + swz<HD>(r, c)), src + voff);
    }
  };
  if (b_begin < b_end) load_tile(b_begin, 0);
  cp_async_commit();
  __syncthreads();

  uint32_t qf[KS][4];
  {
    const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1);
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
      ldsm_x4(smem_u32(sQ) + swz<HD>(rr, 2 * kk + (mi >> 1)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }
  // the thread's rows: lane/4 (a) and lane/4 + 8 (b, always a zero row: GQ <= 8)
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  for (int blk = b_begin; blk < b_end; ++blk) {
    const int s = (blk - b_begin) & 1;
    if (blk + 1 < b_end) load_tile(blk + 1, s ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t kbase = smem_u32(sK + s * TILE), vbase = smem_u32(sV + s * TILE);
    // S = Q K^T for this warp's 16 positions (two n-tiles of 8)
    float sc[2][4];
    sc[0][0] = sc[0][1] = sc[0][2] = sc[0][3] = 0.f;
    sc[1][0] = sc[1][1] = sc[1][2] = sc[1][3] = 0.f;
    {
      const int mi = lane >> 3, kr = (lane & 7) + 8 * (mi >> 1), kc = mi & 1;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + swz<HD>(16 * warp + kr, 2 * kk + kc), b0, b1, b2, b3);
        mma_bf16(sc[0], qf[kk], b0, b1);
        mma_bf16(sc[1], qf[kk], b2, b3);
      }
    }
    const int j0 = blk * TC_KEYS + 16 * warp + 2 * (lane & 3);
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int j = j0 + 8 * n;
      sc[n][0] = j < L ? sc[n][0] * p.scale : -INFINITY;
      sc[n][1] = j + 1 < L ? sc[n][1] * p.scale : -INFINITY;
      sc[n][2] = j < L ? sc[n][2] * p.scale : -INFINITY;
      sc[n][3] = j + 1 < L ? sc[n][3] * p.scale : -INFINITY;
      mx_a = fmaxf(mx_a, fmaxf(sc[n][0], sc[n][1]));
      mx_b = fmaxf(mx_b, fmaxf(sc[n][2], sc[n][3]));
    }
#pragma unroll
    for (int x = 1; x < 4; x <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(~0u, mx_a, x));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(~0u, mx_b, x));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    // a row that has seen only masked positions keeps everything at zero
    const float u_a = mn_a == -INFINITY ? 0.f : mn_a, u_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float c_a = exp2f(m_a - u_a), c_b = exp2f(m_b - u_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a *= c_a;
    l_b *= c_b;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      o[n][0] *= c_a;
      o[n][1] *= c_a;
      o[n][2] *= c_b;
      o[n][3] *= c_b;
    }
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      sc[n][0] = exp2f(sc[n][0] - u_a);
      sc[n][1] = exp2f(sc[n][1] - u_a);
      sc[n][2] = exp2f(sc[n][2] - u_b);
      sc[n][3] = exp2f(sc[n][3] - u_b);
      l_a += sc[n][0] + sc[n][1];
      l_b += sc[n][2] + sc[n][3];
    }
    // O += P V over the warp's 16 positions (one k-step)
    {
      uint32_t ph[4], pl[4];
      split_pair(sc[0][0], sc[0][1], ph[0], pl[0]);
      split_pair(sc[0][2], sc[0][3], ph[1], pl[1]);
      split_pair(sc[1][0], sc[1][1], ph[2], pl[2]);
      split_pair(sc[1][2], sc[1][3], ph[3], pl[3]);
      const int mi = lane >> 3, vr = (lane & 7) + 8 * (mi & 1), vc = mi >> 1;
#pragma unroll
      for (int n = 0; n < ND; n += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + swz<HD>(16 * warp + vr, n + vc), b0, b1, b2, b3);
        mma_bf16(o[n], ph, b0, b1);
        mma_bf16(o[n], pl, b0, b1);
        mma_bf16(o[n + 1], ph, b2, b3);
        mma_bf16(o[n + 1], pl, b2, b3);
      }
    }
    __syncthreads();  // stage s is refilled two blocks on
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused below

  // row sums over the quad; the warps' states of the real rows into shared memory
#pragma unroll
  for (int x = 1; x < 4; x <<= 1) l_a += __shfl_xor_sync(~0u, l_a, x);
  float* red_o = (float*)sK;   // [4][GQ][HD]
  float* red_ml = (float*)sV;  // [4][GQ][2]
  const int ra = lane >> 2, cb = 2 * (lane & 3);
  if (ra < GQ) {
    float* ro = red_o + ((size_t)warp * GQ + ra) * HD;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      ro[8 * n + cb] = o[n][0];
      ro[8 * n + cb + 1] = o[n][1];
    }
    if ((lane & 3) == 0) {
      red_ml[(warp * GQ + ra) * 2] = m_a;
      red_ml[(warp * GQ + ra) * 2 + 1] = l_a;
    }
  }
  __syncthreads();
  for (int t = tid; t < GQ * HD; t += TC_THREADS) {
    const int r = t / HD, d = t - r * HD;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_ml[(w * GQ + r) * 2]);
    float oo = 0.f, ll = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(red_ml[(w * GQ + r) * 2] - M);
        oo = fmaf(red_o[((size_t)w * GQ + r) * HD + d], f, oo);
        ll = fmaf(red_ml[(w * GQ + r) * 2 + 1], f, ll);
      }
    }
    float* dst = p.ws + (((size_t)b * p.H + kvh * GQ + r) * p.nsplit + split) * (HD + 2);
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

// The tensor-pipe pass 1 is the default; IRON_DECODE_ATTN=lanes selects the
// lane-load kernel (for comparisons).  Read once per process.
static bool attn_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("IRON_DECODE_ATTN");
    return !(e && std::strcmp(e, "lanes") == 0);
  }();
  return on;
}

// Split count as launch_split, for the resident CTAs of the tensor-pipe kernel.
template <int HD>
static int launch_split_tc(AttnParams p, int batch, int cap, cudaStream_t st) {
  static bool attr[64] = {false};
  static int occ[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = dev >= 0 && dev < 64 ? occ[dev] : 0;
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(attn_split_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem_bytes<HD>());
    attr[dev] = true;
  }
  if (per_sm < 1) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_split_tc_kernel<HD>, TC_THREADS, tc_smem_bytes<HD>());
    if (per_sm < 1) per_sm = 1;
    if (dev >= 0 && dev < 64) occ[dev] = per_sm;
  }
  const int wave = per_sm * iron_num_sms(), pairs = batch * p.KV;
  const int target = 4 * pairs >= wave ? 3 * wave : wave;
  int ns = target / pairs;
  ns = ns < 1 ? 1 : (ns > cap ? cap : ns);
  p.nsplit = ns;
  attn_split_tc_kernel<HD><<<dim3(ns, p.KV, batch), TC_THREADS, tc_smem_bytes<HD>(), st>>>(p);
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
  // the tensor-pipe kernel stages the query rows with 16-byte loads
  if (attn_tc_enabled() && (HD == 128 || HD == 64) && (GQ == 1 || GQ == 2 || GQ == 4 || GQ == 8) &&
      iron_aligned(q, 16)) {
    ns = HD == 128 ? launch_split_tc<128>(p, batch, cap, st) : launch_split_tc<64>(p, batch, cap, st);
    goto combine;
  }
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
