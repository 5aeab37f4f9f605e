// Multi-query attention over one KV stream: DecodeAttention's verify mode
// (batch_queries / num_new_tokens / causal, iron/operators/decode_attn/op.py:40-56,
// golden cpu_reference_batch in decode_attn/test_batch.py:31-46) and the causal
// self-attention of a prompt (iron/operators/mha/op.py:21-153, golden
// mha/reference.py:26-93).
//
// T new tokens sit at positions base .. base+T-1 of the cache; token t attends the
// positions j < kv_len with, when causal, j <= base + t.  GQA: the GQ query heads of
// a KV head read the same K/V rows, so the query rows of a KV head are (token, head)
// pairs r = t*GQ + g and a CTA owns 64 of them (16 per warp) and one KV head.
//
// Pass 1: grid (row block, KV head, split).  K/V tiles of 64 positions stream
// through a two-stage cp.async ring in shared memory (16-byte chunks XOR-swizzled by
// row, so ldmatrix reads are conflict-free).  S = Q K^T runs on bf16 mma.sync
// m16n8k16 with float32 accumulation (products of bf16 values are exact in float32);
// a base-2 online softmax per row keeps (m, l, o); P V runs with P split into a bf16
// high part and a bf16 remainder (two MMAs), so the probabilities enter at about
// float32 precision.  Each CTA writes one (o, m, l) partial per row.
// Pass 2 merges the splits per (token, head) exactly as the decode combine does.
#include "attn_tc.cuh"
#include "common.cuh"

namespace iron {

struct MqParams {
  const uint16_t* q;   // [T][H][HD]
  const uint16_t* kv;  // [KV][2*max_seq*HD], layout as iron_decode_attn
  float* ws;           // [T][H][nsplit][HD + 2]
  int T, H, KV, max_seq, layout, block_kv, kv_len, causal, base, nsplit;
  const int32_t* base_dev;
  float scale;  // log2(e)/sqrt(HD)
};

constexpr int MQ_ROWS = 64;   // query rows per CTA (4 warps x 16)
constexpr int MQ_KEYS = 64;   // positions per K/V tile
constexpr int MQ_THREADS = 128;
constexpr int MQ_SPLIT_CAP = 64;

template <int HD>
__global__ void __launch_bounds__(MQ_THREADS) attn_mq_kernel(MqParams p) {
  constexpr int CH = HD / 8;        // 16-byte chunks per row
  constexpr int KS = HD / 16;       // k-steps of Q K^T
  constexpr int NT = MQ_KEYS / 8;   // score n-tiles per K tile
  constexpr int ND = HD / 8;        // output n-tiles
  constexpr int TILE = MQ_KEYS * HD * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                      // [64][HD]
  uint8_t* sK = smem + MQ_ROWS * HD * 2;   // [2][64][HD]
  uint8_t* sV = sK + 2 * TILE;             // [2][64][HD]

  const int rb = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int GQ = p.H / p.KV;
  const int rows = p.T * GQ;
  const int base = p.base_dev ? p.base_dev[0] : p.base;
  const int r0 = rb * MQ_ROWS;
  // positions any row of the call may see, and those this CTA's rows may see
  const int kv_len = min(p.kv_len, p.max_seq);
  const int keys_all = p.causal ? min(kv_len, base + p.T) : kv_len;
  const int t_last = min(p.T - 1, (min(r0 + MQ_ROWS, rows) - 1) / GQ);
  const int keys_cta = p.causal ? min(kv_len, base + t_last + 1) : kv_len;
  const int nblk = keys_all > 0 ? (keys_all + MQ_KEYS - 1) / MQ_KEYS : 0;
  const int bps = (nblk + p.nsplit - 1) / p.nsplit;
  const int b_begin = split * bps;
  const int b_end = min(min(nblk, b_begin + bps), (max(keys_cta, 0) + MQ_KEYS - 1) / MQ_KEYS);

  // stage the CTA's 64 query rows (zeros past the last row)
  for (int i = tid; i < MQ_ROWS * CH; i += MQ_THREADS) {
    const int r = i / CH, c = i - r * CH, rg = r0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (rg < rows) {
      const int t = rg / GQ, h = kvh * GQ + (rg - t * GQ);
      v = *(const uint4*)(p.q + ((size_t)t * p.H + h) * HD + c * 8);
    }
    *(uint4*)(sQ + swz<HD>(r, c)) = v;
  }
  const uint16_t* head = p.kv + (size_t)kvh * 2 * (size_t)p.max_seq * HD;
  const size_t voff = p.layout == 0 ? HD : (p.layout == 1 ? (size_t)p.max_seq * HD : (size_t)p.block_kv * HD);
  auto koff = [&](int j) -> size_t {
    if (p.layout == 0) return (size_t)j * 2 * HD;
    if (p.layout == 1) return (size_t)j * HD;
    const int bk = j / p.block_kv, jj = j - bk * p.block_kv;
    return ((size_t)bk * 2 * p.block_kv + jj) * HD;
  };
  // K/V tile of block b into stage s; rows past the visible positions repeat the
  // last visible one (masked below) so every copy reads inside the cache
  auto load_tile = [&](int b, int s) {
    const int jmax = max(keys_cta, 1) - 1;
    for (int i = tid; i < MQ_KEYS * CH; i += MQ_THREADS) {
      const int r = i / CH, c = i - r * CH;
      const int j = min(b * MQ_KEYS + r, jmax);
      const uint16_t* src = head + koff(j) + c * 8;
      cp_async16(smem_u32(sK + s * TILE + swz<HD>(r, c)), src);
      cp_async16(smem_u32(sV + s * TILE + swz<HD>(r, c)), src + voff);
    }
  };
  if (b_begin < b_end) load_tile(b_begin, 0);
  cp_async_commit();
  __syncthreads();

  // this warp's Q fragments (rows 16*warp .. +15), kept in registers
  uint32_t qf[KS][4];
  {
    const int mi = lane >> 3, rr = (lane & 7) + 8 * (mi & 1);
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
      ldsm_x4(smem_u32(sQ) + swz<HD>(16 * warp + rr, 2 * kk + (mi >> 1)), qf[kk][0], qf[kk][1], qf[kk][2],
              qf[kk][3]);
  }
  // the thread's two rows: g0 = lane/4 and g0 + 8 of the warp's 16
  const int ra = r0 + 16 * warp + (lane >> 2), rb8 = ra + 8;
  const int lim_a = p.causal ? min(kv_len, base + ra / GQ + 1) : kv_len;
  const int lim_b = p.causal ? min(kv_len, base + rb8 / GQ + 1) : kv_len;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  for (int b = b_begin; b < b_end; ++b) {
    const int s = (b - b_begin) & 1;
    if (b + 1 < b_end) load_tile(b + 1, s ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t kbase = smem_u32(sK + s * TILE), vbase = smem_u32(sV + s * TILE);
    // S = Q K^T for 64 positions
    float sc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
    {
      const int mi = lane >> 3, kr = (lane & 7) + 8 * (mi >> 1), kc = mi & 1;
#pragma unroll
      for (int n = 0; n < NT; n += 2)
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + swz<HD>(8 * n + kr, 2 * kk + kc), b0, b1, b2, b3);
          mma_bf16(sc[n], qf[kk], b0, b1);
          mma_bf16(sc[n + 1], qf[kk], b2, b3);
        }
    }
    // scale, mask, block maxima of the two rows
    const int j0 = b * MQ_KEYS + 2 * (lane & 3);
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int j = j0 + 8 * n;
      sc[n][0] = j < lim_a ? sc[n][0] * p.scale : -INFINITY;
      sc[n][1] = j + 1 < lim_a ? sc[n][1] * p.scale : -INFINITY;
      sc[n][2] = j < lim_b ? sc[n][2] * p.scale : -INFINITY;
      sc[n][3] = j + 1 < lim_b ? sc[n][3] * p.scale : -INFINITY;
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
    for (int n = 0; n < NT; ++n) {
      sc[n][0] = exp2f(sc[n][0] - u_a);
      sc[n][1] = exp2f(sc[n][1] - u_a);
      sc[n][2] = exp2f(sc[n][2] - u_b);
      sc[n][3] = exp2f(sc[n][3] - u_b);
      l_a += sc[n][0] + sc[n][1];
      l_b += sc[n][2] + sc[n][3];
    }
    // O += P V, P as bf16 high part + bf16 remainder
    {
      const int mi = lane >> 3, vr = (lane & 7) + 8 * (mi & 1), vc = mi >> 1;
#pragma unroll
      for (int kk = 0; kk < MQ_KEYS / 16; ++kk) {
        uint32_t ph[4], pl[4];
        split_pair(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
        split_pair(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
        split_pair(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
        split_pair(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
        for (int n = 0; n < ND; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + swz<HD>(16 * kk + vr, n + vc), b0, b1, b2, b3);
          mma_bf16(o[n], ph, b0, b1);
          mma_bf16(o[n], pl, b0, b1);
          mma_bf16(o[n + 1], ph, b2, b3);
          mma_bf16(o[n + 1], pl, b2, b3);
        }
      }
    }
    __syncthreads();  // stage s is refilled two blocks on
  }
  cp_async_wait<0>();

  // row sums over the quad, then one partial per (row, split)
#pragma unroll
  for (int x = 1; x < 4; x <<= 1) {
    l_a += __shfl_xor_sync(~0u, l_a, x);
    l_b += __shfl_xor_sync(~0u, l_b, x);
  }
  const int cb = 2 * (lane & 3);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int rg = half ? rb8 : ra;
    if (rg >= rows) continue;
    const int t = rg / GQ, h = kvh * GQ + (rg - t * GQ);
    float* dst = p.ws + (((size_t)t * p.H + h) * p.nsplit + split) * (HD + 2);
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      dst[8 * n + cb] = o[n][2 * half];
      dst[8 * n + cb + 1] = o[n][2 * half + 1];
    }
    if ((lane & 3) == 0) {
      dst[HD] = half ? m_b : m_a;
      dst[HD + 1] = half ? l_b : l_a;
    }
  }
}

template <int HD>
__global__ void attn_mq_combine_kernel(const float* ws, int H, int nsplit, uint16_t* out) {
  const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  const float* src = ws + ((size_t)t * H + h) * nsplit * (HD + 2);
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
  out[((size_t)t * H + h) * HD + d] = f2bf(ll > 0.f ? oo / ll : 0.f);
}

// Splits: about four CTAs per SM over (row block, KV head, split), at most one per
// 64-position tile and MQ_SPLIT_CAP; `keys` bounds the positions any row may see.
static int mq_nsplit(int T, int H, int KV, int keys) {
  const int rows = T * (H / KV);
  const int rblocks = (rows + MQ_ROWS - 1) / MQ_ROWS;
  const int target = 4 * iron_num_sms();
  int ns = (target + rblocks * KV - 1) / (rblocks * KV);
  const int tiles = (keys + MQ_KEYS - 1) / MQ_KEYS;
  if (ns > tiles) ns = tiles;
  if (ns > MQ_SPLIT_CAP) ns = MQ_SPLIT_CAP;
  return ns < 1 ? 1 : ns;
}

template <int HD>
static int mq_smem() {
  return MQ_ROWS * HD * 2 + 4 * MQ_KEYS * HD * 2;
}

template <int HD>
static void mq_launch(dim3 g, const MqParams& p, cudaStream_t st) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(attn_mq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, mq_smem<HD>());
    attr[dev] = true;
  }
  attn_mq_kernel<HD><<<g, MQ_THREADS, mq_smem<HD>(), st>>>(p);
}

}  // namespace iron

using namespace iron;

extern "C" int64_t iron_attn_mq_workspace_bytes(int T, int H, int KV, int HD, int max_seq) {
  if (T < 1 || KV < 1 || H % KV || max_seq < 1) return 0;
  return (int64_t)T * H * mq_nsplit(T, H, KV, max_seq) * (HD + 2) * 4;
}

extern "C" int iron_attn_mq(const uint16_t* q, const uint16_t* kv, uint16_t* out, int T, int H, int KV, int HD,
                            int max_seq, int kv_layout, int block_kv, int base, const int32_t* base_dev,
                            int kv_len, int causal, void* workspace, int64_t workspace_bytes, void* stream) {
  IRON_REQUIRE(q && kv && out && workspace, IRON_ERR_ARG, "attn_mq: null pointer");
  IRON_REQUIRE(T >= 1 && KV >= 1 && H % KV == 0 && max_seq >= 1, IRON_ERR_ARG,
               "attn_mq: bad shape T=%d H=%d KV=%d max_seq=%d", T, H, KV, max_seq);
  IRON_REQUIRE(HD == 64 || HD == 128, IRON_ERR_UNSUPPORTED, "attn_mq: head_dim %d (64 or 128)", HD);
  IRON_REQUIRE(kv_layout >= 0 && kv_layout <= 2, IRON_ERR_ARG, "attn_mq: kv_layout must be 0, 1 or 2");
  IRON_REQUIRE(kv_layout != 2 || (block_kv > 0 && max_seq % block_kv == 0), IRON_ERR_ARG,
               "attn_mq: block layout needs block_kv dividing max_seq");
  IRON_REQUIRE(kv_len >= 1 && kv_len <= max_seq, IRON_ERR_ARG, "attn_mq: kv_len %d not in [1, %d]", kv_len,
               max_seq);
  IRON_REQUIRE(base_dev || base >= 0, IRON_ERR_ARG, "attn_mq: negative base %d", base);
  IRON_REQUIRE(iron_aligned(kv, 16) && iron_aligned(q, 16), IRON_ERR_ALIGN,
               "attn_mq: q and kv must be 16-byte aligned");
  IRON_REQUIRE(workspace_bytes >= iron_attn_mq_workspace_bytes(T, H, KV, HD, max_seq), IRON_ERR_ARG,
               "attn_mq: workspace of %lld bytes is too small", (long long)workspace_bytes);
  MqParams p;
  p.q = q;
  p.kv = kv;
  p.ws = (float*)workspace;
  p.T = T;
  p.H = H;
  p.KV = KV;
  p.max_seq = max_seq;
  p.layout = kv_layout;
  p.block_kv = block_kv;
  p.kv_len = kv_len;
  p.causal = causal ? 1 : 0;
  p.base = base;
  p.base_dev = base_dev;
  p.scale = 1.4426950408889634f / sqrtf((float)HD);
  // the split count bounds the positions from the host's view: with the base on
  // the device every position below kv_len may be visible
  const int keys = (causal && !base_dev) ? std::min(kv_len, base + T) : kv_len;
  p.nsplit = std::min(mq_nsplit(T, H, KV, keys), mq_nsplit(T, H, KV, max_seq));
  const int rblocks = (T * (H / KV) + MQ_ROWS - 1) / MQ_ROWS;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 g(rblocks, KV, p.nsplit);
  if (HD == 128)
    mq_launch<128>(g, p, st);
  else
    mq_launch<64>(g, p, st);
  int rc = iron_check_launch("attn_mq_kernel");
  if (rc) return rc;
  dim3 gc(H, T);
  if (HD == 128)
    attn_mq_combine_kernel<128><<<gc, 128, 0, st>>>(p.ws, H, p.nsplit, out);
  else
    attn_mq_combine_kernel<64><<<gc, 64, 0, st>>>(p.ws, H, p.nsplit, out);
  return iron_check_launch("attn_mq_combine_kernel");
}
