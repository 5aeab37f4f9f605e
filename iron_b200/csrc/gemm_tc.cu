// Batched int8 group-quantised projections on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), for decode batches of 16..256 streams.
//
// At batch >= 16 a decode projection Y[b, m] = sum_k q[m,k] s[m,k/G] x[b,k] is a real
// (skinny) contraction.  The weight streams once per launch (the 8-row launches of
// the exact GEMV would stream it batch/8 times):
//   - warp 0 (one lane) issues TMA copies per 64-column k-block: the int8 rows of a
//     128-row tile (box 64 x 128, no swizzle) and the activations (box 64 x N bf16,
//     128-byte swizzle, rows past the batch zero-filled), plus the tile's group
//     scales for its whole K range once;
//   - warps 1-8 dequantise the tile: w = q * s is exact in float32 (an 8-bit q times
//     the 8-bit significand of s), and is written as two bf16 planes, hi = bf16(w) and
//     lo = w - hi (exact in bf16: the low 8 of w's 16 significant bits), straight into
//     the 128-byte-swizzled K-major layout the tensor core reads; after the last
//     k-block they run the epilogue (warp w reads TMEM lane quarter w % 4, half of the
//     columns each);
//   - warp 9 allocates TMEM (N float32 columns per output tile, 2N for a gate/up
//     pair), one lane issues tcgen05.mma (M = 128, N = batch padded to 16, K = 16 per
//     instruction, bf16 x bf16 -> f32) for the hi and the lo plane into the same
//     accumulator and commits each k-block's MMAs to the stage's mbarrier, which frees
//     the stage for the next copies.
// K is split over CTAs so that the grid fills the GPU; each split writes its float32
// partial tile to a fixed scratch array and the tile's last split (per-tile arrival
// counter) adds the partials in split order and applies the epilogue, so results do
// not depend on timing.
//
// Numerics: every product q * s * x is exact (hi and lo planes times the bf16
// activation, each product exact in float32), sums in float32 on the tensor core, the
// same bf16 epilogues as the exact GEMV: the exact dequantised sum up to float32
// summation order.  A single bf16 plane (bf16(q * s), 2^-9 relative per weight) flipped
// enough bf16 roundings that a batch-32 Qwen3 step's logits left the bf16 gate.
//
// Every wait is bounded by %globaltimer; on a timeout the CTA records an error code
// in the status word of its workspace (iron_tc_status), lets its copies and MMAs finish
// (bounded), frees its TMEM and returns.  All scratch (status word, split-K arrival
// counters, float32 partial tiles, RMS-normalised activations) lives in the caller's
// workspace (iron_tc_workspace_bytes), so launches with their own workspaces may run on
// different streams at once.  Every split arrives at its tile's counter, aborted ones
// too, and the last one resets it: a timed-out launch leaves no counter mid-count.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {
namespace tc {

constexpr int BM = 128;         // weight rows per tile (the MMA's M)
constexpr int BK = 64;          // k per stage: one 128-byte swizzled bf16 row
constexpr int NDQ = 8;          // dequantising / epilogue warps (1..8)
constexpr int NTH = 32 * (NDQ + 2);  // warp 0 TMA, warps 1..NDQ dequant + epilogue, warp NDQ+1 MMA
constexpr int MMA_WARP = NDQ + 1;
constexpr int SMEM_MAX = 227 * 1024;
constexpr int SMEM_CTA = 113 * 1024;  // two CTAs per SM
constexpr size_t WS_FLOATS = 4u << 20;  // 16 MB of split-K partials per row block
constexpr int MAX_TILES = 4096;         // weight tiles of one launch
// split-K arrival counters: a fixed region at the head of every workspace, so that
// projections of different shapes sharing one workspace (one after another) never
// find their counters where another left its partial tiles
constexpr int COUNTERS = 16384;
// activation rows of a row block: 128 leaves room for 3 pipeline stages (a 256-row block
// for 2; the prefill's contractions: 5.20 ms with 256, 5.01 ms with 128 per 1024-token
// prompt)
constexpr int BLOCK_ROWS = 128;
constexpr int MAX_ROWS = 4096;          // activation rows of one launch
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;
// Fewest k-blocks per split.  Measured on the batch-32 Qwen3-0.6B step: 2 -> 8,460
// tok/s, 4 -> 9,826, 6 -> 9,354, 8 -> 9,331 (more splits add reduction work to
// the last CTA; fewer leave the small-M projections with too few CTAs).
constexpr int MIN_KB = 4;


struct TcParams {
  int M, K, N, nb;              // N: MMA n (activation rows of a row block, padded to 16); nb: rows
  int splits, kbps;             // k-block splits and k-blocks per split
  int sbox;                     // bytes of scales loaded per row and split
  int stages, ncols;            // pipeline stages, TMEM columns
  int epi;
  const uint16_t* res;
  void* y;
  int ld_y;
  uint32_t xor_mask;
  int* status;    // the workspace's error word
  int* counters;  // [row blocks][tiles] split-K arrival counters (zero between launches)
  float* part;    // [row blocks][tiles][splits][NW * N][BM] float32 partial tiles
  int off_a, off_x, off_raw, off_scale, off_bar;
};

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
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
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the phase of parity `par`; on a timeout (or another role's abort)
// sets the abort flag and returns false.
__device__ __forceinline__ bool wait_phase(uint64_t* b, uint32_t par, volatile int* abort_, int code, int* status) {
  if (mbar_test(b, par)) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_test(b, par)) return true;
    if ((it & 15) == 0) {
      if (*abort_) return false;
      if (gtimer() - t0 > TIMEOUT_NS) {
        *abort_ = 1;
        atomicExch(status, code);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(sa(dst)),
      "l"(map), "r"(x), "r"(y), "r"(sa(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte-swizzled UMMA shared-memory descriptor: 8-row groups 1024 B apart
// (stride byte offset), leading byte offset unused (1), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void bar_epi() { asm volatile("bar.sync 1, %0;" ::"n"(32 * NDQ) : "memory"); }

// bf16(lo) in the low half, bf16(hi) in the high half: one round-to-nearest-even
// conversion instruction for the pair
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// W16: the weight is bf16 already (the tied lm_head, bf16 GEMVs): TMA writes its
// tiles in the swizzled layout directly and warps 1-4 only run the epilogue.
template <int G, bool PAIR, bool W16>
__global__ void __launch_bounds__(NTH, 2)
    gemm_tc_kernel(const __grid_constant__ TcParams p, const __grid_constant__ CUtensorMap tm_raw0,
                   const __grid_constant__ CUtensorMap tm_sc0, const __grid_constant__ CUtensorMap tm_raw1,
                   const __grid_constant__ CUtensorMap tm_sc1, const __grid_constant__ CUtensorMap tm_x) {
  static_assert(!(W16 && PAIR), "bf16 weights: single projections only");
  constexpr int NW = PAIR ? 2 : 1;
  extern __shared__ uint8_t sm_dyn[];
  // 1024-byte alignment for the swizzled tiles (the launch adds 1 KB of slack)
  uint8_t* sm = sm_dyn + ((1024 - (sa(sm_dyn) & 1023)) & 1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x / p.splits, split = blockIdx.x - tile * p.splits;
  // blockIdx.y: the row block of N activation rows starting at row bofs; tix numbers the
  // (row block, weight tile) pairs for the split-K partials and counters
  const int tix = blockIdx.y * (gridDim.x / p.splits) + tile, bofs = blockIdx.y * p.N;
  const int row0 = tile * BM;
  const int kb0 = split * p.kbps;
  const int nkb = min(p.kbps, p.K / BK - kb0);
  const int k0 = kb0 * BK;
  const int N = p.N, S = p.stages;
  constexpr int APL = W16 ? 1 : 2;     // bf16 planes of the weight tile (hi, lo)
  uint8_t* atile = sm + p.off_a;      // [S][NW][APL][128 rows][128 B] bf16, swizzled
  uint8_t* xtile = sm + p.off_x;      // [S][N rows][128 B] bf16, swizzled
  uint8_t* raw = sm + p.off_raw;      // [S][NW][128 rows][64 B] int8
  uint8_t* scales = sm + p.off_scale; // [NW][128 rows][sbox B] bf16 group scales
  uint64_t* bars = (uint64_t*)(sm + p.off_bar);
  uint64_t* raw_full = bars;          // TMA bytes of a stage landed
  uint64_t* a_full = bars + S;        // the stage's A tiles dequantised (4 warps)
  uint64_t* freeb = bars + 2 * S;     // the stage's MMAs done (tcgen05.commit)
  uint64_t* sc_full = bars + 3 * S;
  uint64_t* acc_full = sc_full + 1;
  uint32_t* tmem_slot = (uint32_t*)(acc_full + 1);
  volatile int* abort_ = (volatile int*)(tmem_slot + 1);
  volatile int* lastf = abort_ + 1;
  volatile int* gof = abort_ + 2;
  // the split's first group gfirst sits sdelta bytes into its 16-byte-aligned scale box
  const int gfirst = k0 / G;
  const int sdelta = (2 * gfirst) & 15;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&a_full[i], NDQ);
      mbar_init(&freeb[i], 1);
    }
    mbar_init(sc_full, 1);
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_ = 0;
    *lastf = 0;
    *gof = 0;
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(tmem_slot)),
                 "r"(p.ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {  // ---- TMA producer ----
    int issued = 0;
    if (lane == 0 && nkb > 0) {
      if (!W16) {
        const int xs = p.K + 2 * gfirst - sdelta;
        mbar_expect(sc_full, (uint32_t)(NW * BM * p.sbox));
        tma_2d(scales, &tm_sc0, xs, row0, sc_full);
        if (PAIR) tma_2d(scales + BM * p.sbox, &tm_sc1, xs, row0, sc_full);
      }
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        if (i >= S && !wait_phase(&freeb[s], (uint32_t)((i / S - 1) & 1), abort_, 1, p.status)) break;
        const int kx = k0 + i * BK;
        if (W16) {
          mbar_expect(&raw_full[s], (uint32_t)(BM * 128 + N * 128));
          tma_2d(atile + (size_t)s * BM * 128, &tm_raw0, kx, row0, &raw_full[s]);
        } else {
          mbar_expect(&raw_full[s], (uint32_t)(NW * BM * BK + N * 128));
          tma_2d(raw + (size_t)(s * NW) * BM * BK, &tm_raw0, kx, row0, &raw_full[s]);
          if (PAIR) tma_2d(raw + (size_t)(s * NW + 1) * BM * BK, &tm_raw1, kx, row0, &raw_full[s]);
        }
        tma_2d(xtile + (size_t)s * N * 128, &tm_x, kx, bofs, &raw_full[s]);
        issued = i + 1;
      }
      // no copy may still be in flight when the CTA exits
      for (int i = max(0, issued - S); i < issued; ++i) {
        const unsigned long long t0 = gtimer();
        while (!mbar_test(&raw_full[i % S], (uint32_t)((i / S) & 1)) && gtimer() - t0 < 20ull * 1000 * 1000) {
        }
      }
      const unsigned long long t0 = gtimer();
      while (!W16 && !mbar_test(sc_full, 0) && gtimer() - t0 < 20ull * 1000 * 1000) {
      }
    }
  } else if (warp == MMA_WARP) {  // ---- MMA issuer ----
    if (lane == 0 && nkb > 0) {
      // kind::f16: D float32, A and B bf16, both K-major, N = p.N, M = 128
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                             ((uint32_t)(BM >> 4) << 24);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t par = (uint32_t)((i / S) & 1);
        if (!wait_phase(&raw_full[s], par, abort_, 2, p.status) ||
            (!W16 && !wait_phase(&a_full[s], par, abort_, 3, p.status)))
          break;
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(sa(xtile + (size_t)s * N * 128));
#pragma unroll
        for (int w = 0; w < NW; ++w)
#pragma unroll
          for (int pl = 0; pl < APL; ++pl) {
            const uint64_t adesc = sw128_desc(sa(atile + ((size_t)(s * NW + w) * APL + pl) * BM * 128));
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)  // +32 bytes per 16 columns inside the swizzle atom
              mma_bf16(tmem + (uint32_t)(w * N), adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), idesc,
                       (i > 0 || kk > 0 || pl > 0) ? 1u : 0u);
          }
        mma_commit(&freeb[s]);
      }
      mma_commit(acc_full);  // arrives once every MMA issued above has completed
    }
  } else {  // ---- warps 1..NDQ: dequantise, then the epilogue ----
    const int t = tid - 32;  // 0 .. 32 * NDQ - 1
    // lane 0 waits and the warp follows its answer: warp-uniform control flow
    auto wait_warp = [&](uint64_t* b, uint32_t par, int code) -> bool {
      int r = 1;
      if (lane == 0) r = wait_phase(b, par, abort_, code, p.status);
      r = __shfl_sync(~0u, r, 0);
      if (r) mbar_test(b, par);  // every lane observes the completed phase
      return r != 0;
    };
    bool ok = nkb > 0 && (W16 || wait_warp(sc_full, 0, 4));
    for (int i = 0; !W16 && ok && i < nkb; ++i) {
      const int s = i % S;
      if (!wait_warp(&raw_full[s], (uint32_t)((i / S) & 1), 5)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const uint8_t* rt = raw + (size_t)(s * NW + w) * BM * BK;
        uint8_t* at = atile + (size_t)(s * NW + w) * APL * BM * 128;  // hi plane, lo plane after it
        const uint16_t* sc = (const uint16_t*)(scales + (size_t)w * BM * p.sbox);
#pragma unroll
        for (int it = 0; it < 4 * 4 / NDQ; ++it) {
          const int r = (t >> 2) + 8 * NDQ * it, c = t & 3;  // row, 16-column chunk
          uint4 q = *(const uint4*)(rt + r * BK + c * 16);
          // signed payload byte b -> b + 128 (the biased domain is already b + 128)
          const uint32_t flip = p.xor_mask ^ 0x80808080u;
          const uint32_t qw[4] = {q.x ^ flip, q.y ^ flip, q.z ^ flip, q.w ^ flip};
          const int g = (k0 + i * BK + c * 16) / G;
          const float sf = bf2f(sc[(size_t)r * (p.sbox >> 1) + (sdelta >> 1) + (g - gfirst)]);
          // -(2^23 + 2^7) * s is exact: the 8-bit significand of s shifted by 7 and by 23
          // spans 24 bits
          const float soff = -8388736.0f * sf;
          uint32_t o[8], ol[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // one byte permute gives the float 2^23 + (b + 128); one fma with s and soff
            // gives b * s, exact in float32 (8-bit b times 8-bit s); hi = bf16(b * s) and
            // lo = b * s - hi, both exact in bf16
            float f[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              f[j] = fmaf(__uint_as_float(__byte_perm(qw[e], 0x4B000000u, 0x7440u | (uint32_t)j)), sf, soff);
            o[2 * e] = pack_bf16x2(f[0], f[1]);
            o[2 * e + 1] = pack_bf16x2(f[2], f[3]);
            ol[2 * e] = pack_bf16x2(f[0] - bf_lo(o[2 * e]), f[1] - bf_hi(o[2 * e]));
            ol[2 * e + 1] = pack_bf16x2(f[2] - bf_lo(o[2 * e + 1]), f[3] - bf_hi(o[2 * e + 1]));
          }
          // 16-byte chunk j of row r sits at chunk j ^ (r & 7) (128-byte swizzle)
          const int c0 = r * 128 + (((2 * c) ^ (r & 7)) << 4), c1 = r * 128 + (((2 * c + 1) ^ (r & 7)) << 4);
          *(uint4*)(at + c0) = make_uint4(o[0], o[1], o[2], o[3]);
          *(uint4*)(at + c1) = make_uint4(o[4], o[5], o[6], o[7]);
          *(uint4*)(at + BM * 128 + c0) = make_uint4(ol[0], ol[1], ol[2], ol[3]);
          *(uint4*)(at + BM * 128 + c1) = make_uint4(ol[4], ol[5], ol[6], ol[7]);
        }
      }
      fence_proxy_async();  // the tensor core reads these stores through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
    // ---- epilogue: warp w owns TMEM lane quarter w % 4 (tile rows 32q..32q+31) and
    // the column half (w - 1) / 4 ----
    ok = ok && wait_warp(acc_full, 0, 6);
    if (!ok && lane == 0) *abort_ = 1;
    bar_epi();  // the epilogue warps take one decision
    if (t == 0) *gof = *abort_ ? 0 : 1;
    bar_epi();
    ok = *gof != 0;
    tc_fence_after();
    const int q = warp & 3, row = 32 * q + lane, m = row0 + row;
    const int half = (warp - 1) / 4;  // columns [half * N/2, (half + 1) * N/2) in 16-column steps
    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
    auto finish_at = [&](int mr, int b, float a0, float a1) {
      if (b >= p.nb || mr >= p.M) return;
      uint16_t* yo = (uint16_t*)p.y + (size_t)b * p.ld_y + mr;
      if (PAIR) {
        *yo = f2bf(silu_tanh_bf16(rbf(a0)) * rbf(a1));
      } else if (p.epi == EPI_RESID) {
        *yo = f2bf(bf2f(p.res[(size_t)b * p.ld_y + mr]) + rbf(a0));
      } else if (p.epi == EPI_F32) {
        ((float*)p.y)[(size_t)b * p.ld_y + mr] = a0;
      } else {
        *yo = f2bf(a0);
      }
    };
    auto finish = [&](int b, float a0, float a1) { finish_at(m, bofs + b, a0, a1); };
    if (ok) {
      float* part = p.part + ((size_t)(tix * p.splits + split) * NW * N) * BM;
      for (int c0 = 16 * half; c0 < N; c0 += 32) {
        float v[16], u[16];
        tmem_ld16(taddr + (uint32_t)c0, v);
        if (PAIR) tmem_ld16(taddr + (uint32_t)(N + c0), u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (p.splits == 1) {
            finish(c0 + j, v[j], PAIR ? u[j] : 0.f);
          } else {
            part[(size_t)(c0 + j) * BM + row] = v[j];
            if (PAIR) part[(size_t)(N + c0 + j) * BM + row] = u[j];
          }
        }
      }
    }
    if (p.splits > 1 && nkb > 0) {
      // every split arrives, aborted ones too, and the last resets the counter
      __threadfence();
      bar_epi();
      if (t == 0) {
        *lastf = atomicAdd(&p.counters[tix], 1) == p.splits - 1;
        if (*lastf) p.counters[tix] = 0;
      }
      bar_epi();
      if (*lastf && ok) {
          __threadfence();
          // Thread t sums rows 4(t % 32) .. +3 (float4 loads) of the columns c = t / 32
          // (mod 8): CB columns x U splits x NW float4 loads in flight (fewer for a pair,
          // whose registers are shared with the second accumulator), added in split order
          // as always.  The partial tiles are [split][NW][column][row].
          constexpr int CB = PAIR ? 2 : 4, U = PAIR ? 2 : 4, CS = 32 * NDQ / (BM / 4);  // column stride: 8
          const int r4 = 4 * (t % (BM / 4)), cofs = t / (BM / 4);
          const float* base = p.part + (size_t)tix * p.splits * NW * N * BM + r4;
          for (int b0 = cofs; b0 < N; b0 += CS * CB) {
            float4 a0[CB], a1[CB];
#pragma unroll
            for (int c = 0; c < CB; ++c) a0[c] = a1[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s0 = 0; s0 < p.splits; s0 += U) {
              float4 v0[U][CB], v1[U][CB];
#pragma unroll
              for (int u = 0; u < U; ++u) {
                const float* pp = base + (size_t)(s0 + u) * NW * N * BM;
#pragma unroll
                for (int c = 0; c < CB; ++c) {
                  const int b = b0 + CS * c;
                  const bool in = s0 + u < p.splits && b < N;
                  v0[u][c] = in ? __ldcg((const float4*)(pp + (size_t)b * BM)) : make_float4(0.f, 0.f, 0.f, 0.f);
                  v1[u][c] = (PAIR && in) ? __ldcg((const float4*)(pp + (size_t)(N + b) * BM))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                }
              }
#pragma unroll
              for (int u = 0; u < U; ++u)
                if (s0 + u < p.splits) {
#pragma unroll
                  for (int c = 0; c < CB; ++c) {
                    a0[c].x += v0[u][c].x;
                    a0[c].y += v0[u][c].y;
                    a0[c].z += v0[u][c].z;
                    a0[c].w += v0[u][c].w;
                    if (PAIR) {
                      a1[c].x += v1[u][c].x;
                      a1[c].y += v1[u][c].y;
                      a1[c].z += v1[u][c].z;
                      a1[c].w += v1[u][c].w;
                    }
                  }
                }
            }
#pragma unroll
            for (int c = 0; c < CB; ++c) {
              const int b = b0 + CS * c;
              if (b >= N) continue;
              finish_at(row0 + r4, bofs + b, a0[c].x, a1[c].x);
              finish_at(row0 + r4 + 1, bofs + b, a0[c].y, a1[c].y);
              finish_at(row0 + r4 + 2, bofs + b, a0[c].z, a1[c].z);
              finish_at(row0 + r4 + 3, bofs + b, a0[c].w, a1[c].w);
            }
          }
        }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    // MMAs may still run after an abort: wait (bounded) for the final commit first
    const unsigned long long t0 = gtimer();
    while (nkb > 0 && !mbar_test(acc_full, 0) && gtimer() - t0 < 20ull * 1000 * 1000) {
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.ncols) : "memory");
  }
}

// rms-normalised activations for a batched launch: y[b] = bf16(RMSNorm_w(x[b])), the
// prologue arithmetic of the GEMV kernels
__global__ void rms_rows_kernel(const uint16_t* x, int ld_x, const uint16_t* w, int K, float eps, int mode,
                                uint16_t* y) {
  const int b = blockIdx.x;
  const uint16_t* xr = x + (size_t)b * ld_x;
  __shared__ double red[32];
  double ss = 0.0;
  for (int i = threadIdx.x; i < K; i += blockDim.x) ss += rms_sq(bf2f(xr[i]), mode);
  ss = warp_sum_d(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const RmsCoef rc = rms_coef(red[0], K, eps, mode);
  for (int i = threadIdx.x; i < K; i += blockDim.x)
    y[(size_t)b * K + i] = f2bf(rms_apply(bf2f(xr[i]), bf2f(w[i]), rc));
}


}  // namespace tc

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
  }
  return fn;
}

static bool map2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                  uint64_t stride1_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The activation rows of a launch in nt row blocks of N rows each (N a multiple of 16,
// at most BLOCK_ROWS; the blocks are one grid row each and share the weight tiles, which
// they read from L2 after the first)
static void tc_rows(int nb, int& N, int& nt) {
  using namespace tc;
  nt = nb > BLOCK_ROWS ? (nb + BLOCK_ROWS - 1) / BLOCK_ROWS : 1;
  N = ((nb + nt - 1) / nt + 15) / 16 * 16;
}

// K split over CTAs so that they make about one wave (two per SM for one row block, one
// per SM for several: their stages fill an SM), at least MIN_KB k-blocks per split (a
// shorter split is mostly start-up, and every split adds a partial tile to the last
// CTA's reduction), the partials within WS_FLOATS per row block
static void tc_split_plan(int M, int K, int N, int NW, int nt, int& splits, int& kbps) {
  using namespace tc;
  const int tiles = (M + BM - 1) / BM * nt;  // (row block, weight tile) pairs
  const int kblocks = K / BK;
  splits = (nt > 1 ? 1 : 2) * iron_num_sms() / tiles;
  // from 128 rows on, each k-block is a large MMA and every split adds a large partial
  // tile to the reduction: twice the floor (1024x3072 at 256 rows: 40.0 -> 33.2 us)
  const int min_kb = N >= 128 ? 2 * MIN_KB : MIN_KB;
  if (splits > kblocks / min_kb) splits = kblocks / min_kb;
  if (splits < 1) splits = 1;
  kbps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kbps - 1) / kbps;
  while (splits > 1 && (size_t)tiles * splits * NW * N * BM > WS_FLOATS * nt) {
    kbps *= 2;
    splits = (kblocks + kbps - 1) / kbps;
  }
}

static size_t r256(size_t n) { return (n + 255) & ~(size_t)255; }

// Workspace layout: [status word | COUNTERS counters | partials | normalised activations |
// gate outputs of a split pair | up outputs]
struct TcWs {
  int* status;
  int* counters;
  float* part;
  uint16_t* xnorm;
  uint16_t* gs;  // a gate/up pair above 128 rows: the gate and up outputs (nb x M bf16 each)
  uint16_t* us;
};

// A gate/up pair of more than 128 activation rows runs as two single contractions
// (gate, then up) and a SiLU * up pass: the pair's two weight tiles per stage leave
// room for only two pipeline stages at that width.
static bool tc_split_pair(int NW, int nb) { return NW == 2 && nb > 128; }
static size_t tc_ws_need(int M, int K, int nb, int NW, bool rms) {
  using namespace tc;
  const bool sp = tc_split_pair(NW, nb);
  if (sp) NW = 1;
  int N, nt;
  tc_rows(nb, N, nt);
  const int tiles = (M + BM - 1) / BM * nt;
  int splits, kbps;
  tc_split_plan(M, K, N, NW, nt, splits, kbps);
  size_t n = 256 + (size_t)COUNTERS * 4;
  if (splits > 1) n += r256((size_t)tiles * splits * NW * N * BM * 4);
  if (rms) n += r256((size_t)nb * K * 2);
  if (sp) n += 2 * r256((size_t)nb * M * 2);
  return n;
}
static bool tc_ws_carve(void* ws, int64_t bytes, int M, int K, int nb, int NW, bool rms, TcWs& o) {
  using namespace tc;
  if (!ws || !iron_aligned(ws, 256) || (size_t)bytes < tc_ws_need(M, K, nb, NW, rms)) return false;
  const bool sp = tc_split_pair(NW, nb);
  if (sp) NW = 1;
  int N, nt;
  tc_rows(nb, N, nt);
  const int tiles = (M + BM - 1) / BM * nt;
  if (tiles > COUNTERS) return false;
  int splits, kbps;
  tc_split_plan(M, K, N, NW, nt, splits, kbps);
  uint8_t* b = (uint8_t*)ws;
  o.status = (int*)b;
  size_t off = 256;
  o.counters = (int*)(b + off);
  off += (size_t)COUNTERS * 4;
  o.part = (float*)(b + off);
  if (splits > 1) off += r256((size_t)tiles * splits * NW * N * BM * 4);
  o.xnorm = (uint16_t*)(b + off);
  if (rms) off += r256((size_t)nb * K * 2);
  o.gs = sp ? (uint16_t*)(b + off) : nullptr;
  if (sp) off += r256((size_t)nb * M * 2);
  o.us = sp ? (uint16_t*)(b + off) : nullptr;
  return true;
}

// y[b, m] = bf16(silu_tanh(g) * u) of the split pair's two outputs (the pair epilogue),
// eight values per thread with 16-byte accesses (M and ld_y multiples of 8, y 16-byte
// aligned; the caller checks)
__global__ void silu_mul_rows_kernel(const uint16_t* g, const uint16_t* u, int M, int nb, uint16_t* y, int ld_y) {
  const unsigned m8 = (unsigned)M / 8, n = (unsigned)nb * m8;  // nb * M / 8 < 2^31 (the caller's rows)
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned b = i / m8, m = (i - b * m8) * 8;
    const uint4 gv = __ldcg((const uint4*)(g + (size_t)b * M + m));
    const uint4 uv = __ldcg((const uint4*)(u + (size_t)b * M + m));
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint16_t lo = f2bf(silu_tanh_bf16(bf_lo(gw[e])) * bf_lo(uw[e]));
      const uint16_t hi = f2bf(silu_tanh_bf16(bf_hi(gw[e])) * bf_hi(uw[e]));
      o[e] = lo | ((uint32_t)hi << 16);
    }
    *(uint4*)(y + (size_t)b * ld_y + m) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The split plan is the one the workspace was carved with (the same rows and weights),
// so this launch's partial tiles fit the carved region
template <int G, bool PAIR>
static int tc_launch(const GemvW8Params& p, const uint16_t* x, int ld_x, const TcWs& ws, cudaStream_t st) {
  using namespace tc;
  constexpr int NW = PAIR ? 2 : 1;
  const int M = p.M, K = p.K, nb = p.nb;
  int N, nt;
  tc_rows(nb, N, nt);
  const int tiles = (M + BM - 1) / BM;
  if (tiles > MAX_TILES) return 1;
  int splits, kbps;
  tc_split_plan(M, K, N, NW, nt, splits, kbps);
  TcParams tp = {};
  tp.status = ws.status;
  tp.counters = ws.counters;
  tp.part = ws.part;
  tp.M = M;
  tp.K = K;
  tp.N = N;
  tp.nb = nb;
  tp.splits = splits;
  tp.kbps = kbps;
  // scales of a split: from the 16-byte boundary at or below its first one
  tp.sbox = ((17 + 2 * kbps * BK / G) + 15) / 16 * 16;
  if (tp.sbox > 256) return 1;
  int nc = 32;
  while (nc < NW * N) nc *= 2;
  if (nc > 512) return 1;
  tp.ncols = nc;
  tp.epi = p.epi;
  tp.res = p.res;
  tp.y = p.y;
  tp.ld_y = p.ld_y;
  tp.xor_mask = p.wa.xor_mask;
  const int per_stage = NW * 2 * BM * 128 + N * 128 + NW * BM * BK;  // hi + lo planes, activations, raw int8
  const int fixed = NW * BM * tp.sbox + 1024 /* alignment slack */ + 256 /* barriers, flags */;
  int S = (SMEM_CTA - fixed) / per_stage;
  if (S < 2) S = (SMEM_MAX - fixed) / per_stage;  // large batches: one CTA per SM
  if (S > 6) S = 6;
  if (S < 2) return 1;
  tp.stages = S;
  tp.off_a = 0;
  tp.off_x = tp.off_a + S * NW * 2 * BM * 128;
  tp.off_raw = tp.off_x + S * N * 128;
  tp.off_scale = tp.off_raw + S * NW * BM * BK;
  tp.off_bar = (tp.off_scale + NW * BM * tp.sbox + 15) / 16 * 16;
  const size_t smem = (size_t)tp.off_bar + (3 * S + 2) * 8 + 16 + 1024;  // + tmem slot, flags; + alignment
  const uint64_t RB = (uint64_t)K + 2 * (K / G);
  CUtensorMap mr0, ms0, mr1, ms1, mx;
  if (!map2d(&mr0, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wa.base, RB, M, RB, BK, BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !map2d(&ms0, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wa.base, RB, M, RB, tp.sbox, BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !map2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, nb, (uint64_t)ld_x * 2, BK, N,
             CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  mr1 = mr0;
  ms1 = ms0;
  if (PAIR && (!map2d(&mr1, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wb.base, RB, M, RB, BK, BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
               !map2d(&ms1, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.wb.base, RB, M, RB, tp.sbox, BM,
                      CU_TENSOR_MAP_SWIZZLE_NONE)))
    return 1;
  auto fn = gemm_tc_kernel<G, PAIR, false>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
    attr[dev] = true;
  }
  fn<<<dim3(tiles * splits, nt), NTH, smem, st>>>(tp, mr0, ms0, mr1, ms1, mx);
  return iron_check_launch("gemm_tc_kernel");
}

// bf16 weights: y[b, m] = bf16(sum_k A[m, k] x[b, k]), float32 accumulation.
int gemm_tc_bf16_launch(const uint16_t* A, int M, int K, const uint16_t* x, int ld_x, int nb, uint16_t* y,
                        int ld_y, void* workspace, int64_t workspace_bytes, cudaStream_t st) {
  using namespace tc;
  if (nb < 16 || nb > MAX_ROWS || K % 64 || !iron_aligned(A, 16) || !iron_aligned(x, 16) || ld_x % 8) return 1;
  int N, nt;
  tc_rows(nb, N, nt);
  const int tiles = (M + BM - 1) / BM;
  if (tiles > MAX_TILES) return 1;
  TcWs ws;
  if (!tc_ws_carve(workspace, workspace_bytes, M, K, nb, 1, false, ws)) return 1;
  int splits, kbps;
  tc_split_plan(M, K, N, 1, nt, splits, kbps);
  TcParams tp = {};
  tp.status = ws.status;
  tp.counters = ws.counters;
  tp.part = ws.part;
  tp.M = M;
  tp.K = K;
  tp.N = N;
  tp.nb = nb;
  tp.splits = splits;
  tp.kbps = kbps;
  tp.sbox = 0;
  int nc = 32;
  while (nc < N) nc *= 2;
  tp.ncols = nc;
  tp.epi = EPI_STORE;
  tp.y = y;
  tp.ld_y = ld_y;
  const int per_stage = BM * 128 + N * 128;
  int S = (SMEM_CTA - 1024 - 256) / per_stage;
  if (S < 2) S = (SMEM_MAX - 1024 - 256) / per_stage;
  if (S > 6) S = 6;
  if (S < 2) return 1;
  tp.stages = S;
  tp.off_a = 0;
  tp.off_x = S * BM * 128;
  tp.off_raw = tp.off_x + S * N * 128;
  tp.off_scale = tp.off_raw;
  tp.off_bar = tp.off_scale;
  const size_t smem = (size_t)tp.off_bar + (3 * S + 2) * 8 + 16 + 1024;
  CUtensorMap ma, mx;
  if (!map2d(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, A, K, M, (uint64_t)K * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !map2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, nb, (uint64_t)ld_x * 2, BK, N, CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  auto fn = gemm_tc_kernel<32, false, true>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
    attr[dev] = true;
  }
  fn<<<dim3(tiles * splits, nt), NTH, smem, st>>>(tp, ma, ma, ma, ma, mx);
  return iron_check_launch("gemm_tc_kernel");
}

// 0: launched (or a launch error < 0); 1: not handled (the caller runs the exact GEMV
// in 8-row launches).  Plain wires, 16 <= batch <= MAX_ROWS, K a multiple of 64 and of
// 8 * group, 16-byte aligned activations with rows a multiple of 8 elements apart.
int gemm_tc_launch(const GemvW8Params& p, bool pair, cudaStream_t st) {
  using namespace tc;
  if (p.nb < 16 || p.nb > MAX_ROWS || !p.wa.plain1 || (pair && !p.wb.plain1)) return 1;
  if (p.K % 64 || p.K % (8 * p.wa.G) || p.K > 16384) return 1;
  if (!iron_aligned(p.wa.base, 16) || (pair && !iron_aligned(p.wb.base, 16))) return 1;
  TcWs ws;  // without a workspace large enough the caller runs the exact kernel
  if (!tc_ws_carve(p.tc_ws, p.tc_ws_bytes, p.M, p.K, p.nb, pair ? 2 : 1, p.rms_w != nullptr, ws)) return 1;
  const uint16_t* x = p.x;
  int ld_x = p.ld_x;
  if (p.rms_w) {  // normalise first: the tensor-core kernel reads x through TMA
    uint16_t* xn = ws.xnorm;
    rms_rows_kernel<<<p.nb, 256, 0, st>>>(p.x, p.ld_x, p.rms_w, p.K, p.eps, p.rms_mode, xn);
    int rc = iron_check_launch("rms_rows_kernel");
    if (rc) return rc;
    x = xn;
    ld_x = p.K;
  }
  if (!iron_aligned(x, 16) || ld_x % 8) return 1;
  if (p.wa.G != 32 && p.wa.G != 64 && p.wa.G != 128) return 1;
  auto single = [&](const GemvW8Params& q) -> int {
    switch (q.wa.G) {
      case 32: return tc_launch<32, false>(q, x, ld_x, ws, st);
      case 64: return tc_launch<64, false>(q, x, ld_x, ws, st);
      default: return tc_launch<128, false>(q, x, ld_x, ws, st);
    }
  };
  if (pair && tc_split_pair(2, p.nb)) {
    // the SiLU * up pass moves 8 values per access: otherwise the exact kernel runs
    if (p.M % 8 || p.ld_y % 8 || !iron_aligned(p.y, 16)) return 1;
    // gate and up as single contractions into the workspace, then SiLU * up
    GemvW8Params q = p;
    q.epi = EPI_STORE;
    q.res = nullptr;
    q.ld_y = p.M;
    q.y = ws.gs;
    int rc = single(q);
    if (rc) return rc;  // 1 before any launch: the caller runs the exact kernel
    q.wa = p.wb;
    q.y = ws.us;
    rc = single(q);
    if (rc) return rc < 0 ? rc : iron_set_error(IRON_ERR_UNSUPPORTED, "gemm_tc: up half not launched");
    const int64_t n = (int64_t)p.nb * (p.M / 8);
    int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)iron_num_sms() * 8);
    silu_mul_rows_kernel<<<grid, 256, 0, st>>>(ws.gs, ws.us, p.M, p.nb, p.y, p.ld_y);
    return iron_check_launch("silu_mul_rows_kernel");
  }
  if (pair) {
    switch (p.wa.G) {
      case 32: return tc_launch<32, true>(p, x, ld_x, ws, st);
      case 64: return tc_launch<64, true>(p, x, ld_x, ws, st);
      default: return tc_launch<128, true>(p, x, ld_x, ws, st);
    }
  }
  return single(p);
}

}  // namespace iron

using namespace iron;

// Bytes of workspace a batch >= 16 projection of M rows x K columns needs (a gate/up
// pair with an RMSNorm prologue included; a bf16 weight needs no more).
extern "C" int64_t iron_tc_workspace_bytes(int M, int K, int batch) {
  if (M < 1 || K < 64 || batch < 16 || batch > tc::MAX_ROWS) return 256;
  return (int64_t)std::max(tc_ws_need(M, K, batch, 1, true), tc_ws_need(M, K, batch, 2, true));
}

// Error word of the tensor-core projections that used `workspace`: 0, or the code of
// the first bounded wait that timed out.  clear != 0 also resets it.  Synchronous.
extern "C" int iron_tc_status(void* workspace, int clear) {
  if (!workspace) return IRON_ERR_ARG;
  int v = 0;
  if (cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return IRON_ERR_CUDA;
  if (clear && v) {
    const int z = 0;
    if (cudaMemcpy(workspace, &z, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return IRON_ERR_CUDA;
  }
  return v;
}
