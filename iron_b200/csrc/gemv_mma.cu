// Int8 group-quantised GEMV (W8A16) for plain wires (tile_m = 1, rows contiguous)
// and batch 1..8, with the dot products on the integer tensor-core path.
//
// Data movement.  A decode GEMV is one pass over the weight.  One CTA per SM owns a
// contiguous block of output rows, cut into tiles of 16 rows.  A producer warp
// copies each tile's rows (all of K, or 4096-column pieces when K is larger) into a
// ring of shared-memory slots with one CTA-local cp.async.bulk per row and piece;
// the row stride is padded to 16 mod 128 bytes so that ldmatrix and the scale loads
// are free of bank conflicts.  Eight consumer warps take work items of
// 128..1024 columns of a slot in turn, so a small row block still gives every warp
// work; a slot is released when all its items are done.
//
// Exact dot products.  Each activation group of G values is held in block floating
// point as a 31-bit integer X = rn(v * 2^(30-e)), e the exponent bound of the
// group's absmax (the same integer as hi * 2^15 + lo of the dp2a kernels), written
// as four balanced signed bytes X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3.  One
// mma.sync m16n8k32 (s8 x s8 -> s32) multiplies 16 weight rows x 32 columns by eight
// columns (d0..d3 of two batch rows) and returns exact integer piece sums.  A lane
// holds two adjacent pieces of one batch row and folds them (d0 + 256 d1 or
// d2 + 256 d3, exact in int32), scales by the weight group scale times the
// activation scale (exact in float64) and accumulates in float64; the two lanes of
// a pair are added at the end with the 2^16 weight.  The float64 sum is rounded to
// bf16 once, with the epilogues of gemv_w8_kernel.
//
// The partial sums of a 16-row tile are added in column order by whichever warp
// finishes the tile's last item, so results do not depend on timing.
//
// Waits are bounded by %globaltimer; on a timeout the CTA stops (the outputs of its
// rows are then undefined).  The producer lane always waits (bounded) for its last
// copies to land before it returns, so no CTA exits with a copy in flight.
#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {
namespace gmma {

constexpr int NT = 256, NWARP = NT / 32;
constexpr int TR = 16;  // rows per tile (the MMA's M)
constexpr int NSLOT_MAX = 32;
constexpr int SMEM_MAX = 227 * 1024;
constexpr size_t STAGE_MAX = 120 * 1024;  // activation digits + scales (K = 12288 at batch <= 2)
constexpr unsigned long long TIMEOUT_NS = 200ull * 1000 * 1000;

struct Plan {
  int segc, nc;    // columns per copied piece of a row, pieces per row
  int cseg, nq;    // columns per work item, items per piece
  int rbp;         // shared-memory stride of a copied row (16 mod 128 bytes)
  int slot;        // bytes of one ring slot (a tile's piece, both wires in pair mode)
  int nslot;       // ring slots
  int pt;          // partial-sum tile slots (0 when a tile has one item)
  int off_ring, off_part, off_cnt, off_bar;
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
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   sa(dst)),
               "l"(src), "r"(bytes), "r"(sa(b))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t (&a)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr)
               : "memory");
}
// D = A (16x32 s8, row) * B (32x8 s8, col), exact int32
__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint2 b) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(0));
}
// Wait for the phase of parity `par` of mbarrier b; false after TIMEOUT_NS or when
// another warp gave up (the abort flag), which it then also sets.
__device__ __forceinline__ bool wait_phase(uint64_t* b, uint32_t par, volatile int* abort_) {
  if (mbar_test(b, par)) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 1;; ++it) {
    if (mbar_test(b, par)) return true;
    if ((it & 15) == 0 && (*abort_ || gtimer() - t0 > TIMEOUT_NS)) {
      *abort_ = 1;
      return false;
    }
  }
}

__host__ __device__ inline void rows_of(int M, int c, int N, int& lo, int& hi) {
  lo = (int)((long long)M * c / N);
  hi = (int)((long long)M * (c + 1) / N);
}
// One k-block's B fragments (32 lanes x 8 B) of one MMA column set take xbs(NM)
// bytes: the padding makes consecutive k-blocks of a set 8 banks apart, so the
// prologue's stores of neighbouring k-blocks spread over the banks.
__host__ __device__ constexpr int xbs(int NM) { return 256 + 32 / NM; }
// bytes of the activation staging: digits [K/32][NM][XBS], scales
// [K/G][2 NM] float64, RMS coefficients, a reduction scratch and the abort flag
__host__ __device__ inline size_t stage_bytes(int K, int G, int NM) {
  return (size_t)(K / 32) * NM * xbs(NM) + (size_t)(K / G) * 2 * NM * 8 + 2 * NM * sizeof(RmsCoef) + NWARP * 8 + 16;
  // (the last 16 bytes: the abort flag and the producer's issued-unit count)
}

template <int G, int NM, bool PAIR>
__global__ void __launch_bounds__(NT + 32, 1)
    gemv_mma_kernel(const __grid_constant__ GemvW8Params p, const __grid_constant__ Plan pl) {
  constexpr int NBP = 2 * NM;       // batch rows held (two per MMA)
  constexpr int NW = PAIR ? 2 : 1;  // wires (gate and up in pair mode)
  constexpr int XBS = xbs(NM);
  extern __shared__ __align__(128) uint8_t sm[];
  const int K = p.K, KB = K / 32, KG = K / G;
  const size_t RB = (size_t)K + 2 * KG;  // wire row bytes
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  uint8_t* xb = sm;                                            // [KB][NM] blocks of XBS bytes
  double* xsd = (double*)(sm + (size_t)KB * NM * XBS);         // [KG][NBP]
  RmsCoef* rcs = (RmsCoef*)(xsd + (size_t)KG * NBP);           // [NBP]
  double* red = (double*)(rcs + NBP);                          // [NWARP]
  volatile int* abort_ = (volatile int*)(red + NWARP);
  volatile int* issued_ = abort_ + 1;          // copy units the producer has issued
  uint8_t* ring = sm + pl.off_ring;
  double* part = (double*)(sm + pl.off_part);  // [pt][nc * nq][NW][TR][NBP]
  int* tcnt = (int*)(sm + pl.off_cnt);         // [pt]
  uint64_t* full = (uint64_t*)(sm + pl.off_bar);
  uint64_t* empty = full + pl.nslot;
  const int NS = pl.nc * pl.nq;                // work items per tile

  int r0, r1;
  rows_of(p.M, blockIdx.x, gridDim.x, r0, r1);
  const int ntile = (r1 - r0 + TR - 1) / TR;
  const int nu = ntile * pl.nc;                // copy units (tile, piece)
  if (tid == 0) {
    for (int i = 0; i < pl.nslot; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], pl.nq);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_ = 0;
    *issued_ = 0;
  }
  for (int i = tid; i < pl.pt; i += NT + 32) tcnt[i] = 0;
  __syncthreads();  // the only barrier of all NT + 32 threads

  if (wid == NWARP) {  // ---- producer warp: lane (w, row) copies row `row` of wire w ----
    const int w = lane >> 4, rl = lane & 15;
    int issued = 0;
    for (int j = 0; j < nu; ++j) {
      const int s = j % pl.nslot;
      if (j >= pl.nslot) {  // unit j - nslot must have released the slot
        int ok = 1;
        if (lane == 0) ok = wait_phase(&empty[s], (uint32_t)((j / pl.nslot - 1) & 1), abort_);
        if (!__shfl_sync(~0u, ok, 0)) break;
      }
      const int t = j / pl.nc, c = j - t * pl.nc;
      const int row0 = r0 + t * TR, nr = min(TR, r1 - row0);
      const int k0 = c * pl.segc, len = min(pl.segc, K - k0), sb = len / G * 2;
      if (lane == 0) mbar_expect(&full[s], (uint32_t)(nr * (len + sb) * NW));
      __syncwarp();
      if (w < NW && rl < nr) {
        const uint8_t* src = (w ? p.wb.base : p.wa.base) + (size_t)(row0 + rl) * RB;
        uint8_t* d = ring + (size_t)s * pl.slot + (size_t)(w * TR + rl) * pl.rbp;
        if (pl.nc == 1) {  // the whole wire row: K weights then K/G scales
          bulk_g2s(d, src, (uint32_t)RB, &full[s]);
        } else {
          bulk_g2s(d, src + k0, (uint32_t)len, &full[s]);
          bulk_g2s(d + len, src + K + (k0 / G) * 2, (uint32_t)sb, &full[s]);
        }
      }
      __syncwarp();
      if (lane == 0) {  // consumers test the slot's phase only once unit j is armed
        __threadfence_block();
        *issued_ = j + 1;
      }
      issued = j + 1;
    }
    if (lane == 0) {  // the CTA must not exit while copies are in flight: wait for the last ones
      for (int k = max(0, issued - pl.nslot); k < issued; ++k) {
        const unsigned long long t0 = gtimer();
        while (!mbar_test(&full[k % pl.nslot], (uint32_t)((k / pl.nslot) & 1)) &&
               gtimer() - t0 < 20ull * 1000 * 1000) {
        }
      }
    }
    return;
  }

  // ---- prologue: activations -> (optionally RMS-normalised) bf16 -> digits ----
  if (p.rms_w) {
    for (int b = 0; b < p.nb; ++b) {
      const uint16_t* xr = p.x + (size_t)b * p.ld_x;
      double ss = 0.0;
      for (int i = tid; i < K; i += NT) ss += rms_sq(bf2f(xr[i]), p.rms_mode);
      ss = warp_sum_d(ss);
      if (lane == 0) red[wid] = ss;
      csync();
      ss = warp_sum_d(lane < NWARP ? red[lane] : 0.0);
      if (tid == 0) rcs[b] = rms_coef(ss, K, p.eps, p.rms_mode);
      csync();  // red is reused by the next row; rcs[b] is read below
    }
  }
  {
    // Thread per 8-value chunk, TEAM = G / 8 consecutive lanes per quantisation group,
    // U chunks' loads in flight per thread.  Batch rows >= nb are not staged: their
    // digits are never stored outputs, and their scales are zeroed.
    constexpr int TEAM = G / 8, U = 4;
    const int cpr = K / 8, nchunk = p.nb * cpr;
    for (int c0 = 0; c0 < nchunk; c0 += NT * U) {
      uint4 raw[U], rw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * NT + tid;
        raw[u] = rw[u] = make_uint4(0u, 0u, 0u, 0u);
        if (c < nchunk) {
          const int b = c / cpr, k = (c - b * cpr) * 8;
          raw[u] = __ldg((const uint4*)(p.x + (size_t)b * p.ld_x + k));
          if (p.rms_w) rw[u] = __ldg((const uint4*)(p.rms_w + k));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * NT + tid;
        const bool ok = c < nchunk;  // a group's TEAM lanes are all in range or all out
        const int b = ok ? c / cpr : 0, k = ok ? (c - b * cpr) * 8 : 0;
        const uint32_t xw[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
        const uint32_t ww[4] = {rw[u].x, rw[u].y, rw[u].z, rw[u].w};
        float v[8];
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float x = bf2f((uint16_t)(xw[e >> 1] >> (16 * (e & 1))));
          if (p.rms_w && ok) x = bf2f(f2bf(rms_apply(x, bf2f((uint16_t)(ww[e >> 1] >> (16 * (e & 1)))), rcs[b])));
          v[e] = x;
          mx = fmaxf(mx, fabsf(x));
        }
#pragma unroll
        for (int o = 1; o < TEAM; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(~0u, mx, o));
        if (!ok) continue;
        float sc, inv;
        bfp_scale(mx, sc, inv);
        // X = rn(v * 2^(30-e)); Y = (X + 0x808080) ^ 0x808080 has the balanced base-256
        // digits d0..d3 of X as its four bytes
        uint32_t Y[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) Y[e] = (uint32_t)(__float2int_rn(v[e] * sc * 32768.0f) + 0x808080) ^ 0x808080u;
        uint8_t* blk = xb + (size_t)((k >> 5) * NM + (b >> 1)) * XBS;
#pragma unroll
        for (int qd = 0; qd < 2; ++qd) {  // 4 values -> one word per digit (4x4 byte transpose)
          const uint32_t t0 = __byte_perm(Y[4 * qd], Y[4 * qd + 1], 0x5140);
          const uint32_t t1 = __byte_perm(Y[4 * qd], Y[4 * qd + 1], 0x7362);
          const uint32_t t2 = __byte_perm(Y[4 * qd + 2], Y[4 * qd + 3], 0x5140);
          const uint32_t t3 = __byte_perm(Y[4 * qd + 2], Y[4 * qd + 3], 0x7362);
          const uint32_t wd[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632),
                                  __byte_perm(t1, t3, 0x5410), __byte_perm(t1, t3, 0x7632)};
          // B fragment: column n = (b & 1) * 4 + digit, lane n * 4 + (kk & 15) / 4, register kk / 16
          const int kk = (k & 31) + 4 * qd;
#pragma unroll
          for (int d = 0; d < 4; ++d)
            *(uint32_t*)(blk + ((((b & 1) * 4 + d) * 4 + ((kk & 15) >> 2)) * 8 + (kk >> 4) * 4)) = wd[d];
        }
        if (k % G == 0) xsd[(k / G) * NBP + b] = (double)inv * (1.0 / 32768.0);
      }
    }
    for (int i = tid; i < KG * (NBP - p.nb); i += NT) xsd[(i / (NBP - p.nb)) * NBP + p.nb + i % (NBP - p.nb)] = 0.0;
  }
  csync();

  auto epi = [&](int row, int b, double s0, double s1) {
    uint16_t* yo = p.y + (size_t)b * p.ld_y + row;
    if (PAIR) {
      *yo = f2bf(silu_tanh_bf16(rbf_d(s0)) * rbf_d(s1));
    } else if (p.epi == EPI_RESID) {
      *yo = f2bf(bf2f(p.res[(size_t)b * p.ld_y + row]) + rbf_d(s0));
    } else if (p.epi == EPI_F32) {
      ((float*)p.y)[(size_t)b * p.ld_y + row] = (float)s0;
    } else {
      *yo = f2bf((float)s0);
    }
  };

  // ---- work items: (tile, piece, column range); warp w takes items w, w + 8, ... ----
  const uint32_t xm = p.xor_mask;
  const int bl = (lane >> 1) & 1;  // batch row of this lane within an MMA's column pair
  const uint32_t a_lane = (uint32_t)(((lane & 7) + ((lane >> 3) & 1) * 8) * pl.rbp + (lane >> 4) * 16);
  const int nitem = nu * pl.nq;
  for (int i = wid; i < nitem; i += NWARP) {
    const int j = i / pl.nq, qq = i - j * pl.nq;
    const int s = j % pl.nslot;
    {
      int ok = 1;
      if (lane == 0) {
        const unsigned long long t0 = gtimer();
        for (unsigned it = 0; *issued_ <= j; ++it) {
          __nanosleep(32);
          if ((it & 15) == 15 && (*abort_ || gtimer() - t0 > TIMEOUT_NS)) {
            *abort_ = 1;
            ok = 0;
            break;
          }
        }
        if (ok) ok = wait_phase(&full[s], (uint32_t)((j / pl.nslot) & 1), abort_);
      }
      if (!__shfl_sync(~0u, ok, 0)) break;
      mbar_test(&full[s], (uint32_t)((j / pl.nslot) & 1));  // every lane observes the completed phase
    }
    const int t = j / pl.nc, c = j - t * pl.nc;
    const int row0 = r0 + t * TR;
    const int k0 = c * pl.segc, len = min(pl.segc, K - k0);
    const int kq = qq * pl.cseg, qlen = max(0, min(pl.cseg, len - kq));
    const uint8_t* slot = ring + (size_t)s * pl.slot;
    const uint32_t a_base = sa(slot) + a_lane + kq;
    const uint8_t* scb = slot + (size_t)(lane >> 2) * pl.rbp + len;  // this lane's scale row
    const int WOFS = TR * pl.rbp;
    double acc[NW][NM][2];
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int m = 0; m < NM; ++m) acc[w][m][0] = acc[w][m][1] = 0.0;
    const int nkb = qlen >> 5, kb0 = (k0 + kq) >> 5;
#pragma unroll 2
    for (int kb = 0; kb < nkb; ++kb) {
      const int gl = (kq + kb * 32) / G, gg = ((kb0 + kb) * 32) / G;
      uint32_t a[NW][4];
      double s0[NW], s1[NW];
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        ldsm_x4(a[w], a_base + w * WOFS + kb * 32);
        if (xm) {
#pragma unroll
          for (int e = 0; e < 4; ++e) a[w][e] ^= xm;
        }
        s0[w] = (double)bf2f(((const uint16_t*)(scb + w * WOFS))[gl]);
        s1[w] = (double)bf2f(((const uint16_t*)(scb + w * WOFS + 8 * pl.rbp))[gl]);
      }
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const uint2 bv = *(const uint2*)(xb + (size_t)((kb0 + kb) * NM + m) * XBS + lane * 8);
        const double xs = xsd[gg * NBP + 2 * m + bl];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          int cc[4];
          mma_s8(cc, a[w], bv);
          acc[w][m][0] = fma((double)(cc[0] + 256 * cc[1]), s0[w] * xs, acc[w][m][0]);
          acc[w][m][1] = fma((double)(cc[2] + 256 * cc[3]), s1[w] * xs, acc[w][m][1]);
        }
      }
    }
    // odd lanes hold the pieces weighted 2^16; after the pair sum even lanes hold
    // rows (lane / 4) and (lane / 4 + 8) of batch row 2m + bl
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          double v = acc[w][m][h];
          if (lane & 1) v *= 65536.0;
          acc[w][m][h] = v + __shfl_xor_sync(~0u, v, 1);
        }
    if (NS == 1) {
      __syncwarp();
      if (lane == 0) {
        fence_proxy_async();
        mbar_arrive(&empty[s]);
      }
      if (!(lane & 1)) {
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = row0 + (lane >> 2) + 8 * h, b = 2 * m + bl;
            if (row < r1 && b < p.nb) epi(row, b, acc[0][m][h], PAIR ? acc[NW - 1][m][h] : 0.0);
          }
      }
      continue;
    }
    // partial sums of this item; the tile's last item to finish adds them in column order
    double* pt0 = part + (size_t)(t % pl.pt) * NS * (NW * TR * NBP);
    if (!(lane & 1)) {
      double* pp = pt0 + (size_t)(c * pl.nq + qq) * (NW * TR * NBP);
#pragma unroll
      for (int w = 0; w < NW; ++w)
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) pp[(w * TR + (lane >> 2) + 8 * h) * NBP + 2 * m + bl] = acc[w][m][h];
    }
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&tcnt[t % pl.pt], 1) == NS - 1;
    }
    if (__shfl_sync(~0u, last, 0)) {
      __threadfence_block();
      if (lane == 0) tcnt[t % pl.pt] = 0;
      for (int e = lane; e < TR * NBP; e += 32) {
        const int rl = e / NBP, b = e - rl * NBP;
        double a0 = 0.0, a1 = 0.0;
        for (int q2 = 0; q2 < NS; ++q2) {
          const double* pq = pt0 + (size_t)q2 * (NW * TR * NBP);
          a0 += pq[rl * NBP + b];
          if (PAIR) a1 += pq[(TR + rl) * NBP + b];
        }
        const int row = row0 + rl;
        if (row < r1 && b < p.nb) epi(row, b, a0, a1);
      }
    }
    __syncwarp();
    if (lane == 0) {  // released only now, after any combine: partial slots are reused by later tiles
      fence_proxy_async();
      mbar_arrive(&empty[s]);
    }
  }
}

}  // namespace gmma

// 0: launched (or a launch error < 0); 1: shape not handled here; 2: the activation
// staging of this batch does not fit (fewer batch rows per launch would).
template <int G, int NM, bool PAIR>
static int mma_launch(const GemvW8Params& p, cudaStream_t st) {
  using namespace gmma;
  const int K = p.K, NW = PAIR ? 2 : 1;
  const size_t fixed = stage_bytes(K, G, NM);
  if (fixed > STAGE_MAX) return 2;
  const int grid = iron_num_sms() < p.M ? iron_num_sms() : p.M;
  const int rows = (p.M + grid - 1) / grid, ntile = (rows + TR - 1) / TR;
  auto stride = [](int bytes) {  // 16-byte multiple, 16 mod 128: conflict-free ldmatrix rows
    int r = (bytes + 15) / 16 * 16;
    return r + (int)((144 - r % 128) % 128);
  };
  // One plan per candidate length of the copied row pieces (whole rows first); the
  // first that keeps >= 120 KB of weight in flight wins, else the one with the most.
  auto make = [&](int segc, Plan& pl) {
    pl.segc = segc;
    pl.nc = (K + segc - 1) / segc;
    pl.rbp = stride(segc + 2 * (segc / G));
    pl.slot = TR * pl.rbp * NW;
    // the longest work item that still gives the eight consumer warps two items each
    for (int cand : {1024, 512, 256}) {
      if (cand % G) continue;
      pl.cseg = cand < segc ? cand : segc;
      pl.nq = (segc + pl.cseg - 1) / pl.cseg;
      if ((long long)ntile * pl.nc * pl.nq >= 2 * NWARP) break;
    }
    const int NS = pl.nc * pl.nq;
    pl.off_ring = (int)((fixed + 127) & ~(size_t)127);
    for (pl.nslot = NSLOT_MAX; pl.nslot >= 2; --pl.nslot) {
      // a tile's partial sums are reused by the tile pt later, whose first copy needs
      // all of the older tile's slots released
      pl.pt = NS > 1 ? (pl.nslot + pl.nc - 1 + pl.nc - 1) / pl.nc + 1 : 0;
      pl.off_part = pl.off_ring + pl.nslot * pl.slot;
      pl.off_cnt = pl.off_part + pl.pt * NS * NW * TR * 2 * NM * 8;
      pl.off_bar = (pl.off_cnt + pl.pt * 4 + 7) & ~7;
      if ((size_t)pl.off_bar + 2 * pl.nslot * 8 <= (size_t)SMEM_MAX) return true;
    }
    return false;
  };
  Plan pl{};
  long long best = 0;
  for (int segc : {K, 4096, 2048, 1024, 512}) {
    if (segc > K || (segc != K && segc % (8 * G))) continue;
    Plan c{};
    if (!make(segc, c)) continue;
    const long long inflight = (long long)c.nslot * c.slot;
    if (inflight > best) {
      best = inflight;
      pl = c;
    }
    if (inflight >= 120 * 1024) break;
  }
  if (best == 0) return 2;
  const size_t total = (size_t)pl.off_bar + 2 * pl.nslot * 8;
  auto fn = gemv_mma_kernel<G, NM, PAIR>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
    attr[dev] = true;
  }
  fn<<<grid, NT + 32, total, st>>>(p, pl);
  return iron_check_launch("gemv_mma_kernel");
}

template <int G, bool PAIR>
static int mma_launch_nb(const GemvW8Params& p, cudaStream_t st) {
  if (p.nb <= 2) return mma_launch<G, 1, PAIR>(p, st);
  if (p.nb <= 4) return mma_launch<G, 2, PAIR>(p, st);
  return mma_launch<G, 4, PAIR>(p, st);
}

template <int G>
static int mma_launch_g(const GemvW8Params& p, bool pair, cudaStream_t st) {
  if (p.K % (8 * G) || gmma::stage_bytes(p.K, G, 1) > gmma::STAGE_MAX) return 1;
  const int rc = pair ? mma_launch_nb<G, true>(p, st) : mma_launch_nb<G, false>(p, st);
  if (rc != 2) return rc;
  if (p.nb == 1) return 1;
  // the staging of this many batch rows does not fit: two launches over halves
  const int n0 = (p.nb + 1) / 2;
  const int a = mma_launch_g<G>(gemv_rows(p, 0, n0), pair, st);
  if (a) return a;
  return mma_launch_g<G>(gemv_rows(p, n0, p.nb - n0), pair, st);
}

// 0: launched (or a launch error code < 0); 1: not a shape for this kernel
int gemv_mma_launch(const GemvW8Params& p, bool pair, cudaStream_t st) {
  if (!p.wa.plain1 || (pair && !p.wb.plain1) || p.nb < 1 || p.nb > 8) return 1;
  // the prologue reads activations (and RMS weights) as 16-byte vectors
  if (!iron_aligned(p.x, 16) || p.ld_x % 8 || (p.rms_w && !iron_aligned(p.rms_w, 16))) return 1;
  switch (p.wa.G) {
    case 32: return mma_launch_g<32>(p, pair, st);
    case 64: return mma_launch_g<64>(p, pair, st);
    case 128: return mma_launch_g<128>(p, pair, st);
  }
  return 1;
}

}  // namespace iron
