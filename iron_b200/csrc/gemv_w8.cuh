// int8 weight-wire descriptor and the W8A16 GEMV launch interface.
#pragma once
#include "common.cuh"

namespace iron {

// Row addressing of IRON's int8 tile wire (see include/iron_b200.h).
struct Wire {
  const uint8_t* base;
  int K, G;
  int tile_m, rows_per_core, tiles_per_core;
  long long tile_bytes;
  uint32_t xor_mask;  // 0x80808080 for the biased (q+128) payload domain
  int plain1;         // tile_m == 1 and a single window: row r at r * tile_bytes
};

__device__ __forceinline__ void wire_row(const Wire& w, int r, const uint8_t*& pw,
                                         const uint16_t*& ps) {
  if (w.plain1) {
    const uint8_t* t = w.base + (long long)r * w.tile_bytes;
    pw = t;
    ps = (const uint16_t*)(t + w.K);
  } else {
    const int core = r / w.rows_per_core;
    const int j = r - core * w.rows_per_core;
    const int t = j / w.tile_m;
    const int rr = j - t * w.tile_m;
    const uint8_t* tb = w.base + (long long)(core * w.tiles_per_core + t) * w.tile_bytes;
    pw = tb + (long long)rr * w.K;
    ps = (const uint16_t*)(tb + (long long)w.tile_m * w.K) + rr * (w.K / w.G);
  }
}

enum { EPI_STORE = 0, EPI_RESID = 1, EPI_F32 = 2 };

struct GemvW8Params {
  Wire wa, wb;          // wb: second wire of a gate/up pair
  int M, K;             // output rows (pairs in pair mode), reduction length
  const uint16_t* x;    // [nb][ld_x] bf16 activations
  int ld_x;
  const uint16_t* rms_w;  // non-null: RMS-normalise x with this weight first
  float eps;
  int rms_mode;           // 0 kernel form, 1 golden form (see RmsCoef)
  const uint16_t* res;  // residual [nb][ld_y]
  uint16_t* y;          // [nb][ld_y]
  int ld_y;
  int nb;               // batch rows (1..8)
  int epi;
  int ksplit;           // warps sharing one row group along K (set by the launcher)
  uint32_t xor_mask;
  void* tc_ws;          // scratch of the tensor-core path (batch >= 16), or null
  int64_t tc_ws_bytes;
};

// The same call restricted to batch rows [b0, b0 + n).
inline GemvW8Params gemv_rows(GemvW8Params p, int b0, int n) {
  p.nb = n;
  p.x += (size_t)b0 * p.ld_x;
  if (p.res) p.res += (size_t)b0 * p.ld_y;
  p.y = p.epi == EPI_F32 ? (uint16_t*)((float*)p.y + (size_t)b0 * p.ld_y) : p.y + (size_t)b0 * p.ld_y;
  return p;
}

int make_wire(Wire& w, const void* base, int M, int K, int group, int tile_m, int rows_per_core,
              int tiles_per_core, int domain);
// pair: rows of wa (gate) and wb (up) combined as bf16(silu_tanh(g) * u)
int gemv_w8_launch(GemvW8Params p, bool pair, cudaStream_t st);

}  // namespace iron
