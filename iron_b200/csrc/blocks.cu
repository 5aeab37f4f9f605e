// Fused-operator entry points built from the GEMV family: the QKV head, the
// SwiGLU MLP block and the int8 lm_head with argmax.
#include "common.cuh"
#include "gemv_w8.cuh"

namespace iron {
int qk_norm_rope_kv_launch(const uint16_t* raw, const uint16_t* n_qn, const uint16_t* n_kn,
                           const uint16_t* ang, int ang_is_table, uint16_t* q_out, uint16_t* kv,
                           int HD, int Hq, int Hkv, int max_seq, int batch, int kv_off,
                           const int32_t* kv_off_dev, float eps, int norm_mode, cudaStream_t st, int pos0);
}
using namespace iron;

extern "C" int iron_qkv_head(const uint16_t* cur, const uint16_t* n_in, const void* wqkv_wire, int group,
                             int tile_m, int domain, const uint16_t* n_qn, const uint16_t* n_kn,
                             const uint16_t* ang, int ang_is_table, uint16_t* q_out, uint16_t* kv_cache,
                             int D, int HD, int Hq, int Hkv, int max_seq, int batch, int kv_off,
                             const int32_t* kv_off_dev, float eps, int norm_mode, uint16_t* raw_ws,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  IRON_REQUIRE(cur && n_in && n_qn && n_kn && ang && q_out && kv_cache && raw_ws, IRON_ERR_ARG,
               "qkv_head: null pointer");
  IRON_REQUIRE(kv_off_dev || (kv_off >= 0 && kv_off % (2 * HD) == 0 && kv_off / (2 * HD) < max_seq),
               IRON_ERR_ARG, "qkv_head: kv_off %d is not a token slot of a %d-token cache", kv_off, max_seq);
  const int M = (Hq + 2 * Hkv) * HD;
  GemvW8Params p = {};
  int rc = make_wire(p.wa, wqkv_wire, M, D, group, tile_m, 0, 0, domain);
  if (rc) return rc;
  p.wb = p.wa;
  p.M = M;
  p.K = D;
  p.x = cur;
  p.ld_x = D;
  p.rms_w = n_in;
  p.eps = eps;
  p.rms_mode = norm_mode;
  p.y = raw_ws;
  p.ld_y = M;
  p.nb = batch;
  p.epi = EPI_STORE;
  p.tc_ws = workspace;
  p.tc_ws_bytes = workspace_bytes;
  cudaStream_t st = (cudaStream_t)stream;
  rc = gemv_w8_launch(p, false, st);
  if (rc) return rc;
  return qk_norm_rope_kv_launch(raw_ws, n_qn, n_kn, ang, ang_is_table, q_out, kv_cache, HD, Hq, Hkv,
                                max_seq, batch, kv_off, kv_off_dev, eps, norm_mode, st, -1);
}

extern "C" int iron_mlp_block(const uint16_t* cur, const uint16_t* a_or_cx, int fuse_o, const uint16_t* n_pf,
                              const void* wo, int wo_tile_m, int wo_rows_per_core, int wo_tiles_per_core,
                              const void* wg, const void* wu, int gu_tile_m, const void* wd, int d_tile_m,
                              int group, int domain, uint16_t* x1_ws, uint16_t* gh_ws, uint16_t* nxt, int D,
                              int FF, int QD, int batch, float eps, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  IRON_REQUIRE(cur && a_or_cx && n_pf && wg && wu && wd && x1_ws && gh_ws && nxt, IRON_ERR_ARG,
               "mlp_block: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  // x1 = bf16(cur + a) with a = bf16(Wo @ cx) under fuse_o
  if (fuse_o) {
    IRON_REQUIRE(wo && QD > 0, IRON_ERR_ARG, "mlp_block: fuse_o needs Wo and QD");
    GemvW8Params p = {};
    rc = make_wire(p.wa, wo, D, QD, group, wo_tile_m, wo_rows_per_core, wo_tiles_per_core, domain);
    if (rc) return rc;
    p.wb = p.wa;
    p.M = D;
    p.K = QD;
    p.x = a_or_cx;
    p.ld_x = QD;
    p.res = cur;
    p.y = x1_ws;
    p.ld_y = D;
    p.nb = batch;
    p.epi = EPI_RESID;
    p.tc_ws = workspace;
    p.tc_ws_bytes = workspace_bytes;
    rc = gemv_w8_launch(p, false, st);
  } else {
    rc = iron_add(cur, a_or_cx, x1_ws, (int64_t)batch * D, stream);
  }
  if (rc) return rc;
  // gh = bf16(silu_tanh(bf16(Wg @ hf)) * bf16(Wu @ hf)), hf = RMSNorm_w(x1, n_pf)
  {
    GemvW8Params p = {};
    rc = make_wire(p.wa, wg, FF, D, group, gu_tile_m, 0, 0, domain);
    if (rc) return rc;
    rc = make_wire(p.wb, wu, FF, D, group, gu_tile_m, 0, 0, domain);
    if (rc) return rc;
    p.M = FF;
    p.K = D;
    p.x = x1_ws;
    p.ld_x = D;
    p.rms_w = n_pf;
    p.eps = eps;
    p.y = gh_ws;
    p.ld_y = FF;
    p.nb = batch;
    p.epi = EPI_STORE;
    p.xor_mask = p.wa.xor_mask;
    p.tc_ws = workspace;
    p.tc_ws_bytes = workspace_bytes;
    rc = gemv_w8_launch(p, true, st);
    if (rc) return rc;
  }
  // nxt = bf16(x1 + bf16(Wd @ gh))
  {
    GemvW8Params p = {};
    rc = make_wire(p.wa, wd, D, FF, group, d_tile_m, 0, 0, domain);
    if (rc) return rc;
    p.wb = p.wa;
    p.M = D;
    p.K = FF;
    p.x = gh_ws;
    p.ld_x = FF;
    p.res = x1_ws;
    p.y = nxt;
    p.ld_y = D;
    p.nb = batch;
    p.epi = EPI_RESID;
    p.tc_ws = workspace;
    p.tc_ws_bytes = workspace_bytes;
    return gemv_w8_launch(p, false, st);
  }
}

extern "C" int iron_lm_head_w8_argmax(const void* wire, int M, int K, int group, const uint16_t* x, int batch,
                                      uint16_t* logits, int32_t* token_out, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  IRON_REQUIRE(logits != nullptr, IRON_ERR_ARG, "lm_head_w8_argmax: logits buffer required");
  IRON_REQUIRE(workspace && workspace_bytes >= iron_argmax_workspace_bytes(batch), IRON_ERR_ARG,
               "lm_head_w8_argmax: workspace below iron_lm_head_workspace_bytes");
  // batch 16+ with iron_lm_head_workspace_bytes: [tensor-core scratch | argmax
  // candidates]; otherwise the candidates from offset 0 and launches of 8 rows
  const bool tc = batch >= 16 && workspace_bytes >= iron_lm_head_workspace_bytes(M, K, batch);
  const int64_t tcb = tc ? iron_tc_workspace_bytes(M, K, batch) : 0;
  int rc = iron_gemv_w8a16(wire, M, K, group, 1, 0, 0, 0, x, batch, nullptr, logits, tc ? workspace : nullptr,
                           tcb, stream);
  if (rc) return rc;
  return iron_argmax_bf16(logits, M, batch, token_out, (uint8_t*)workspace + tcb, stream);
}
