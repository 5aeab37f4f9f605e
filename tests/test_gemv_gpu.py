"""GPU parity of the int8 group-dequant GEMV, the bf16 GEMV and the lm_head argmax.

Oracle: ``oracle.ops`` (the premul golden of gemv_int8/reference.py:25-40, the
exact dequantised sum, and the bf16 golden of gemv/reference.py:9-11).
"""

import numpy as np
import pytest
import torch

from iron_b200 import _lib
from iron_b200.operators import GEMV, GEMVInt8
from iron_b200.qwen3 import quantize_to_wire, wire_to_numpy
from iron_b200.test_utils import verify_buffer
from oracle import ops
from oracle.bf16 import from_bits, rnd

from helpers import assert_close, assert_ulps, assert_w8_exact, dev_bf16, dev_u8, host

pytestmark = pytest.mark.gpu


def _run_w8(wire_u8, M, K, group, tile_m, domain, x, batch=1, residual=None, rpc=0, tpc=0):
    y = torch.empty(batch, M, dtype=torch.bfloat16, device="cuda")
    tw = _lib.tc_workspace([(M, K)], batch, "cuda")
    _lib.call("iron_gemv_w8a16", wire_u8.data_ptr(), M, K, group, tile_m, rpc, tpc, domain,
              x.data_ptr(), batch, None if residual is None else residual.data_ptr(), y.data_ptr(),
              tw.data_ptr(), tw.numel(), _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.lib().iron_tc_status(tw.data_ptr(), 0) == 0
    return host(y)


@pytest.mark.parametrize("domain,tile_m,cols", [("biased", 2, 1), ("signed", 4, 2), ("signed", 1, 1)])
def test_gemvint8_op_against_reference_golden(golden, domain, tile_m, cols):
    """The reference's own golden (M=256, K=1024, group 128) through the GEMVInt8 op."""
    g = golden("gemv_int8")
    wire = ops.pack_tile_wire(g["w_int8"], g["scales"], tile_m, cols, domain)
    op = GEMVInt8(M=256, K=1024, tile_size_input=tile_m,
                  kernel_source="mv_int8_signed.cc" if domain == "signed" else None)
    assert wire.size // 2 == op.get_arg_spec()[0].shape[0]
    call = op.get_callable()
    y = torch.empty(256, dtype=torch.bfloat16, device="cuda")
    call(dev_u8(wire).view(torch.bfloat16), dev_bf16(g["x"]), y)
    torch.cuda.synchronize()
    out = host(y)
    _check_against_premul_golden(out, g["w_int8"], g["scales"], from_bits(g["x"]), from_bits(g["y"]))
    # and the exact dequantised sum (GEMVInt8.reference, op.py:173-178) to its error bound
    assert_w8_exact(out, g["w_int8"], g["scales"], from_bits(g["x"]), "vs exact")


def _premul_bound(q, s_bits, x):
    """max |premul golden - exact sum| = sum_i |q_i x_i s| 2^-9 (one bf16 rounding of x*s)."""
    G = q.shape[1] // s_bits.shape[1]
    se = np.repeat(from_bits(s_bits), G, axis=1).astype(np.float64)
    w = np.abs(q.astype(np.float64)) * se
    return (np.abs(np.atleast_2d(np.asarray(x, np.float64))) @ w.T * 2.0 ** -9).reshape(
        (-1,) if np.asarray(x).ndim == 1 else (np.asarray(x).shape[0], -1))


def _check_against_premul_golden(out, q, s_bits, x, golden_y):
    """The kernel computes the exact dequantised sum; the reference golden
    (gemv_int8/reference.py:25-40) rounds bf16(x*s) first, which moves each output by at
    most sum_i |q_i x_i s| 2^-9.  Every element must lie within the reference test's
    tolerance (gemv_int8/test.py:76-77: rel 0.04, abs 1e-2) widened by that bound and one
    bf16 rounding of each side; at most 1% may miss the unwidened tolerance."""
    out = np.asarray(out, np.float64).reshape(-1)
    ref = np.asarray(golden_y, np.float64).reshape(-1)
    bound = _premul_bound(q, s_bits, x).reshape(-1)
    tol = np.maximum(1e-2, 0.04 * (np.abs(out) + np.abs(ref))) + bound + 2.0 ** -8 * (np.abs(out) + np.abs(ref))
    assert np.all(np.abs(out - ref) <= tol), np.max(np.abs(out - ref) / tol)
    assert not verify_buffer(out, "y", ref, rel_tol=0.04, abs_tol=1e-2, max_error_rate=0.01)


def test_gemvint8_group32_reference_golden(golden):
    g = golden("gemv_int8")
    wire = ops.pack_tile_wire(g["w_int8"], g["scales_g32"], 1, 1, "signed")
    out = _run_w8(dev_u8(wire), 256, 1024, 32, 1, 0, dev_bf16(g["x"]))
    _check_against_premul_golden(out[0], g["w_int8"], g["scales_g32"], from_bits(g["x"]), from_bits(g["y_g32"]))
    assert_w8_exact(out[0], g["w_int8"], g["scales_g32"], from_bits(g["x"]), "vs exact")


SHAPES = [(6144, 1024), (3072, 1024), (1024, 3072), (12288, 4096), (4096, 12288)]


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("batch", [1, 8, 32])
def test_gemv_w8_baseline_shapes(N, K, batch):
    """The operator sweep's shapes, group 32, masters N(0,0.02), x ~ N(0,1)."""
    torch.manual_seed(N + K + batch)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    wire = quantize_to_wire(w, 32)
    x = torch.randn(batch, K, device="cuda").to(torch.bfloat16)
    out = _run_w8(wire, N, K, 32, 1, 0, x, batch)
    q, s = wire_to_numpy(wire, N, K, 32)
    xh = host(x)
    if batch >= 16:  # the tcgen05 path: bf16-dequantised weights (tests/test_gemm_tc_gpu.py)
        mag = np.abs(xh).astype(np.float64) @ (np.abs(q) * np.repeat(from_bits(s), 32, axis=1)).T
        exact = ops.gemv_int8_exact(q, s, xh)
        assert np.all(np.abs(out - exact) <= 2.0 ** -8 * (np.abs(exact) + mag) + 1e-30)
    else:
        assert_w8_exact(out, q, s, xh, "vs exact")
    # vs the premul golden: the bf16 gate widened by that golden's own rounding bound
    premul = rnd(ops.gemv_int8_premul(q, s, xh))
    bound = _premul_bound(q, s, xh)
    err = np.abs(out - premul)
    lim = 1e-2 + 2e-2 * np.abs(premul) + bound + 2.0 ** -8 * np.abs(premul)
    assert np.all(err <= lim), np.max(err / lim)


@pytest.mark.parametrize("N,K,group,domain", [(6144, 1024, 32, 0), (1024, 3072, 32, 0), (12288, 4096, 32, 0),
                                               (4096, 12288, 32, 0), (40, 256, 32, 0), (1000, 3072, 64, 1),
                                               (300, 2048, 128, 0), (148 * 16 + 5, 768, 32, 1)])
def test_gemv_w8_batch_rows_match_single_rows(N, K, group, domain):
    """Every batch row of a batch-5 and a batch-8 call is bit-identical to the batch-1 call on
    that row: the activations are held at the same precision at every batch size and each
    output is accumulated in the same order.  Covers K split into segments, ragged row
    blocks, groups 64/128 and the biased payload domain."""
    torch.manual_seed(N * 7 + K)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    wire = quantize_to_wire(w, group, domain=domain)
    q, s = wire_to_numpy(quantize_to_wire(w, group, domain=0), N, K, group)  # the signed decode
    x = torch.randn(8, K, device="cuda").to(torch.bfloat16)
    singles = np.stack([_run_w8(wire, N, K, group, 1, domain, x[b:b + 1].contiguous(), 1)[0] for b in range(8)])
    assert_w8_exact(singles, q, s, host(x), "batch 1")
    for batch in (5, 8):
        out = _run_w8(wire, N, K, group, 1, domain, x[:batch].contiguous(), batch)
        assert np.array_equal(out, singles[:batch]), f"batch {batch} differs from single rows"


def test_gemv_w8_residual_and_biased():
    torch.manual_seed(3)
    M, K = 512, 2048
    w = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    wire_s = quantize_to_wire(w, 64, domain=0)
    wire_b = quantize_to_wire(w, 64, domain=1)
    x = torch.randn(1, K, device="cuda").to(torch.bfloat16)
    r = torch.randn(1, M, device="cuda").to(torch.bfloat16)
    ys = _run_w8(wire_s, M, K, 64, 1, 0, x, 1, r)
    yb = _run_w8(wire_b, M, K, 64, 1, 1, x, 1, r)
    assert np.array_equal(ys, yb)  # both payload domains decode the same integer q
    q, s = wire_to_numpy(wire_s, M, K, 64)
    want = rnd(host(r)[0] + rnd(ops.gemv_int8_exact(q, s, host(x)[0])))
    assert_close(ys[0], want, what="residual")


def test_dequant_and_quantizer_bit_exact(golden):
    """GPU RTN quantiser == Qwen3NPU._set_int8_rtn wire; GPU dequant == q*s exactly."""
    g = golden("rtn_pack")
    w = dev_bf16(g["w"]).reshape(64, 256)
    wire = torch.empty(64 * (256 + 4), dtype=torch.uint8, device="cuda")
    _lib.call("iron_quantize_rtn", w.data_ptr(), 64, 256, 128, 4, 0, wire.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(wire.cpu().numpy().view(np.uint16), g["wire_signed_t4"])
    out = torch.empty(64, 256, dtype=torch.float32, device="cuda")
    _lib.call("iron_dequant_w8", wire.data_ptr(), 64, 256, 128, 4, 0, 0, 0, out.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    q, s = ops.quantize_rtn(from_bits(g["w"]).reshape(64, 256), 128)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ops.dequant_f32(q, s).view(np.uint32))


def test_quantizer_group32_matches_oracle():
    torch.manual_seed(5)
    w = (torch.randn(96, 512, device="cuda") * 0.02).to(torch.bfloat16)
    w[3, :32] = 0
    wire = quantize_to_wire(w, 32)
    q, s = wire_to_numpy(wire, 96, 512, 32)
    q2, s2 = ops.quantize_rtn(host(w), 32)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)


def test_bf16_gemv_against_reference_golden(golden):
    g = golden("gemv_bf16")
    op = GEMV(M=256, K=512)
    y = torch.empty(256, dtype=torch.bfloat16, device="cuda")
    op.get_callable()(dev_bf16(g["A"]).reshape(256, 512), dev_bf16(g["B"]), y)
    torch.cuda.synchronize()
    assert_ulps(host(y), from_bits(g["C"]), max_ulp=1, frac_exact=0.95, what="gemv bf16")


def test_bf16_gemv_independent_batches():
    torch.manual_seed(9)
    A = torch.randn(3, 128, 256, device="cuda").to(torch.bfloat16)
    x = torch.randn(3, 256, device="cuda").to(torch.bfloat16)
    y = torch.empty(3, 128, dtype=torch.bfloat16, device="cuda")
    GEMV(M=128, K=256, num_batches=3).get_callable()(A, x, y)
    torch.cuda.synchronize()
    for b in range(3):
        assert_ulps(host(y[b]), ops.gemv_bf16(host(A[b]), host(x[b])), max_ulp=1, what=f"batch {b}")


@pytest.mark.parametrize("batch", [1, 3, 11, 16, 40])
def test_lm_head_bf16_argmax(batch):
    """Fused lm_head + argmax over the Qwen3 vocabulary; ties resolve to the lowest index."""
    torch.manual_seed(11)
    V, D = 151936, 1024
    E = (torch.randn(V, D, device="cuda") * 0.02).to(torch.bfloat16)
    E[1234] = E[777]  # an exact tie in the logits
    x = torch.randn(batch, D, device="cuda").to(torch.bfloat16)
    x[0] = E[777].float() * 40
    logits = torch.empty(batch, V, dtype=torch.bfloat16, device="cuda")
    tok = torch.empty(batch, dtype=torch.int32, device="cuda")
    ws = _lib.tc_workspace([(V, D)], batch, "cuda", lm_head=True)
    _lib.call("iron_lm_head_bf16_argmax", E.data_ptr(), V, D, x.data_ptr(), batch, logits.data_ptr(),
              tok.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
    torch.cuda.synchronize()
    lg = host(logits)
    for b in range(batch):
        assert int(tok[b]) == int(np.argmax(lg[b]))
    assert int(tok[0]) == 777
    want = ops.gemv_bf16(host(E)[:4096], host(x)[0])
    assert_ulps(lg[0][:4096], want, max_ulp=1, frac_exact=0.95, what="logits")
    if batch >= 16:
        # the tensor-core path with no logits buffer (kept in the workspace) gives the same tokens
        tok2 = torch.empty(batch, dtype=torch.int32, device="cuda")
        _lib.call("iron_lm_head_bf16_argmax", E.data_ptr(), V, D, x.data_ptr(), batch, None, tok2.data_ptr(),
                  ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        torch.cuda.synchronize()
        assert torch.equal(tok, tok2)
        assert _lib.lib().iron_tc_status(ws.data_ptr(), 0) == 0
        # a workspace of the argmax candidates only: the launches of 8 rows, same tokens
        small = _lib.workspace(_lib.lib().iron_argmax_workspace_bytes(batch), "cuda")
        tok3 = torch.empty(batch, dtype=torch.int32, device="cuda")
        _lib.call("iron_lm_head_bf16_argmax", E.data_ptr(), V, D, x.data_ptr(), batch, None, tok3.data_ptr(),
                  small.data_ptr(), small.numel(), _lib.stream_ptr())
        torch.cuda.synchronize()
        near = sum(int(tok3[b]) != int(tok[b]) and lg[b][int(tok3[b])] == lg[b][int(tok[b])] for b in range(batch))
        assert sum(int(tok3[b]) != int(tok[b]) for b in range(batch)) == near


def test_bf16_gemv_shared_weight_batch32_tensor_cores():
    torch.manual_seed(12)
    M, K, B = 4096, 1024, 32
    A = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(B, M, dtype=torch.bfloat16, device="cuda")
    tw = _lib.tc_workspace([(M, K)], B, "cuda")
    _lib.call("iron_gemv_bf16", A.data_ptr(), M, K, x.data_ptr(), B, 0, y.data_ptr(), tw.data_ptr(), tw.numel(),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.lib().iron_tc_status(tw.data_ptr(), 0) == 0
    for b in (0, 13, 31):
        assert_ulps(host(y[b]), ops.gemv_bf16(host(A), host(x[b])), max_ulp=1, frac_exact=0.95, what=f"row {b}")
