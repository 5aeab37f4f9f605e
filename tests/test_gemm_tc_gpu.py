"""Batch >= 16 int8 projections on the tcgen05 tensor cores (csrc/gemm_tc.cu).

The kernel writes each dequantised weight q*s (exact in float32) as a bf16 hi plane
and a bf16 lo plane and multiplies both, so every product is exact and only the
float32 summation order differs from the exact dequantised sum
(oracle.ops.gemv_int8_exact).  Checked (a) tightly against that sum: one bf16 output
rounding plus float32 summation error, and (b) against the decode path's bf16 gate
(rtol 2e-2, atol 1e-2).  Shapes cover split K, ragged row tiles, groups 64/128 (a
split may start inside a group), the biased payload domain, the residual / float32 /
gate-up + RMSNorm epilogues, and batches 16..1024 (above 128 rows a launch runs row
blocks of equal size, up to 128 rows each, as a second grid dimension)."""

import numpy as np
import pytest
import torch

from iron_b200 import _lib
from iron_b200.qwen3 import quantize_to_wire, wire_to_numpy
from oracle import ops
from oracle.bf16 import from_bits, rnd

from helpers import assert_close, host

pytestmark = pytest.mark.gpu


def _deq(q, s_bits, G):
    return (q.astype(np.float64) * np.repeat(from_bits(s_bits), G, axis=1).astype(np.float64))


def _check(out, q, s_bits, x, G, what):
    x = np.asarray(x, np.float64)
    exact = ops.gemv_int8_exact(q, s_bits, x)
    mag = np.abs(x) @ np.abs(_deq(q, s_bits, G)).T
    lim = 2.0 ** -8 * np.abs(exact) + 1e-5 * mag + 1e-30
    err = np.abs(np.asarray(out, np.float64) - exact)
    assert np.all(err <= lim), f"{what}: vs the exact sum, worst {np.max(err / lim):.3g}"
    # the decode path's bf16 gate against the exact dequantised sum
    assert_close(np.asarray(out, np.float64), exact, what=f"{what}: bf16 gate vs exact")


def _gemv(wire, M, K, G, domain, x, residual=None, ws="new", stream=None, sync=True):
    """One projection; ws: a workspace tensor, "new" (a fresh one) or None (no workspace:
    the exact launches of 8 rows)."""
    B = x.shape[0]
    if isinstance(ws, str):
        ws = _lib.tc_workspace([(M, K)], B, "cuda")
    y = torch.empty(B, M, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_gemv_w8a16", wire.data_ptr(), M, K, G, 1, 0, 0, domain, x.data_ptr(), B,
              None if residual is None else residual.data_ptr(), y.data_ptr(),
              None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _lib.stream_ptr(stream))
    if sync:
        torch.cuda.synchronize()
        if ws is not None:
            assert _lib.lib().iron_tc_status(ws.data_ptr(), 0) == 0
    return y


@pytest.mark.parametrize("M,K,G,B,domain", [(6144, 1024, 32, 32, 0), (12288, 4096, 32, 32, 0),
                                            (4096, 12288, 32, 16, 0), (1000, 3072, 64, 20, 1),
                                            (300, 2048, 128, 64, 0), (3072, 1024, 32, 256, 0),
                                            (1024, 3072, 32, 33, 0), (4096, 1024, 32, 1024, 0),
                                            (1024, 3072, 32, 300, 0), (1000, 2048, 64, 600, 1)])
def test_tc_projection_matches_dequantised_reference(M, K, G, B, domain):
    torch.manual_seed(M + K + B)
    w = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    wire = quantize_to_wire(w, G, domain=domain)
    q, s = wire_to_numpy(quantize_to_wire(w, G, domain=0), M, K, G)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    ws = _lib.tc_workspace([(M, K)], B, "cuda")
    y1 = _gemv(wire, M, K, G, domain, x, ws=ws)
    # the last split of each (row block, 128-row tile) puts its arrival counter back to
    # zero, so the workspace is ready for the next launch with nothing to clear
    blocks = max(1, -(-B // 128))
    assert int(ws[:256 + 4 * ((M + 127) // 128) * blocks].count_nonzero()) == 0
    y2 = _gemv(wire, M, K, G, domain, x, ws=ws)
    assert torch.equal(y1, y2), "not deterministic"
    _check(host(y1), q, s, host(x), G, f"{M}x{K} g{G} b{B}")


def test_tc_residual_f32_and_gate_up_rms_epilogues():
    torch.manual_seed(5)
    M, K, G, B = 3072, 1024, 32, 24
    wg = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    wu = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    qg, sg = wire_to_numpy(quantize_to_wire(wg, G), M, K, G)
    qu, su = wire_to_numpy(quantize_to_wire(wu, G), M, K, G)
    gw, uw = quantize_to_wire(wg, G), quantize_to_wire(wu, G)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    r = torch.randn(B, M, device="cuda").to(torch.bfloat16)
    st = _lib.stream_ptr()
    # residual: y = bf16(r + bf16(sum))
    y = _gemv(gw, M, K, G, 0, x, r)
    base = host(_gemv(gw, M, K, G, 0, x))
    want = rnd(host(r) + base)
    assert np.array_equal(host(y), want)
    # float32 partial sums (epilogue 2) round to the bf16 result
    y32 = torch.empty(B, M, dtype=torch.float32, device="cuda")
    tw = _lib.tc_workspace([(M, K)], B, "cuda")
    _lib.call("iron_gemv_w8a16_ex", gw.data_ptr(), None, M, K, G, 0, x.data_ptr(), K, B, None, 0.0, 0, None, 2,
              y32.data_ptr(), M, tw.data_ptr(), tw.numel(), st)
    torch.cuda.synchronize()
    assert np.array_equal(rnd(host(y32)), base)
    _check(host(y32), qg, sg, host(x), G, "f32 epilogue")
    # gate/up pair with the RMSNorm prologue: bf16(silu_tanh(bf16(Wg h)) * bf16(Wu h))
    nw = (1 + 0.1 * torch.randn(K, device="cuda")).to(torch.bfloat16)
    gh = torch.empty(B, M, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_gemv_w8a16_ex", gw.data_ptr(), uw.data_ptr(), M, K, G, 0, x.data_ptr(), K, B, nw.data_ptr(),
              1e-6, 0, None, 0, gh.data_ptr(), M, tw.data_ptr(), tw.numel(), st)
    torch.cuda.synchronize()
    assert _lib.lib().iron_tc_status(tw.data_ptr(), 0) == 0
    h = ops.rms_norm_f32(host(x), host(nw), 1e-6)
    g = rnd(h.astype(np.float64) @ _deq(qg, sg, G).T)
    u = rnd(h.astype(np.float64) @ _deq(qu, su, G).T)
    want = rnd(ops.silu_tanh_bf16(g) * u)
    got = host(gh)
    # one bf16 step of g or u (float32 summation order) moves an output by ~2 ulps
    err = np.abs(got - want)
    lim = 2.0 ** -6 * np.abs(want) + 1e-4
    assert np.mean(err <= lim) >= 0.999 and np.max(err) <= 0.05, f"pair: {np.mean(err <= lim):.4f}, max {err.max()}"


@pytest.mark.parametrize("B", [128, 200, 256, 520, 1024])
def test_tc_gate_up_pair_wide_batches(B):
    """A gate/up pair with the RMSNorm prologue at 128 rows (one pair launch) and above
    (gate and up as single contractions, then SiLU * up: the prefill's 256-row blocks):
    the pair epilogue's arithmetic, bf16(silu_tanh(bf16(Wg h)) * bf16(Wu h)), against the
    exact sums."""
    torch.manual_seed(40 + B)
    M, K, G = 3072, 1024, 32
    wg = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    wu = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    gw, uw = quantize_to_wire(wg, G), quantize_to_wire(wu, G)
    qg, sg = wire_to_numpy(gw, M, K, G)
    qu, su = wire_to_numpy(uw, M, K, G)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda")).to(torch.bfloat16)
    gh = torch.full((B, M), float("nan"), dtype=torch.bfloat16, device="cuda")
    tw = _lib.tc_workspace([(M, K)], B, "cuda")
    _lib.call("iron_gemv_w8a16_ex", gw.data_ptr(), uw.data_ptr(), M, K, G, 0, x.data_ptr(), K, B, nw.data_ptr(),
              1e-6, 0, None, 0, gh.data_ptr(), M, tw.data_ptr(), tw.numel(), _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.lib().iron_tc_status(tw.data_ptr(), 0) == 0
    rows = sorted({0, B // 2, 255 % B, 256 % B, B - 1})
    h = ops.rms_norm_f32(host(x)[rows], host(nw), 1e-6)
    g = rnd(h.astype(np.float64) @ _deq(qg, sg, G).T)
    u = rnd(h.astype(np.float64) @ _deq(qu, su, G).T)
    want = rnd(ops.silu_tanh_bf16(g) * u)
    got = host(gh)[rows]
    err = np.abs(got - want)
    lim = 2.0 ** -6 * np.abs(want) + 1e-4
    assert not np.isnan(host(gh)).any()
    assert np.mean(err <= lim) >= 0.999 and np.max(err) <= 0.05, f"pair: {np.mean(err <= lim):.4f}, max {err.max()}"


def test_tc_without_workspace_runs_the_exact_launches():
    """No workspace: batch 16+ runs the exact kernel in launches of 8 rows, whose every
    output is the exact dequantised sum rounded once to bf16."""
    torch.manual_seed(8)
    M, K, G, B = 2048, 1024, 32, 24
    w = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    wire = quantize_to_wire(w, G)
    q, s = wire_to_numpy(wire, M, K, G)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    y = _gemv(wire, M, K, G, 0, x, ws=None)
    assert np.array_equal(host(y), rnd(ops.gemv_int8_exact(q, s, host(x).astype(np.float64))))
    # a workspace too small for the split-K counters takes the same exact path
    assert torch.equal(_gemv(wire, M, K, G, 0, x, ws=_lib.workspace(256, "cuda")), y)


def test_tc_concurrent_projections_on_two_streams():
    """Two batch-32 projections in flight at once on two streams, each with its own
    workspace, give the results each gives alone: the kernels share no global scratch."""
    torch.manual_seed(9)
    G, B = 32, 32
    shapes = [(6144, 1024), (1024, 3072)]
    cases = []
    for M, K in shapes:
        w = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
        x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
        wire = quantize_to_wire(w, G)
        cases.append((M, K, wire, x, _gemv(wire, M, K, G, 0, x)))
    streams = [torch.cuda.Stream() for _ in cases]
    wss = [_lib.tc_workspace([(M, K)], B, "cuda") for M, K, *_ in cases]
    torch.cuda.synchronize()
    outs = [[] for _ in cases]
    for _ in range(8):  # interleaved launches: the two kernels overlap on the GPU
        for i, (M, K, wire, x, _) in enumerate(cases):
            with torch.cuda.stream(streams[i]):
                outs[i].append(_gemv(wire, M, K, G, 0, x, ws=wss[i], stream=streams[i], sync=False))
    torch.cuda.synchronize()
    for i, (M, K, wire, x, want) in enumerate(cases):
        assert _lib.lib().iron_tc_status(wss[i].data_ptr(), 0) == 0
        for y in outs[i]:
            assert torch.equal(y, want), f"projection {M}x{K} changed under a concurrent one"


@pytest.mark.parametrize("B", [32, 520])
def test_tc_bf16_weight_row_blocks(B):
    """bf16 weights (the lm_head and shared-weight bf16 GEMV path) at 32 rows and in row
    blocks (520 rows: five blocks of 112) against the float64 sum: one bf16 output
    rounding plus float32 summation error (which is relative to the terms' magnitudes,
    so an output near zero may sit a few ulps away), 95 % bit-exact."""
    torch.manual_seed(70 + B)
    M, K = 2048, 1024
    A = (torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
    y = torch.full((B, M), float("nan"), dtype=torch.bfloat16, device="cuda")
    tw = _lib.tc_workspace([(M, K)], B, "cuda")
    _lib.call("iron_gemv_bf16", A.data_ptr(), M, K, x.data_ptr(), B, 0, y.data_ptr(), tw.data_ptr(), tw.numel(),
              _lib.stream_ptr())
    torch.cuda.synchronize()
    assert _lib.lib().iron_tc_status(tw.data_ptr(), 0) == 0
    a64, x64 = host(A).astype(np.float64), host(x).astype(np.float64)
    exact = x64 @ a64.T
    lim = 2.0 ** -8 * np.abs(exact) + 1e-5 * (np.abs(x64) @ np.abs(a64).T) + 1e-30
    err = np.abs(host(y).astype(np.float64) - exact)
    assert np.all(err <= lim), f"{B} rows: worst {np.max(err / lim):.3g} of the bound"
    assert np.mean(host(y) == rnd(exact.astype(np.float32))) >= 0.95


def test_tc_shared_workspace_across_shapes():
    """Projections of different shapes one after another on ONE workspace at 300 rows
    (the prefill's pattern: down, then the next layer's QKV): the split-K arrival
    counters sit in a fixed region, so a projection with many (row block, tile) pairs
    never reads another's partial tiles as counters.  Every row against the exact
    kernel."""
    torch.manual_seed(90)
    G, B = 32, 300
    shapes = [(1024, 3072), (4096, 1024), (1024, 2048), (3072, 1024), (4096, 1024)]
    ws = _lib.tc_workspace(shapes, B, "cuda")
    for M, K in shapes:
        w = quantize_to_wire((torch.randn(M, K, device="cuda") * 0.02).to(torch.bfloat16), G)
        x = torch.randn(B, K, device="cuda").to(torch.bfloat16)
        got = host(_gemv(w, M, K, G, 0, x, ws=ws))
        q, s = wire_to_numpy(w, M, K, G)
        _check(got, q, s, host(x), G, f"{M}x{K} after other shapes")
