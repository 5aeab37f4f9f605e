"""Shared helpers for the parity tests (host <-> device, tolerance asserts)."""

import numpy as np
import torch

from iron_b200.test_utils import allclose_report, cosine
from oracle.bf16 import from_bits, round_bits

RTOL, ATOL = 2e-2, 1e-2  # the decode path's bf16 gate


def dev_bf16(x) -> torch.Tensor:
    """float32 numpy values (bf16-representable) or uint16 bits -> bf16 CUDA tensor."""
    a = np.asarray(x)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(round_bits(a)).view(torch.bfloat16).cuda()


def dev_u8(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x)).view(np.uint8).copy()).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def assert_close(got, want, rtol=RTOL, atol=ATOL, what=""):
    ok, err, ratio = allclose_report(got, want, rtol, atol)
    assert ok, f"{what}: max |err| {err:.3g}, worst err/limit {ratio:.3g} (rtol {rtol}, atol {atol})"


def assert_ulps(got, want, max_ulp=1, frac_exact=0.0, what=""):
    """bf16 values within ``max_ulp`` units in the last place."""
    g = round_bits(np.asarray(got, np.float32).reshape(-1)).astype(np.int32)
    w = round_bits(np.asarray(want, np.float32).reshape(-1)).astype(np.int32)
    sg = np.where(g >= 0x8000, 0x8000 - g, g)  # sign-magnitude -> ordered integers
    sw = np.where(w >= 0x8000, 0x8000 - w, w)
    d = np.abs(sg - sw)
    assert d.max() <= max_ulp, f"{what}: max ulp distance {d.max()}"
    assert np.mean(d == 0) >= frac_exact, f"{what}: only {np.mean(d == 0):.4f} bit-exact"


def w8_error_bound(q, s_bits, x):
    """Bound on |kernel - exact| for the int8 GEMV before its bf16 output rounding.

    The kernel rounds each activation to int16 block floating point per quant group
    (error <= max|x_g| 2^-15 per element) and accumulates the per-chunk integer sums
    in float32; returns (bfp bound + float32 bound) per output row, (B, M) or (M,)."""
    q = np.asarray(q, np.float64)
    s = from_bits(s_bits).astype(np.float64)
    x = np.atleast_2d(np.asarray(x, np.float64))
    M, K = q.shape
    G = K // s.shape[1]
    qa = np.abs(q).reshape(M, K // G, G).sum(2) * s                        # (M, KG)
    xmax = np.abs(x).reshape(x.shape[0], K // G, G).max(2)                   # (B, KG)
    bfp = (xmax * 2.0 ** -15) @ qa.T                                         # (B, M)
    terms = np.abs(x) @ (np.abs(q) * np.repeat(s, G, axis=1)).T             # (B, M)
    out = bfp + 1e-6 * terms
    return out[0] if np.asarray(x).shape[0] == 1 and out.shape[0] == 1 else out


def assert_w8_exact(got, q, s_bits, x, what=""):
    """|kernel - exact dequantised sum| <= one bf16 rounding + 2 * w8_error_bound."""
    from oracle import ops
    exact = ops.gemv_int8_exact(q, s_bits, x)
    got = np.asarray(got, np.float64).reshape(np.shape(exact))
    lim = 2.0 ** -8 * np.abs(exact) + 2 * w8_error_bound(q, s_bits, x).reshape(np.shape(exact))
    bad = np.abs(got - exact) > lim
    assert not bad.any(), f"{what}: {bad.sum()} rows off the exact sum, worst {np.max(np.abs(got - exact) / lim):.3g}"


def logit_gate(got, want, what, max_outside):
    """Full-model logit agreement: at most ``max_outside`` of the logits outside the bf16
    tolerance, none more than 0.1 away (a few bf16 ulps of the largest logits), and the
    two vectors aligned."""
    err = np.abs(got - want)
    outside = np.mean(err > ATOL + RTOL * np.abs(want))
    assert outside <= max_outside, f"{what}: {outside:.2%} of logits outside rtol {RTOL} / atol {ATOL}"
    assert err.max() <= 0.1, f"{what}: max |err| {err.max():.3g}"
    assert cosine(got, want) >= 0.9995, f"{what}: cosine {cosine(got, want):.6f}"


__all__ = ["logit_gate", "w8_error_bound", "assert_w8_exact", "dev_bf16", "dev_u8", "host", "bits", "assert_close", "assert_ulps", "from_bits", "RTOL", "ATOL"]
