"""Shared helpers for the parity tests (host <-> device, tolerance asserts)."""

import numpy as np
import torch

from iron_b200.test_utils import allclose_report
from oracle.bf16 import from_bits, round_bits

RTOL, ATOL = 2e-2, 1e-2  # the BASELINE bf16 gate


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
    g = round_bits(np.asarray(got, np.float32)).astype(np.int32)
    w = round_bits(np.asarray(want, np.float32)).astype(np.int32)
    sg = np.where(g >= 0x8000, 0x8000 - g, g)  # sign-magnitude -> ordered integers
    sw = np.where(w >= 0x8000, 0x8000 - w, w)
    d = np.abs(sg - sw)
    assert d.max() <= max_ulp, f"{what}: max ulp distance {d.max()}"
    assert np.mean(d == 0) >= frac_exact, f"{what}: only {np.mean(d == 0):.4f} bit-exact"


__all__ = ["dev_bf16", "dev_u8", "host", "bits", "assert_close", "assert_ulps", "from_bits", "RTOL", "ATOL"]
