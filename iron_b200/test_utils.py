"""Buffer comparison helpers with IRON's tolerance semantics.

``verify_buffer`` keeps the rule of iron/common/test_utils.py:51-126: element i
fails when ``|out - ref| > max(abs_tol, rel_tol * (|out| + |ref|))``, and an
optional ``max_error_rate`` lets a fraction of elements fail.  ``allclose``
is the torch-style rule ``|out - ref| <= atol + rtol * |ref|`` used for the
decode path's bf16 gate (rtol 2e-2, atol 1e-2).
"""

from __future__ import annotations

import numpy as np
import torch


def _np(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        return x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float64)


def verify_buffer(output, buf_name, reference, rel_tol=0.04, abs_tol=1e-6, max_error_rate=0.0):
    """Indices of elements outside tolerance (empty list = pass)."""
    out = _np(output).reshape(-1).astype(np.float64)
    ref = _np(reference).reshape(-1).astype(np.float64)
    errors = []
    if len(out) < len(ref):
        errors.extend(range(len(ref) - len(out)))
    n = min(len(out), len(ref))
    diff = np.abs(out[:n] - ref[:n])
    norm = np.minimum(np.abs(out[:n]) + np.abs(ref[:n]), np.finfo(np.float32).max)
    errors.extend(np.where(diff > np.maximum(abs_tol, rel_tol * norm))[0].tolist())
    if max_error_rate > 0.0 and errors and len(errors) <= int(n * max_error_rate):
        return []
    return errors


def allclose_report(output, reference, rtol=2e-2, atol=1e-2):
    """(ok, max_abs_err, worst_ratio) for ``|out-ref| <= atol + rtol*|ref|``."""
    out = _np(output).reshape(-1).astype(np.float64)
    ref = _np(reference).reshape(-1).astype(np.float64)
    err = np.abs(out - ref)
    lim = atol + rtol * np.abs(ref)
    ratio = float(np.max(err / lim)) if err.size else 0.0
    return bool(np.all(err <= lim)), float(err.max() if err.size else 0.0), ratio


def cosine(a, b) -> float:
    a = _np(a).reshape(-1).astype(np.float64)
    b = _np(b).reshape(-1).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
