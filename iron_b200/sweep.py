"""Operator sweep: achieved HBM bandwidth of the decode kernels (int8 GEMV shapes x batch 1/8/32,
decode attention batch x context).

``python -m iron_b200.sweep [--reps N] [--json FILE]`` times, on synthetic data
(``--capture`` instead runs the small case of an ncu capture of the GEMV):

- the int8 group-32 GEMV ``iron_gemv_w8a16`` at (N, K) in {(6144,1024), (3072,1024),
  (1024,3072), (12288,4096), (4096,12288)} and batch in {1, 8, 32};
- decode attention ``iron_decode_attn`` with 32 query / 8 KV heads, head_dim 128, at
  batch in {1, 8, 32, 64} and KV length in {512, 4096, 32768} (values N(0, 1)).

Launches run back to back over enough copies of the weight (or KV cache) that the
copies together exceed twice the 126 MB L2, each launch reading a copy the previous
ones evicted, so the operands come from HBM as in a decode step; CUDA events time
the whole sequence, queued behind a short device sleep so host launch cost is hidden.
A first row times an 8-element add the same way: the per-launch floor of this method.  Achieved GB/s = algorithmic bytes / time per launch:
GEMV ``N*K + N*(K/G)*2 + B*K*2 + B*N*2``, attention ``B*2*Hkv*HD*L*2 + B*Hq*HD*4``; the
fraction is against ``MEASURED_PEAKS.json`` ``hbm_gbs``.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib
from .qwen3 import quantize_to_wire

GEMV_SHAPES = [(6144, 1024), (3072, 1024), (1024, 3072), (12288, 4096), (4096, 12288)]
GEMV_BATCH = [1, 8, 32]
ATTN_BATCH = [1, 8, 32, 64]
ATTN_LEN = [512, 4096, 32768]
G = 32
L2_BYTES = 126 * 1024 * 1024


def _copies(nbytes: int, cap: int) -> int:
    """Operand copies whose total exceeds twice the L2."""
    return max(2, min(cap, -(-2 * L2_BYTES // nbytes)))


def _timed(fns, reps: int) -> float:
    """Mean milliseconds per launch of ``fns`` (one per operand copy) run back to back."""
    for f in fns:
        f()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(reps, len(fns))
    # Hold the stream for ~10 ms so every launch below is queued before the first event
    # fires: the host's per-launch cost stays outside the measured interval.
    torch.cuda._sleep(20_000_000)
    e0.record(st)
    for i in range(n):
        fns[i % len(fns)]()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1) / n


CAPTURE_CASES = [(6144, 1024, 8), (1024, 3072, 8), (6144, 1024, 1)]


def capture_case(shapes=None):
    """The small case of an ncu capture of the GEMV kernel: for each case (N, K, batch)
    ~300 MB of weight copies, each run once (the launches ``ncu --launch-skip`` passes
    over), then one launch per case on a copy that has left the L2."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    st = torch.cuda.current_stream().cuda_stream
    cases, warm = [], 0
    shapes = shapes or CAPTURE_CASES
    for N, K, B in shapes:
        w0 = quantize_to_wire((torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16), G)
        ws = [w0] + [w0.clone() for _ in range(max(1, 300 * 2**20 // (N * K)) - 1)]
        x = torch.randn(B, K, generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
        cases.append((N, K, B, ws, x, y))

    def run(N, K, B, w, x, y):
        _lib.call("iron_gemv_w8a16", w.data_ptr(), N, K, G, 1, 0, 0, 0, x.data_ptr(), B, None, y.data_ptr(), st)

    for N, K, B, ws, x, y in cases:
        for w in ws[1:]:
            run(N, K, B, w, x, y)
            warm += 1
    torch.cuda.synchronize()
    for N, K, B, ws, x, y in cases:
        run(N, K, B, ws[0], x, y)
    torch.cuda.synchronize()
    print(f"warm-up launches: {warm}; then one launch each of {shapes}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--json", type=str, default=None)
    ap.add_argument("--capture", nargs="?", const="", default=None,
                    help="run only the small ncu capture case of the GEMV (optional NxKxB,NxKxB,... shapes)")
    args = ap.parse_args()
    if args.capture is not None:
        shapes = [tuple(int(v) for v in c.split("x")) for c in args.capture.split(",") if c]
        capture_case(shapes or None)
        return
    root = Path(__file__).resolve().parents[1]
    peaks = root / "MEASURED_PEAKS.json"
    peak = json.loads(peaks.read_text())["hbm_gbs"] if peaks.exists() else 6650.0
    dev = torch.device("cuda")
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    rows = []
    g = torch.Generator(device=dev).manual_seed(0)
    # launch floor: an 8-element add through the same C ABI, timed the same way
    a = torch.zeros(8, dtype=torch.bfloat16, device=dev)
    s_ = st()
    ms = _timed([lambda: _lib.call("iron_add", a.data_ptr(), a.data_ptr(), a.data_ptr(), 8, s_)], args.reps)
    rows.append({"kernel": "launch_floor", "us": ms * 1e3})
    print(json.dumps(rows[-1]), flush=True)
    for N, K in GEMV_SHAPES:
        wbytes = N * K + N * (K // G) * 2
        w0 = quantize_to_wire((torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16), G)
        ws = [w0] + [w0.clone() for _ in range(_copies(wbytes, 64) - 1)]
        for B in GEMV_BATCH:
            x = torch.randn(B, K, generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
            s_ = st()
            fns = [(lambda w=w: _lib.call("iron_gemv_w8a16", w.data_ptr(), N, K, G, 1, 0, 0, 0, x.data_ptr(), B,
                                          None, y.data_ptr(), s_)) for w in ws]
            ms = _timed(fns, args.reps)
            nbytes = wbytes + B * K * 2 + B * N * 2
            rows.append({"kernel": "gemv_w8a16", "N": N, "K": K, "batch": B, "us": ms * 1e3,
                         "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak, "bytes": nbytes,
                         "copies": len(ws)})
            print(json.dumps(rows[-1]), flush=True)
        del ws, w0
    H, KV, HD = 32, 8, 128
    for B in ATTN_BATCH:
        for L in ATTN_LEN:
            kvbytes = B * 2 * KV * HD * L * 2
            q = torch.randn(B, H, HD, generator=g, device=dev).to(torch.bfloat16)
            kvs = [torch.randn(B, KV, 2 * L * HD, generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(_copies(kvbytes, 16))]
            out = torch.empty(B, H, HD, dtype=torch.bfloat16, device=dev)
            nws = _lib.lib().iron_decode_attn_workspace_bytes(B, H, HD, L)
            wsp = torch.empty(nws, dtype=torch.uint8, device=dev)
            s_ = st()
            fns = [(lambda kv=kv: _lib.call("iron_decode_attn", q.data_ptr(), kv.data_ptr(), out.data_ptr(), B, H, KV,
                                            HD, L, 0, 0, L, None, wsp.data_ptr(), nws, s_)) for kv in kvs]
            ms = _timed(fns, args.reps)
            nbytes = kvbytes + B * H * HD * 4
            rows.append({"kernel": "decode_attn", "batch": B, "kv_len": L, "us": ms * 1e3,
                         "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak, "bytes": nbytes,
                         "copies": len(kvs)})
            print(json.dumps(rows[-1]), flush=True)
            del kvs, wsp
    if args.json:
        Path(args.json).write_text("\n".join(json.dumps(r) for r in rows) + "\n")


if __name__ == "__main__":
    main()
