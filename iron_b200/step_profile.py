"""Phase breakdown of the one-launch decode step (``qwen3_step_kernel``).

``python -m iron_b200.step_profile [--prompt N] [--samples K]`` builds a second copy
of the library with ``-DIRON_STEP_PROFILE`` (``iron_b200/libiron_b200_prof.so``; the
product library is untouched), decodes a synthetic Qwen3-0.6B int8-g32 model to
``--prompt`` positions, then runs K steps through the profiling copy.  In that copy
thread 0 of every CTA stores ``%globaltimer`` at fixed points of each layer
(``STEP_MARK`` in ``csrc/qwen3_step.cu``); this module turns the stamps into
microseconds per token for each phase, summed over the layers: the mean over CTAs,
the slowest CTA, and per layer (mean over layers) the slowest and the fastest CTA.
For a barrier wait the fastest CTA is the last to arrive: its wait is the barrier's
own latency, the rest is skew.

The stamps cost a global store per mark on one thread; the step time with and
without them is printed for comparison.
"""

from __future__ import annotations

import argparse
import ctypes as C
import subprocess
from pathlib import Path

from . import build as _build

PROF_LIB = _build.PKG / "libiron_b200_prof.so"
PROF_OBJ = _build.PKG / "_build_prof"
MARKS = 32   # stamps per layer row
ROWS = 64    # layer rows per CTA

# (label, first mark, second mark, from layer): the phase is the time between them
SPANS = [
    ("wait for the down sums (B1)", 0, 1, 1), ("residual + RMSNorm + BFP staging", 1, 2, 1),
    ("QKV weights wait", 2, 16, 0),
    ("QKV GEMV", 16, 20, 0), ("QKV slot release", 20, 3, 0), ("group barrier after QKV", 3, 4, 0),
    ("q/k norm + RoPE + v", 4, 14, 0), ("attention split", 14, 5, 0), ("group barrier after splits", 5, 6, 0),
    ("split merge (bulk copy)", 6, 15, 0), ("merged-head BFP staging", 15, 7, 0), ("O weights wait", 7, 17, 0),
    ("O GEMV (K split by head)", 17, 21, 0), ("O slot release", 21, 8, 0), ("grid barrier after O (B2)", 8, 9, 0),
    ("x1 = x + O sums, RMSNorm, BFP", 9, 10, 0), ("gate/up weights wait", 10, 18, 0),
    ("gate/up GEMV + SiLU*mul", 18, 22, 0), ("gate/up slot release", 22, 11, 0), ("down slice BFP", 11, 12, 0),
    ("down weights wait", 12, 19, 0), ("down GEMV (K slice) + reductions", 19, 23, 0),
    ("down slot release", 23, 13, 0),
]


def build_profiling_library() -> Path:
    """Compile the library once more with the phase stamps compiled in (skipped when the
    profiling library is newer than every source)."""
    srcs = sorted(_build.CSRC.glob("*.cu"))
    deps = srcs + sorted(_build.CSRC.glob("*.cuh")) + sorted(_build.INCLUDE.glob("*.h"))
    if PROF_LIB.exists() and all(d.stat().st_mtime <= PROF_LIB.stat().st_mtime for d in deps):
        return PROF_LIB
    PROF_OBJ.mkdir(exist_ok=True)
    objs = []
    for src in srcs:
        obj = PROF_OBJ / (src.stem + ".o")
        if not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in _build._deps(src)):
            cmd = [_build.nvcc(), *_build.ARCH, *_build.FLAGS, "-DIRON_STEP_PROFILE", f"-I{_build.INCLUDE}", "-c",
                   str(src), "-o", str(obj)]
            subprocess.run(cmd, check=True, capture_output=True, text=True)
        objs.append(str(obj))
    subprocess.run([_build.nvcc(), *_build.ARCH, "-shared", "-o", str(PROF_LIB), *objs, "-lcudart"], check=True)
    return PROF_LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--samples", type=int, default=10)
    args = ap.parse_args()

    import numpy as np
    import torch

    from .qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights

    lib = C.CDLL(str(build_profiling_library()))
    lib.iron_qwen3_decode_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    lib.iron_qwen3_step_profile_buffer.argtypes = [C.c_void_p]
    cfg = Qwen3Config.qwen3_0_6b()
    dec = Qwen3B200(Qwen3Weights.synthetic(cfg, seed=0, group=32), max_seq=args.prompt + 64 + args.samples,
                    impl="step")
    for p in range(args.prompt):
        dec.step_tokens([p % 1000], p)
    dec.set_position(args.prompt)
    st, mp = dec.stream, C.addressof(dec._model)
    n_cta = _build_grid(lib, mp)

    def run(n):
        for _ in range(n):
            if lib.iron_qwen3_decode_step(mp, 1, 1, st.cuda_stream) != 0:
                raise RuntimeError("profiling step failed")

    run(5)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(st)
    run(20)
    ev[1].record(st)
    st.synchronize()
    plain_ms = ev[0].elapsed_time(ev[1]) / 20
    buf = torch.zeros(n_cta * ROWS * MARKS, dtype=torch.int64, device=dec.x.device)
    lib.iron_qwen3_step_profile_buffer(C.c_void_p(buf.data_ptr()))
    NL = cfg.n_layers
    acc, totals = {}, []
    for _ in range(args.samples):
        run(1)
        st.synchronize()
        t = buf.cpu().numpy().reshape(n_cta, ROWS, MARKS).astype(np.float64)
        lay = t[:, :NL]
        for name, a, b, first in SPANS:
            v = (lay[:, first:, b] - lay[:, first:, a]) / 1000.0
            acc.setdefault(name, []).append((v.sum(1).mean(), v.sum(1).max(), v.max(0).mean(), v.min(0).mean()))
        tail = (lay[:, 1:, 0] - lay[:, :-1, 13]) / 1000.0
        acc.setdefault("layer tail (arrive B1)", []).append((tail.sum(1).mean(), tail.sum(1).max(), tail.max(0).mean(),
                                                            tail.min(0).mean()))
        fin = t[:, NL]
        lm = (fin[:, 2] - fin[:, 1]) / 1000.0
        acc.setdefault("final norm + lm_head + argmax", []).append((lm.mean(), lm.max(), lm.max(), lm.min()))
        totals.append((fin[:, 2].max() - t[:, 0, 0].min()) / 1000.0)
    lib.iron_qwen3_step_profile_buffer(C.c_void_p(0))
    print(f"step time without stamps: {plain_ms * 1000:.1f} us; with stamps (first to last stamp): "
          f"{np.mean(totals):.1f} us; context {args.prompt} positions; {n_cta} CTAs")
    print(f"{'phase':34s} {'mean/CTA':>9s} {'max/CTA':>9s} {'per layer':>10s} {'fastest':>8s}"
          "   (us per token summed over layers; per layer: slowest and fastest CTA)")
    for name, vals in acc.items():
        m = np.mean(np.array(vals), axis=0)
        print(f"{name:34s} {m[0]:9.1f} {m[1]:9.1f} {m[2]:10.2f} {m[3]:8.2f}")


def _build_grid(lib, mp) -> int:
    lib.iron_qwen3_grid.argtypes = [C.c_void_p]
    return int(lib.iron_qwen3_grid(mp))


if __name__ == "__main__":
    main()
