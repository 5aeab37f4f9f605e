"""Per-kernel device time of decode steps, from a CUPTI trace (torch.profiler).

``python -m iron_b200.kernel_breakdown [--batch B] [--prompt P] [--steps N]``
prefills ``batch`` random prompts of ``P`` tokens into a synthetic Qwen3-0.6B
(int8 g32), then traces ``N`` decode steps and prints, per kernel name, the device
time per step, its share and the launches per step.  At batch 1 the step is the
one persistent kernel; above, the chained kernels replayed as a CUDA graph.
"""

from __future__ import annotations

import argparse

import torch
from torch.profiler import ProfilerActivity, profile

from .qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    B, P = args.batch, args.prompt
    dev = torch.device("cuda")
    cfg = Qwen3Config.qwen3_0_6b()
    w = Qwen3Weights.synthetic(cfg, seed=args.seed, group=32, device=dev)
    dec = Qwen3B200(w, max_seq=P + args.steps + 16, batch=B, device=dev)
    g = torch.Generator().manual_seed(args.seed + 1)
    prompts = torch.randint(0, cfg.V, (B, P), generator=g).tolist()
    for p in range(P):
        nxt = dec.step_tokens([prompts[b][p] for b in range(B)], p)
    dec.set_position(P)
    with torch.cuda.stream(dec.stream):
        dec.tok.copy_(nxt.to(dev))
    for _ in range(3):
        dec.run_step(from_tokens=True, advance=True)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            dec.run_step(from_tokens=True, advance=True)
        torch.cuda.synchronize()
    tot: dict[str, tuple[int, float]] = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            k = e.name.split("(")[0][:70]
            c, t = tot.get(k, (0, 0.0))
            tot[k] = (c + 1, t + e.device_time)
    all_t = sum(t for _, t in tot.values())
    n = args.steps
    print(f"batch {B}, context ~{P}: {all_t / n:.1f} us of kernels per step")
    for k, (c, t) in sorted(tot.items(), key=lambda x: -x[1][1]):
        print(f"{t / n:9.1f} us/step {100 * t / all_t:5.1f} %  x{c / n:.0f}  {k}")


if __name__ == "__main__":
    main()
