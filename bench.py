#!/usr/bin/env python3
"""Qwen3-0.6B int8 (group 32) batch-1 greedy decode throughput on B200.

Workload (Qwen3-0.6B, the headline configuration): 28 layers, hidden 1024, 16/8 heads, head_dim 128,
SwiGLU 3072, vocab 151936 with a tied bf16 embedding/lm_head, projection
weights int8 RTN in groups of 32 (synthetic, seeded), batch 1.  A 1024-token
random prompt is prefilled (all prompt rows of a layer at once, Qwen3B200.prefill;
reported as prefill_s), then greedy decode steps are timed.  One step = one decoded token.  Every step streams
~0.78 GB of weights + the KV cache from HBM, far more than the 126 MB L2, so no
L2 flush is needed between steps.

  value   tokens/s of K back-to-back decode steps, inputs resident in HBM, CUDA
          events on the decoder's stream, max over ranks (whole-job aggregate).
  e2e     tokens/s through the public API (Qwen3B200.step_tokens): per step the
          token id and position go host->device from pinned memory and the next
          token comes back device->host.
  --gpus N: N independent replicas (the 0.6B batch-1 path does not shard), one
          per GPU, launched under torchrun; the value sums the replicas.
  --impl reference: the reference's CPU golden path (the numpy restatement in
          oracle/, the reference being NPU-only) on the host cores, one rank.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Qwen3 decode tokens/s"
# DRAM traffic of one step launch beyond its algorithmic bytes, from an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum = 795.5 MB at context 71, where the
# algorithmic bytes are 788.4 MB): accumulator zeroing, K/V and logit writes.  The
# weights and the K/V reads scale with the algorithmic bytes, so a launch's traffic is
# its algorithmic bytes plus this.
STEP_TRAFFIC_EXTRA = 7.1e6
UNIT = "tokens/s"
PROMPT = 1024
GROUP = 32


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prompt", type=int, default=PROMPT)
    ap.add_argument("--batch", type=int, default=1,
                    help="independent decode streams per GPU (1: the one-launch step; more: the chained "
                         "kernels as a CUDA graph)")
    ap.add_argument("--model", choices=["qwen3-0.6b", "qwen3-8b", "llama-1b"], default="qwen3-0.6b",
                    help="qwen3-8b: Qwen3-8B int8, tensor parallel over the torchrun world "
                         "(NCCL), a synthetic --prompt-position KV context (default 4096); llama-1b: "
                         "config 5, --batch streams per GPU (default 64) with ragged synthetic KV "
                         "lengths U[256, 8192], replicas across GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--oracle-steps", type=int, default=32,
                    help="teacher-forced oracle steps (greedy top-1 agreement; also the CPU baseline sample)")
    ap.add_argument("--no-extra", action="store_true", help="no bs32 / tp sub-records")
    ap.add_argument("--tp-collective", choices=["peer", "nccl"], default="nccl",
                    help="cross-rank steps of the tensor-parallel decoder: the library's peer-memory exchange "
                         "(one GPU per rank) or NCCL")
    ap.add_argument("--phases", action="store_true",
                    help="phase breakdown of the one-launch step (a profiling copy of the library), not a bench line")
    ap.add_argument("--breakdown", action="store_true",
                    help="per-kernel device time of --steps decode steps at --batch (CUPTI), not a bench line")
    ap.add_argument("--sweep", action="store_true", help="operator sweep of configuration 3, not a bench line")
    ap.add_argument("--sweep-reps", type=int, default=50)
    ap.add_argument("--sweep-only", choices=["gemv", "attn"], default=None,
                    help="run only the GEMV or only the decode-attention rows of the sweep")
    ap.add_argument("--sweep-json", type=str, default=None)
    ap.add_argument("--sweep-capture", nargs="?", const="", default=None,
                    help="with --sweep: only the small ncu capture case of the GEMV (optional NxKxB,... shapes)")
    args = ap.parse_args()
    if args.model == "qwen3-8b" and args.prompt == PROMPT:
        args.prompt = 4096
    if args.model == "llama-1b" and args.batch == 1:
        args.batch = 64
    return args


def workload(args):
    return {"workload": f"qwen3-0.6b int8-g{GROUP} greedy decode, batch {args.batch}, bf16 tied lm_head, "
                        f"{args.prompt}-token random prompt{'s' if args.batch > 1 else ''} prefilled",
            "batch": args.batch, "layers": 28, "vocab": 151936, "group": GROUP, "prompt_tokens": args.prompt,
            "l2": "no flush: ~0.78 GB of weights streamed per step, larger than the 126 MB L2",
            "parallelism": f"replicas x{args.gpus}" if args.gpus > 1 else "single GPU"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.flush()

    def summary(self):
        rows = []
        try:
            for line in Path(self.f.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def aggregate_replicas(t_ms, e2e_ms, steps, world, device):
    """Whole-job numbers of ``world`` independent replicas that each decoded ``steps``
    tokens: the slowest rank's device time (MAX all-reduce over the process group when
    world > 1) and the tokens of all ranks over it.  Returns (t_ms, e2e_ms, tokens/s,
    e2e tokens/s)."""
    import torch
    tt = torch.tensor([t_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms = float(tt[0]), float(tt[1])
    return t_ms, e2e_ms, world * steps / (t_ms / 1000.0), world * steps / (e2e_ms / 1000.0)


def token_bytes(cfg, group, ctx, batch=1):
    """Algorithmic HBM bytes of one decode step of ``batch`` streams attending over ``ctx``
    positions each: every int8 projection wire (payload + one bf16 scale per group) and the
    norm weights once, the bf16 tied lm_head once; per stream the embedding row, K/V of all
    ``ctx`` positions read and the new position's K/V written, plus the activations in and
    out of each GEMV."""
    D, FF, HD = cfg.D, cfg.FF, cfg.HD
    QD, QKV = cfg.Hq * HD, (cfg.Hq + 2 * cfg.Hkv) * HD
    wire = lambda M, K: M * K + M * (K // group) * 2
    per_layer = (wire(QKV, D) + wire(D, QD) + 2 * wire(FF, D) + wire(D, FF)
                 + (2 * D + 2 * HD) * 2                                   # norm weights
                 + batch * (2 * cfg.Hkv * HD * 2 * ctx                    # K/V read
                            + 2 * cfg.Hkv * HD * 2                        # K/V write
                            + (D + QKV + QD + D + D + 2 * FF + FF + D) * 2))  # GEMV activations
    head = cfg.V * D * 2 + D * 2 + batch * (D * 2 + 4)                   # lm_head, final norm, x, token
    return cfg.n_layers * per_layer + head + batch * D * 2


# ---------------------------------------------------------------------------
# CPU oracle sample (test infrastructure: the checker and the CPU baseline only)
# ---------------------------------------------------------------------------
def oracle_replay(weights_np, kv_np, shape, pos, inputs, gpu_next, threads, angles=None):
    """Teacher-forced replay of ``len(inputs)`` GPU decode steps on the composed CPU oracle
    (oracle/qwen3.py), from the GPU's own weights and K/V cache at ``pos``: step i feeds
    the GPU's input token ``inputs[i]`` at ``pos + i`` (the oracle keeps its own K/V from
    there on) and compares the oracle's greedy token with the GPU's ``gpu_next[i]``.  A
    disagreement counts as a near-tie when the two tokens' oracle logits differ by no
    more than the bf16 gate (atol 1e-2 + rtol 2e-2 of the larger).  Returns (tokens/s of
    the oracle, threads used, agreement record)."""
    import numpy as np
    from oracle import ops
    from oracle.qwen3 import OracleQwen3
    used = ops.set_threads(threads)
    orc = OracleQwen3(shape, weights_np, kv_np.shape[2], angles=angles)
    orc.kv[...] = kv_np
    t_tok, agree, near = [], 0, 0
    for i, (tin, tgpu) in enumerate(zip(inputs, gpu_next)):
        t0 = time.perf_counter()
        logits, want = orc.step(orc.embed(tin), pos + i)
        t_tok.append(time.perf_counter() - t0)
        if want == tgpu:
            agree += 1
        elif abs(float(logits[want]) - float(logits[tgpu])) <= 1e-2 + 2e-2 * float(np.abs(logits[want])):
            near += 1
    n = len(inputs)
    rec = {"steps": n, "from_position": pos, "top1_agree": agree / n, "near_ties": near,
           "top1_agree_or_near_tie": (agree + near) / n,
           "method": "teacher-forced: the oracle steps on the GPU's input tokens from the GPU's K/V cache"}
    return 1.0 / statistics.mean(t_tok), used, rec


def oracle_spot(weights_np, kv_np, shape, pos, token, threads, angles=None):
    """One oracle decode token at ``pos`` from a GPU K/V cache: its greedy token."""
    from oracle import ops
    from oracle.qwen3 import OracleQwen3
    ops.set_threads(threads)
    orc = OracleQwen3(shape, weights_np, kv_np.shape[2], angles=angles)
    orc.kv[...] = kv_np
    return orc.step(orc.embed(token), pos)[1]


# ---------------------------------------------------------------------------
def run_reference(args, rank):
    """Reference arm: the CPU golden path on the host cores (one rank).

    The weights follow the GPU arm's distributions (N(0, 0.02) bf16 masters quantised
    RTN int8 per group of 32 by the numpy restatement of Qwen3NPU._set_int8_rtn; norm
    weights 1 + N(0, 0.1); a tied N(0, 0.02) bf16 embedding), the K/V cache holds
    ``--prompt`` positions of N(0, 1).  One step is one decoder layer of a token at that
    position (a bounded sample: a whole token takes over a second on the host); the
    final RMSNorm + bf16 lm_head + argmax is timed on its own, three times, whatever
    ``--steps`` is.  tokens/s = 1 / (28 x mean layer time + mean head time)."""
    import numpy as np
    if rank != 0:
        return
    from oracle import ops
    from oracle.bf16 import rnd
    from oracle.qwen3 import OracleQwen3, Qwen3Shape
    shape = Qwen3Shape(group=GROUP)
    rng = np.random.default_rng(args.seed)
    threads = ops.set_threads(len(os.sched_getaffinity(0)))
    D, FF, QD, QKV = shape.D, shape.FF, shape.Hq * shape.HD, (shape.Hq + 2 * shape.Hkv) * shape.HD
    layers = []
    for _ in range(shape.n_layers):
        L = {}
        for name, (M, K) in (("wqkv", (QKV, D)), ("wo", (D, QD)), ("wg", (FF, D)), ("wu", (FF, D)),
                             ("wd", (D, FF))):
            master = rnd(np.float32(0.02) * rng.standard_normal((M, K), dtype=np.float32))
            L[name + "_q"], L[name + "_s"] = ops.quantize_rtn(master, GROUP)
        for name, n in (("norm1", D), ("norm2", D), ("qn", shape.HD), ("kn", shape.HD)):
            L[name] = rnd(1 + np.float32(0.1) * rng.standard_normal(n, dtype=np.float32))
        layers.append(L)
    w = {"layers": layers, "final_norm": rnd(1 + np.float32(0.1) * rng.standard_normal(D, dtype=np.float32)),
         "embed": rnd(np.float32(0.02) * rng.standard_normal((shape.V, D), dtype=np.float32))}
    max_seq = args.prompt + 8
    orc = OracleQwen3(shape, w, max_seq)
    orc.kv[...] = rnd(rng.standard_normal(orc.kv.shape, dtype=np.float32))
    pos = args.prompt
    x = orc.embed(int(rng.integers(0, shape.V)))

    def layer_step(i):
        nonlocal x
        t0 = time.perf_counter()
        x = orc.layer(i % shape.n_layers, x, pos)
        return time.perf_counter() - t0

    def head_step():
        t0 = time.perf_counter()
        xf = ops.rms_norm_ref(x.reshape(1, -1), w["final_norm"], weighted=True, eps=shape.eps).reshape(-1)
        int(np.argmax(ops.gemv_bf16(w["embed"], xf)))
        return time.perf_counter() - t0

    for i in range(args.warmup):
        layer_step(i)
    t0 = time.perf_counter()
    t_layer = [layer_step(args.warmup + i) for i in range(args.steps)]
    elapsed = time.perf_counter() - t0
    head_step()  # warm-up of the lm_head pass
    t_head = [head_step() for _ in range(3)]
    lay, head = statistics.mean(t_layer), statistics.mean(t_head)
    tps = 1.0 / (lay * shape.n_layers + head)
    sample = (f"{args.steps} steps of one decoder layer at position {pos} (mean {1000 * lay:.1f} ms) and 3 timed "
              f"passes of the final norm + bf16 lm_head + argmax (mean {1000 * head:.1f} ms); tokens/s = "
              f"1/(28 x layer + head); weights N(0,0.02) masters, RTN int8 g{GROUP}")
    line = {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * elapsed / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xbf16",
            "data": "synthetic", "config": workload(args), "impl": "reference",
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    """The headline line (Qwen3-0.6B, ``--batch`` streams per GPU, replicas across the
    world), with sub-records under ``extra``: ``bs32`` (the same workload at 32 streams
    per GPU) and, under ``--gpus N``, ``tp`` (Qwen3-8B tensor parallel over the N ranks,
    batch 1, context 4096, 16 steps)."""
    import torch
    oracle = world == 1 and not args.no_cpu_baseline
    line = qwen3_line(args, rank, world, local_rank, oracle=oracle)
    torch.cuda.empty_cache()
    extra = {}
    if args.batch == 1 and not args.no_extra:
        # a sub-record that fails (the same way on every rank) is reported, not fatal
        try:
            sub = qwen3_line(argparse.Namespace(**{**vars(args), "batch": 32}), rank, world, local_rank,
                             oracle=False, spot=oracle)
            if rank == 0:
                extra["bs32"] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "e2e", "roofline",
                                                     "gpu_launches", "oracle_spot_check", "prefill_s") if k in sub}
                extra["bs32"]["config"] = sub["config"]["workload"]
        except Exception as e:  # noqa: BLE001
            extra["bs32"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()
        if world > 1:
            tp_args = argparse.Namespace(**{**vars(args), "model": "qwen3-8b", "batch": 1, "prompt": 4096,
                                            "steps": 16, "warmup": 4, "no_cpu_baseline": True})
            try:
                sub = run_tp(tp_args, rank, world, local_rank, emit=False)
                if rank == 0:
                    extra["tp"] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "e2e", "roofline",
                                                       "gpu_launches", "n_gpus", "steps", "warmup", "limiter")
                                   if k in sub}
                    extra["tp"]["config"] = sub["config"]["workload"] + f", tp{world}"
            except Exception as e:  # noqa: BLE001
                extra["tp"] = {"error": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.empty_cache()
    if rank == 0:
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)


def qwen3_line(args, rank, world, local_rank, oracle=False, spot=False):
    """Qwen3-0.6B greedy decode at ``args.batch`` streams per GPU: batched prefill, W
    warm-up and K timed device-fed steps, K end-to-end steps through the public API.
    ``oracle``: the CPU baseline and the teacher-forced oracle agreement on stream 0
    (rank 0, one GPU); ``spot``: one oracle token of stream 0.  Returns the bench line
    (rank 0; None elsewhere)."""
    import torch
    import torch.distributed as dist
    from iron_b200.qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = Qwen3Config.qwen3_0_6b()
    K, W, NA = args.steps, args.warmup, args.oracle_steps if oracle else 0
    max_seq = (args.prompt + W + 2 * K + NA + 8 + 63) // 64 * 64
    w = Qwen3Weights.synthetic(cfg, seed=args.seed, group=GROUP, device=dev)
    B = args.batch
    dec = Qwen3B200(w, max_seq=max_seq, batch=B, device=dev)
    g = torch.Generator().manual_seed(args.seed + 1000 * rank)
    prompts = torch.randint(0, cfg.V, (B, args.prompt), generator=g).tolist()

    def barrier():
        if world > 1:
            dist.barrier()

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[0])
                          if "CUDA_VISIBLE_DEVICES" in os.environ and world == 1 else local_rank)
    clocks.start()
    # prefill: each stream's prompt through every layer at once (Qwen3B200.prefill; the
    # reference runs its prompt loop token by token, check_cosine_int8.py:49-54).  The
    # first pass loads the kernels; the second, over the same positions (it rewrites
    # the same K/V), is the one timed.
    for b in range(B):
        dec.prefill(prompts[b], stream=b)
    torch.cuda.synchronize()
    t_pre = time.perf_counter()
    for b in range(B):
        dec.prefill(prompts[b], stream=b)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pre
    pos = args.prompt
    dec.set_position(pos)
    for _ in range(W):
        dec.run_step(from_tokens=True, advance=True)
    pos += W
    # ---- timed region: K back-to-back decode steps, device-resident inputs ----
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(dec.stream)
    for _ in range(K):
        dec.run_step(from_tokens=True, advance=True)
    e1.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    pos += K
    t_ms = e0.elapsed_time(e1)
    # ---- e2e: public API per step (H2D token+position, D2H token) ----
    toks = dec.tok.cpu().tolist()
    # one untimed call first: it captures the host-fed step's graph
    toks = dec.step_tokens(toks, pos).tolist()
    pos += 1
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e2.record(dec.stream)
    for _ in range(K):
        toks = dec.step_tokens(toks, pos).tolist()
        pos += 1
    e3.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e2.elapsed_time(e3)
    clocks.stop()
    clk = clocks.summary()
    # ---- oracle material (stream 0): the K/V cache at pos, then NA teacher-forced steps ----
    if (oracle or spot) and rank == 0:
        kvnp = dec.kv[:, 0].float().cpu().numpy().reshape(cfg.n_layers, cfg.Hkv, max_seq, 2, cfg.HD)
        ins, outs, p0 = [], [], pos
        for _ in range(max(NA, 1)):
            ins.append(toks[0])
            toks = dec.step_tokens(toks, pos).tolist()
            outs.append(toks[0])
            pos += 1
    # ---- dominant kernel: the persistent step kernel (the only launch of a step) ----
    # algorithmic bytes of the timed steps, averaged over their attention lengths
    ctx0 = args.prompt + W + 1
    step_bytes = sum(token_bytes(cfg, GROUP, ctx0 + i, B) for i in range(K)) / K
    # ---- aggregate over ranks ----
    t_ms, e2e_ms, value, e2e = aggregate_replicas(t_ms, e2e_ms, K * B, world, dev)
    if rank != 0:
        return None
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = step_bytes / (t_ms / K / 1000.0) / 1e9
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": t_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xbf16", "data": "synthetic", "config": workload(args),
            # the step kernel reads (token, position); the chained kernels also the valid
            # lengths and K/V offsets, written on the host and copied with them
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 8 * B if dec.impl == "step" else 16 * B,
                    # the tokens, and the step kernel's error word / the two tensor-core status words
                    "d2h_bytes_per_step": 8 * B if dec.impl == "step" else 4 * B + (8 if B >= 16 else 0)},
            "gpu_launches": K * dec.launches_per_step(),
            "roofline": {"bound": "hbm",
                         "kernel": ("qwen3_step_kernel (one persistent launch per token)" if dec.impl == "step"
                                    else f"the chained kernels of one step ({dec.launches_per_step()} launches)"),
                         "bytes_per_launch": step_bytes, "achieved": achieved, "peak": peak,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650",
                         "unit": "GB/s", "frac": achieved / peak,
                         "traffic": step_bytes + STEP_TRAFFIC_EXTRA if dec.impl == "step" else None,
                         "traffic_source": "ncu dram bytes of one launch at context 71, scaled by the K/V bytes"},
            "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "prefill_s": prefill_s}
    if oracle or spot:
        from oracle.qwen3 import Qwen3Shape
        wnp = w.to_numpy()
        threads = len(os.sched_getaffinity(0))
        angles = dec.angles.float().cpu().numpy()
        if oracle:
            tps, used, rec = oracle_replay(wnp, kvnp, Qwen3Shape(group=GROUP), p0, ins, outs, threads, angles)
            line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": used, "kind": "port",
                                    "sample": f"{len(ins)} full decode tokens (28 layers + bf16 lm_head) of the "
                                              f"numpy oracle from position {p0}, teacher-forced on this run's "
                                              f"weights, K/V cache and tokens" + (" (stream 0)" if B > 1 else "")}
            line["oracle_agreement"] = rec
        line["oracle_spot_check"] = {"position": p0, "input_token": ins[0], "gpu_token": outs[0],
                                     "oracle_token": oracle_spot(wnp, kvnp, Qwen3Shape(group=GROUP), p0, ins[0],
                                                                 threads, angles)}
    return line


def run_tp(args, rank, world, local_rank, emit=True):
    """Qwen3-8B int8-g32 greedy decode, tensor parallel over the
    torchrun world (iron_b200/tp.py): the O / down partials summed and the
    vocabulary-parallel argmax pairs gathered over peer memory (``--tp-collective peer``,
    the library's exchange) or NCCL.  The context is ``--prompt`` positions of N(0, 1)
    K/V per stream (synthetic: prefilling 4096 tokens through 36 layers would only
    repeat the decode step); then W warm-up and K timed greedy steps."""
    import numpy as np
    import torch
    from iron_b200.qwen3 import Qwen3Config, Qwen3Weights
    from iron_b200.tp import Qwen3TP

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = Qwen3Config.qwen3_8b()
    K, W, B, P = args.steps, args.warmup, args.batch, args.prompt
    max_seq = (P + W + 2 * K + 8 + 63) // 64 * 64
    w = Qwen3Weights.synthetic(cfg, seed=args.seed, group=GROUP, device=dev)
    cpu_layer = w.to_numpy(n_layers=1) if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    coll = args.tp_collective if world > 1 else None
    dec = Qwen3TP(w, rank, world, max_seq=max_seq, batch=B, device=dev, collective=coll)
    del w
    torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(args.seed + 17 + rank)
    dec.kv[..., :P * 2 * cfg.HD].normal_(generator=g)  # per-token [K_t | V_t]: positions [0, P)
    dec.set_position(P)
    first = torch.randint(0, cfg.V, (B,), generator=torch.Generator().manual_seed(args.seed + 1))
    with torch.cuda.stream(dec.stream):
        dec.tok.copy_(first.to(dev, torch.int32))

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[0])
                          if "CUDA_VISIBLE_DEVICES" in os.environ and world == 1 else local_rank)
    clocks.start()
    for _ in range(W):
        dec.run_step(from_tokens=True, advance=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(dec.stream)
    for _ in range(K):
        dec.run_step(from_tokens=True, advance=True)
    e1.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    t_ms = e0.elapsed_time(e1)
    pos = P + W + K
    toks = dec.tok.cpu().tolist()
    # one untimed call first: it runs the host-fed step's first (eager) pass, which also
    # sets up the collectives, and captures its graph on the next
    for _ in range(2):
        toks = dec.step_tokens(toks, pos).tolist()
        pos += 1
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e2.record(dec.stream)
    for _ in range(K):
        toks = dec.step_tokens(toks, pos).tolist()
        pos += 1
    e3.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e2.elapsed_time(e3)
    # the cross-rank steps alone: a step's 2 x n_layers sums of its float32 partials and
    # one gather of the argmax pairs, through the step's own collective, back to back
    coll_ms = 0.0
    if world > 1:
        n_ar = 2 * cfg.n_layers
        with torch.cuda.stream(dec.stream):
            for _ in range(2 * n_ar):
                dec.collective(("sum", dec.part))
            barrier()
            torch.cuda.synchronize()
            e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e4.record(dec.stream)
            for _ in range(4 * n_ar):
                dec.collective(("sum", dec.part))
            for _ in range(4):
                dec.collective(("gather", dec.gathered, dec.pairs))
            e5.record(dec.stream)
        torch.cuda.synchronize()
        coll_ms = e4.elapsed_time(e5) / 4
    clocks.stop()
    clk = clocks.summary()
    tt = torch.tensor([t_ms, e2e_ms, coll_ms], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_ms, coll_ms = float(tt[0]), float(tt[1]), float(tt[2])
    dec.close()
    if rank != 0:
        return None
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    # every weight, the lm_head and the K/V heads are split over the ranks: bytes per GPU
    step_bytes = sum(token_bytes(cfg, GROUP, P + W + 1 + i, B) for i in range(K)) / K / world
    achieved = step_bytes / (t_ms / K / 1000.0) / 1e9
    line = {"metric": METRIC, "value": K * B / (t_ms / 1000.0), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": t_ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8xbf16", "data": "synthetic",
            "config": {"workload": f"qwen3-8b int8-g{GROUP} greedy decode, batch {B}, bf16 tied lm_head, "
                                   f"{P}-position synthetic N(0,1) KV context",
                       "batch": B, "layers": 36, "hidden": 4096, "vocab": 151936, "group": GROUP,
                       "context": P, "parallelism": f"tp{world}",
                       "collectives": (f"{args.tp_collective if world > 1 else 'none'}: all-reduce of batch x "
                                       f"4096 float32 twice per layer, all-gather of 8 bytes per stream per step"),
                       "l2": "no flush: ~9 GB / world of weights streamed per step, larger than the L2"},
            "e2e": {"value": K * B / (e2e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": 16 * B,
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": K * dec.launches_per_step(),
            "roofline": {"bound": "hbm", "kernel": f"the chained kernels of one step ({dec.launches_per_step()} "
                                                   f"launches) per GPU",
                         "bytes_per_launch": step_bytes, "achieved": achieved, "peak": peak,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650",
                         "unit": "GB/s", "frac": achieved / peak, "traffic": None},
            "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    if world > 1:
        line["limiter"] = {"collectives_ms_per_step": coll_ms, "step_ms": t_ms / K,
                           "share": coll_ms / (t_ms / K),
                           "what": f"{2 * cfg.n_layers} all-reduces of {B} x {cfg.D} float32 + one all-gather "
                                   f"per step over {args.tp_collective}, timed alone back to back"}
    if cpu_layer is not None:
        from oracle import ops
        from oracle.bf16 import rnd
        from oracle.qwen3 import OracleQwen3, Qwen3Shape
        threads = ops.set_threads(len(os.sched_getaffinity(0)))
        shape = Qwen3Shape(D=cfg.D, FF=cfg.FF, Hq=cfg.Hq, Hkv=cfg.Hkv, HD=cfg.HD, V=cfg.V, n_layers=1, group=GROUP)
        orc = OracleQwen3(shape, cpu_layer, P + 1)
        rng = np.random.default_rng(args.seed)
        orc.kv[...] = rnd(rng.standard_normal(orc.kv.shape).astype(np.float32))
        x = cpu_layer["embed"][int(first[0])]
        t0 = time.perf_counter()
        orc.layer(0, x, P)
        t_layer = time.perf_counter() - t0
        rows = cfg.V // 16  # the lm_head on 1/16 of its rows, scaled
        t0 = time.perf_counter()
        ops.gemv_bf16(cpu_layer["embed"][:rows], x)
        t_head = (time.perf_counter() - t0) * 16
        tps = 1.0 / (cfg.n_layers * t_layer + t_head)
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"one Qwen3-8B decoder layer of the numpy oracle at position {P} "
                                          f"(x 36) + the bf16 lm_head on 1/16 of its rows (x 16), this run's "
                                          f"weights"}
    if emit:
        print(json.dumps(line), flush=True)
    return line


def llama_step_bytes(cfg, lens):
    """Algorithmic HBM bytes of one batched Llama decode step: every bf16 weight and the
    tied lm_head once, each stream's K/V of its positions read and the new one
    written, the activations in and out of each projection."""
    D, FF, HD = cfg.D, cfg.FF, cfg.HD
    weights = (cfg.QKV * D + D * cfg.QD + 3 * FF * D) * 2 + 2 * D * 2
    kv = sum(2 * cfg.Hkv * HD * 2 * (n + 1) for n in lens)
    acts = len(lens) * (D + cfg.QKV + 2 * cfg.QD + 3 * D + 4 * FF) * 2
    return cfg.n_layers * weights + cfg.n_layers * (kv + acts) + cfg.V * D * 2 + D * 2


def run_llama(args, rank, world, local_rank):
    """Llama-3.2-1B-shaped bf16 decode, --batch independent streams per
    GPU (64 by default) whose K/V lengths are drawn uniform in [256, 8192] (seeded per
    rank) over a synthetic N(0, 1) cache; replicas across the torchrun world."""
    import numpy as np
    import torch
    from iron_b200.llama import LlamaB200, LlamaConfig, LlamaWeights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = LlamaConfig.llama_3_2_1b()
    K, W, B = args.steps, args.warmup, args.batch
    rng = np.random.default_rng(args.seed + 31 * rank)
    lens = [int(v) for v in rng.integers(256, 8193, B)]
    max_seq = (max(lens) + W + 2 * K + 8 + 63) // 64 * 64
    w = LlamaWeights.synthetic(cfg, seed=args.seed, device=dev)
    dec = LlamaB200(w, max_seq=max_seq, batch=B, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed + 17 + rank)
    dec.kv.normal_(generator=g)
    dec.set_positions(lens)
    first = torch.randint(0, cfg.V, (B,), generator=torch.Generator().manual_seed(args.seed + 1))
    with torch.cuda.stream(dec.stream):
        dec.tok.copy_(first.to(dev, torch.int32))

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[0])
                          if "CUDA_VISIBLE_DEVICES" in os.environ and world == 1 else local_rank)
    clocks.start()
    for _ in range(W):
        dec.run_step(advance=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(dec.stream)
    for _ in range(K):
        dec.run_step(advance=True)
    e1.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    t_ms = e0.elapsed_time(e1)
    pos = [n + W + K for n in lens]
    toks = dec.tok.cpu().tolist()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e2.record(dec.stream)
    for _ in range(K):
        toks = dec.step_tokens(toks, pos).tolist()
        pos = [p + 1 for p in pos]
    e3.record(dec.stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e2.elapsed_time(e3)
    clocks.stop()
    clk = clocks.summary()
    t_ms, e2e_ms, value, e2e = aggregate_replicas(t_ms, e2e_ms, K * B, world, dev)
    if rank != 0:
        return
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    step_bytes = sum(llama_step_bytes(cfg, [n + W + i for n in lens]) for i in range(K)) / K
    achieved = step_bytes / (t_ms / K / 1000.0) / 1e9
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": t_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"llama-3.2-1b-shaped bf16 greedy decode, {B} streams per GPU, ragged "
                                   f"synthetic N(0,1) KV lengths U[256, 8192] (mean {sum(lens) / B:.0f})",
                       "batch_per_gpu": B, "layers": 16, "hidden": 2048, "vocab": 128256,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "no flush: ~11 GB streamed per step per GPU, larger than the L2"},
            # tokens, positions, lengths and K/V offsets in; tokens and the two status words out
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 16 * B,
                    "d2h_bytes_per_step": 4 * B + (8 if B >= 16 else 0)},
            "gpu_launches": K * dec.launches_per_step(),
            "roofline": {"bound": "hbm", "kernel": f"the chained kernels of one step ({dec.launches_per_step()} "
                                                   f"launches)",
                         "bytes_per_launch": step_bytes, "achieved": achieved, "peak": peak,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650",
                         "unit": "GB/s", "frac": achieved / peak, "traffic": None},
            "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    if world == 1 and not args.no_cpu_baseline:
        from oracle import ops
        from oracle.llama import LlamaShape, OracleLlama, linear
        threads = ops.set_threads(len(os.sched_getaffinity(0)))
        wn = w.to_numpy(n_layers=1)
        n = lens[0]
        orc = OracleLlama(LlamaShape(n_layers=1), wn, n + 1, angles=dec.angles[:n + 1].float().cpu().numpy())
        orc.kv[0] = dec.kv[0, 0].float().cpu().numpy().reshape(cfg.Hkv, max_seq, 2, cfg.HD)[:, :n + 1]
        x = wn["embed"][int(first[0])]
        t0 = time.perf_counter()
        orc.layer(0, x, n)
        t_layer = time.perf_counter() - t0
        rows = cfg.V // 16
        t0 = time.perf_counter()
        linear(wn["embed"][:rows], x)
        t_head = (time.perf_counter() - t0) * 16
        tps = 1.0 / (cfg.n_layers * t_layer + t_head)
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"one stream: one decoder layer of the numpy oracle (llama_cpu.py "
                                          f"restated) at position {n} (x 16) + the lm_head on 1/16 of its rows "
                                          f"(x 16), this run's weights and K/V"}
    print(json.dumps(line), flush=True)



# ---------------------------------------------------------------------------
# measurement modes behind the numbers in profiles/ (not the bench line)
# ---------------------------------------------------------------------------
SWEEP_GEMV_SHAPES = [(6144, 1024), (3072, 1024), (1024, 3072), (12288, 4096), (4096, 12288)]
SWEEP_GEMV_BATCH = [1, 8, 32]
SWEEP_ATTN_BATCH = [1, 8, 32, 64]
SWEEP_ATTN_LEN = [512, 4096, 32768]
L2_BYTES = 126 * 1024 * 1024
SWEEP_CAPTURE_CASES = [(6144, 1024, 8), (1024, 3072, 8), (6144, 1024, 1)]


def _sweep_copies(nbytes: int, cap: int) -> int:
    """Operand copies whose total exceeds twice the L2."""
    return max(2, min(cap, -(-2 * L2_BYTES // nbytes)))


def _sweep_timed(fns, reps: int) -> float:
    """Mean milliseconds per launch of ``fns`` (one per operand copy) run back to back."""
    import torch
    for f in fns:
        f()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(reps, len(fns))
    # hold the stream for ~10 ms so every launch below is queued before the first event
    # fires: the host's per-launch cost stays outside the measured interval
    torch.cuda._sleep(20_000_000)
    e0.record(st)
    for i in range(n):
        fns[i % len(fns)]()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1) / n


def run_sweep(args):
    """Operator sweep (configuration 3): achieved HBM bandwidth of the int8 group-32 GEMV
    ``iron_gemv_w8a16`` at (N, K) x batch {1, 8, 32} and of decode attention
    ``iron_decode_attn`` (32 query / 8 KV heads, head_dim 128) at batch {1, 8, 32, 64} x
    KV length {512, 4096, 32768}, values N(0, 1).  Launches run back to back over enough
    operand copies to exceed twice the L2 (each reads a copy the previous ones evicted);
    a first row times an 8-element add the same way: the per-launch floor of the method.
    GB/s = algorithmic bytes / time per launch (GEMV N*K + N*(K/G)*2 + B*K*2 + B*N*2,
    attention B*2*Hkv*HD*L*2 + B*Hq*HD*4).  ``--sweep-capture [NxKxB,...]`` instead runs
    the small case of an ncu capture of the GEMV: ~300 MB of weight copies each run once,
    then one launch per case on a copy that has left the L2."""
    import torch
    from iron_b200 import _lib
    from iron_b200.qwen3 import quantize_to_wire
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    G = GROUP
    if args.sweep_capture is not None:
        shapes = [tuple(int(v) for v in c.split("x")) for c in args.sweep_capture.split(",") if c] or SWEEP_CAPTURE_CASES
        st = torch.cuda.current_stream().cuda_stream
        cases, warm = [], 0
        for N, K, B in shapes:
            w0 = quantize_to_wire((torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16), G)
            ws = [w0] + [w0.clone() for _ in range(max(1, 300 * 2**20 // (N * K)) - 1)]
            x = torch.randn(B, K, generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
            cases.append((N, K, B, ws, x, y, _lib.tc_workspace([(N, K)], B, dev)))

        def run(N, K, B, w, x, y, tw):
            _lib.call("iron_gemv_w8a16", w.data_ptr(), N, K, G, 1, 0, 0, 0, x.data_ptr(), B, None, y.data_ptr(),
                      tw.data_ptr(), tw.numel(), st)

        for N, K, B, ws, x, y, tw in cases:
            for w in ws[1:]:
                run(N, K, B, w, x, y, tw)
                warm += 1
        torch.cuda.synchronize()
        for N, K, B, ws, x, y, tw in cases:
            run(N, K, B, ws[0], x, y, tw)
        torch.cuda.synchronize()
        print(f"warm-up launches: {warm}; then one launch each of {shapes}")
        return
    peaks = ROOT / "MEASURED_PEAKS.json"
    peak = json.loads(peaks.read_text())["hbm_gbs"] if peaks.exists() else 6650.0
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    reps = args.sweep_reps
    rows = []
    a = torch.zeros(8, dtype=torch.bfloat16, device=dev)
    s_ = st()
    ms = _sweep_timed([lambda: _lib.call("iron_add", a.data_ptr(), a.data_ptr(), a.data_ptr(), 8, s_)], reps)
    rows.append({"kernel": "launch_floor", "us": ms * 1e3})
    print(json.dumps(rows[-1]), flush=True)
    for N, K in (SWEEP_GEMV_SHAPES if args.sweep_only != "attn" else []):
        wbytes = N * K + N * (K // G) * 2
        w0 = quantize_to_wire((torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16), G)
        ws = [w0] + [w0.clone() for _ in range(_sweep_copies(wbytes, 64) - 1)]
        for B in SWEEP_GEMV_BATCH:
            x = torch.randn(B, K, generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
            s_ = st()
            tw = _lib.tc_workspace([(N, K)], B, dev)
            fns = [(lambda w=w: _lib.call("iron_gemv_w8a16", w.data_ptr(), N, K, G, 1, 0, 0, 0, x.data_ptr(), B,
                                          None, y.data_ptr(), tw.data_ptr(), tw.numel(), s_)) for w in ws]
            ms = _sweep_timed(fns, reps)
            nbytes = wbytes + B * K * 2 + B * N * 2
            rows.append({"kernel": "gemv_w8a16", "N": N, "K": K, "batch": B, "us": ms * 1e3,
                         "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak, "bytes": nbytes,
                         "copies": len(ws)})
            print(json.dumps(rows[-1]), flush=True)
        del ws, w0
    H, KV, HD = 32, 8, 128
    for B in (SWEEP_ATTN_BATCH if args.sweep_only != "gemv" else []):
        for L in SWEEP_ATTN_LEN:
            kvbytes = B * 2 * KV * HD * L * 2
            q = torch.randn(B, H, HD, generator=g, device=dev).to(torch.bfloat16)
            kvs = [torch.randn(B, KV, 2 * L * HD, generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(_sweep_copies(kvbytes, 16))]
            out = torch.empty(B, H, HD, dtype=torch.bfloat16, device=dev)
            nws = _lib.lib().iron_decode_attn_workspace_bytes(B, H, HD, L)
            wsp = torch.empty(nws, dtype=torch.uint8, device=dev)
            s_ = st()
            fns = [(lambda kv=kv: _lib.call("iron_decode_attn", q.data_ptr(), kv.data_ptr(), out.data_ptr(), B, H, KV,
                                            HD, L, 0, 0, L, None, wsp.data_ptr(), nws, s_)) for kv in kvs]
            ms = _sweep_timed(fns, reps)
            nbytes = kvbytes + B * H * HD * 4
            rows.append({"kernel": "decode_attn", "batch": B, "kv_len": L, "us": ms * 1e3,
                         "gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / peak, "bytes": nbytes,
                         "copies": len(kvs)})
            print(json.dumps(rows[-1]), flush=True)
            del kvs, wsp
    if args.sweep_json:
        Path(args.sweep_json).write_text("\n".join(json.dumps(r) for r in rows) + "\n")


def run_breakdown(args):
    """Per-kernel device time of decode steps from a CUPTI trace (torch.profiler):
    ``--batch`` random prompts of ``--prompt`` tokens prefilled into a synthetic
    Qwen3-0.6B (int8 g32), then ``--steps`` traced decode steps; per kernel name the
    device time per step, its share and the launches per step.  Then the same table for
    one traced prefill of stream 0's prompt."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    from iron_b200.qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights
    B, P = args.batch, args.prompt
    dev = torch.device("cuda")
    cfg = Qwen3Config.qwen3_0_6b()
    w = Qwen3Weights.synthetic(cfg, seed=args.seed, group=GROUP, device=dev)
    dec = Qwen3B200(w, max_seq=P + args.steps + 16, batch=B, device=dev)
    g = torch.Generator().manual_seed(args.seed + 1)
    prompts = torch.randint(0, cfg.V, (B, P), generator=g).tolist()
    for b in range(B):
        dec.prefill(prompts[b], stream=b)
    dec.set_position(P)
    for _ in range(3):
        dec.run_step(from_tokens=True, advance=True)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            dec.run_step(from_tokens=True, advance=True)
        torch.cuda.synchronize()
    _print_kernel_table(prof, args.steps, f"batch {B}, context ~{P}", "step")
    # one more prefill of stream 0's prompt over the same positions (it rewrites the same K/V)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        dec.prefill(prompts[0], stream=0)
        torch.cuda.synchronize()
    _print_kernel_table(prof, 1, f"prefill of a {P}-token prompt", "prefill")


def _print_kernel_table(prof, n, title, unit):
    """Per kernel name of a torch.profiler trace: device time per ``unit``, share, launches."""
    import torch
    tot: dict[str, tuple[int, float]] = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            k = e.name.split("(")[0][:70]
            c, t = tot.get(k, (0, 0.0))
            tot[k] = (c + 1, t + e.device_time)
    all_t = sum(t for _, t in tot.values())
    print(f"{title}: {all_t / n:.1f} us of kernels per {unit}")
    for k, (c, t) in sorted(tot.items(), key=lambda x: -x[1][1]):
        print(f"{t / n:9.1f} us/{unit} {100 * t / all_t:5.1f} %  x{c / n:.0f}  {k}")


PHASE_MARKS = 32   # stamps per layer row
PHASE_ROWS = 64    # layer rows per CTA
# (label, first mark, second mark, from layer): time between two stamps of qwen3_step.cu
PHASE_SPANS = [("x poll (previous layer's down)", 0, 1, 1), ("QKV RMSNorm + staging", 1, 2, 0),
               ("QKV weights wait", 2, 3, 0), ("QKV tiles + publish", 3, 4, 0), ("q/k/v poll", 4, 5, 0),
               ("q/k RMSNorm + RoPE", 5, 6, 0), ("attention split", 6, 7, 0), ("split reduce + publish", 7, 8, 0),
               ("merge (first CTA of a group)", 8, 9, 0), ("merged poll + staging (O CTAs)", 9, 10, 0),
               ("O weights wait", 10, 11, 0), ("O tiles + publish", 11, 12, 0), ("x1 poll", 12, 13, 0),
               ("MLP RMSNorm + staging", 13, 14, 0), ("gate/up weights wait", 14, 15, 0),
               ("gate/up tiles + publish", 15, 16, 0), ("down inputs poll + staging", 16, 17, 0),
               ("down weights wait", 18, 19, 0), ("down slices + publish", 19, 20, 0)]
PHASE_EVENTS = [("QKV rows published", 4), ("q/k/v polled", 5), ("attention splits published", 8),
                ("merged heads published", 9), ("merged heads polled + staged", 10), ("x1 rows published", 12),
                ("x1 polled", 13), ("SwiGLU outputs published", 16), ("down inputs polled", 17),
                ("down slices published", 20)]


def build_profiling_library():
    """A second copy of the library with the step kernel's phase stamps compiled in
    (-DIRON_STEP_PROFILE: thread 0 of each CTA stores %globaltimer at fixed points of
    each layer); the product library is untouched."""
    from iron_b200 import build as b
    lib = b.PKG / "libiron_b200_prof.so"
    objd = b.PKG / "_build_prof"
    objd.mkdir(exist_ok=True)
    objs = []
    for src in sorted(b.CSRC.glob("*.cu")):
        obj = objd / (src.stem + ".o")
        if not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in b._deps(src)):
            subprocess.run([b.nvcc(), *b.ARCH, *b.FLAGS, "-DIRON_STEP_PROFILE", f"-I{b.INCLUDE}", "-c", str(src),
                            "-o", str(obj)], check=True, capture_output=True, text=True)
        objs.append(str(obj))
    subprocess.run([b.nvcc(), *b.ARCH, "-shared", "-o", str(lib), *objs, "-lcudart"], check=True)
    return lib


def run_phases(args):
    """Phase breakdown of the one-launch decode step at context ``--prompt``: per phase the
    microseconds per token summed over the layers (mean over CTAs) and per layer the
    slowest and the fastest CTA; then the global timeline of a layer: when the LAST CTA
    reached each hand-off, relative to the moment the last CTA had the layer's input
    (mean over the inner layers)."""
    import ctypes as C
    import numpy as np
    import torch
    from iron_b200.qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights
    lib = C.CDLL(str(build_profiling_library()))
    lib.iron_qwen3_decode_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    lib.iron_qwen3_step_profile_buffer.argtypes = [C.c_void_p]
    lib.iron_qwen3_grid.argtypes = [C.c_void_p]
    cfg = Qwen3Config.qwen3_0_6b()
    P = args.prompt
    dec = Qwen3B200(Qwen3Weights.synthetic(cfg, seed=args.seed, group=GROUP), max_seq=P + 128, impl="step")
    for p in range(P):
        dec.step_tokens([p % 1000], p)
    dec.set_position(P)
    st, mp = dec.stream, C.addressof(dec._model)
    n_cta = int(lib.iron_qwen3_grid(mp))

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
    plain_us = ev[0].elapsed_time(ev[1]) / 20 * 1000
    buf = torch.zeros(n_cta * PHASE_ROWS * PHASE_MARKS, dtype=torch.int64, device=dec.x.device)
    lib.iron_qwen3_step_profile_buffer(C.c_void_p(buf.data_ptr()))
    NL = cfg.n_layers
    spans, events, lm, totals = {}, {}, [], []
    for _ in range(10):
        buf.zero_()
        run(1)
        st.synchronize()
        t = buf.cpu().numpy().reshape(n_cta, PHASE_ROWS, PHASE_MARKS).astype(np.float64)
        lay = t[:, :NL]
        for name, a, b2, first in PHASE_SPANS:
            A, B_ = lay[:, first:, a], lay[:, first:, b2]
            v = np.where((A > 0) & (B_ > 0), (B_ - A) / 1000.0, np.nan)
            spans.setdefault(name, []).append((np.nanmean(np.nansum(v, 1)), np.nanmean(np.nanmax(v, 0)),
                                               np.nanmean(np.nanmin(v, 0))))
        for name, mk in PHASE_EVENTS:
            vals = []
            for l in range(1, NL - 1):
                col = lay[:, l, mk]
                col = col[col > 0]
                vals.append((col.max() - lay[:, l, 1].max()) / 1000.0)
            events.setdefault(name, []).append(np.mean(vals))
        fin = t[:, NL]
        lm.append(((fin[:, 2] - fin[:, 1]) / 1000.0).mean())
        totals.append((fin[:, 2].max() - t[:, 0, 0].min()) / 1000.0)
    lib.iron_qwen3_step_profile_buffer(C.c_void_p(0))
    print(f"step without stamps {plain_us:.1f} us; with stamps {np.mean(totals):.1f} us (first to last stamp); "
          f"context {P}; {n_cta} CTAs; per layer {np.mean(totals) / NL:.2f} us incl. the lm_head share")
    print(f"{'phase':34s} {'us/token':>9s} {'slowest/layer':>14s} {'fastest/layer':>14s}")
    for name, vals in spans.items():
        m = np.nanmean(np.array(vals, dtype=np.float64), axis=0)
        print(f"{name:34s} {m[0]:9.1f} {m[1]:14.2f} {m[2]:14.2f}")
    print(f"{'final RMSNorm + lm_head + argmax':34s} {np.mean(lm):9.1f}")
    print("timeline of a layer (last CTA, us after the last CTA had x):")
    for name, vals in events.items():
        print(f"  {name:32s} {np.mean(vals):6.2f}")

def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.phases or args.breakdown or args.sweep:
        (run_phases if args.phases else run_breakdown if args.breakdown else run_sweep)(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.model == "qwen3-8b":
            run_tp(args, rank, world, local_rank)
        elif args.model == "llama-1b":
            run_llama(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
