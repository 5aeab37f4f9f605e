"""Tensor-parallel decode (iron_b200/tp.py) on the GPU.

world = 1 reproduces the chained single-GPU path bit for bit (the float32 partial
is the rounding of the fused residual epilogue).  world = 2 / 4 runs every rank's
real kernels on one GPU in lock step (tp.step_lockstep sums the O / down partials
and gathers the argmax pairs on the device) and is checked against the unsplit
chained path, with each rank given its heads' slice of the same KV cache before
every step; the Qwen3-8B shape (D 4096, FF 12288, 32/8 heads) is checked the same
way on two of its layers.  A multi-process NCCL run is bench.py --model qwen3-8b."""

import numpy as np
import pytest
import torch

from iron_b200.qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights
from iron_b200.tp import Qwen3TP, step_lockstep

from helpers import host, logit_gate

pytestmark = pytest.mark.gpu


def _prompt(n, V, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, V, n)]


def test_tp1_equals_chained_path():
    cfg = Qwen3Config.qwen3_0_6b()
    w = Qwen3Weights.synthetic(cfg, seed=5, n_layers=4)
    a = Qwen3B200(w, max_seq=64, impl="ops", keep_logits=True)
    b = Qwen3TP(w, 0, 1, max_seq=64)
    for p, t in enumerate(_prompt(12, cfg.V, 6)):
        ta, tb = a.step_tokens([t], p), b.step_tokens([t], p)
        assert torch.equal(a.logits, b.logits), f"pos {p}: logits differ"
        assert int(ta[0]) == int(tb[0])
        assert torch.equal(a.kv, b.kv)


def _lockstep_vs_single(cfg, w, world, n_steps, batch=1, seed=7):
    ref = Qwen3B200(w, max_seq=64, batch=batch, impl="ops", keep_logits=True, use_graph=False)
    ranks = [Qwen3TP(w, r, world, max_seq=64, batch=batch, use_graph=False) for r in range(world)]
    hk = cfg.Hkv // world
    agree = 0
    prompts = [_prompt(n_steps, cfg.V, seed + b) for b in range(batch)]
    for p in range(n_steps):
        toks = [prompts[b][p] for b in range(batch)]
        for r, rk in enumerate(ranks):
            rk.kv.copy_(ref.kv[:, :, r * hk:(r + 1) * hk])
        got = step_lockstep(ranks, toks, p)
        want = ref.step_tokens(toks, p)
        logits = torch.cat([rk.logits for rk in ranks], dim=1)
        for b in range(batch):  # one bf16 step of a hidden value moves a few logits by an ulp
            logit_gate(host(logits[b]), host(ref.logits[b]), f"pos {p} stream {b}", max_outside=0.02)
        for b in range(batch):
            tg, tw = int(got[b]), int(want[b])
            if tg == tw:
                agree += 1
            else:  # the partial sums add in another order: only a near-tie may flip
                la, lb = host(logits[b]), host(ref.logits[b])
                noise = float(np.abs(la - lb).max())
                assert abs(lb[tg] - lb[tw]) <= noise, f"pos {p} stream {b}: not a near-tie"
        # every rank decides the same token
        for rk in ranks[1:]:
            assert torch.equal(rk.tok, ranks[0].tok)
    assert agree >= 0.8 * n_steps * batch


@pytest.mark.parametrize("world", [2, 4])
def test_tp_lockstep_matches_single_gpu(world):
    cfg = Qwen3Config.qwen3_0_6b()
    w = Qwen3Weights.synthetic(cfg, seed=8, n_layers=4)
    _lockstep_vs_single(cfg, w, world, n_steps=10)


def test_tp_lockstep_batch_streams():
    cfg = Qwen3Config.qwen3_0_6b()
    w = Qwen3Weights.synthetic(cfg, seed=9, n_layers=3)
    _lockstep_vs_single(cfg, w, 2, n_steps=6, batch=3)


def test_tp_qwen3_8b_shape_two_layers():
    cfg = Qwen3Config.qwen3_8b()
    w = Qwen3Weights.synthetic(cfg, seed=10, n_layers=2)
    a = Qwen3B200(w, max_seq=64, impl="ops", keep_logits=True)
    b = Qwen3TP(w, 0, 1, max_seq=64)
    for p, t in enumerate(_prompt(4, cfg.V, 11)):
        ta, tb = a.step_tokens([t], p), b.step_tokens([t], p)
        assert torch.equal(a.logits, b.logits)
        assert int(ta[0]) == int(tb[0])
    _lockstep_vs_single(cfg, w, 2, n_steps=4, seed=12)
