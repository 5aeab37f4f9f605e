"""Tensor-parallel decode on CPU: the wire slicing and shard ranges of iron_b200/tp.py,
and the split of a decode step into rank-local work plus cross-rank sums, run as two
gloo ranks over the numpy oracle (oracle/qwen3.py) and checked against the unsplit
model.  The CUDA path of the same split is tests/test_tp_gpu.py."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from iron_b200.qwen3 import Qwen3Config
from iron_b200.tp import shard_config, shard_ranges, wire_cols, wire_rows
from oracle import ops
from oracle.bf16 import rnd

ROOT = Path(__file__).resolve().parents[1]


def _wire(q, s):
    return torch.from_numpy(ops.pack_tile_wire(q, s, 1, 1, "signed").view(np.uint8).copy())


def test_wire_slicing_matches_sliced_quantisation():
    rng = np.random.default_rng(0)
    M, K, G = 48, 256, 32
    q, s = ops.quantize_rtn(rng.standard_normal((M, K)).astype(np.float32) * 0.02, G)
    wire = _wire(q, s)
    assert torch.equal(wire_rows(wire, M, K, G, 8, 40), _wire(q[8:40], s[8:40]))
    assert torch.equal(wire_cols(wire, M, K, G, 64, 192), _wire(q[:, 64:192], s[:, 2:6]))
    with pytest.raises(ValueError):
        wire_cols(wire, M, K, G, 16, 192)


@pytest.mark.parametrize("cfg", [Qwen3Config.qwen3_0_6b(), Qwen3Config.qwen3_8b()])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_ranges_partition_the_model(cfg, world):
    """Every row of Wqkv / Wg / Wu / lm_head and every column of Wo / Wd belongs to
    exactly one rank, and a rank's Wqkv rows are its query, key, value heads."""
    lc = shard_config(cfg, world)
    cover = {k: np.zeros(n, int) for k, n in (("qkv", cfg.QKV), ("o", cfg.QD), ("ff", cfg.FF), ("d", cfg.FF),
                                              ("v", cfg.V))}
    for r in range(world):
        sr = shard_ranges(cfg, r, world)
        (qa, qb), (ka, kb), (va, vb) = sr["qkv_rows"]
        assert (qb - qa, kb - ka, vb - va) == (lc.Hq * cfg.HD, lc.Hkv * cfg.HD, lc.Hkv * cfg.HD)
        assert ka >= cfg.QD and va >= cfg.QD + cfg.Hkv * cfg.HD
        for a, b in sr["qkv_rows"]:
            cover["qkv"][a:b] += 1
        for key, name in (("o", "o_cols"), ("ff", "ff_rows"), ("d", "d_cols"), ("v", "vocab_rows")):
            a, b = sr[name]
            cover[key][a:b] += 1
        # the query heads of a rank attend to its own KV heads (GQA groups stay whole)
        assert qa // (cfg.Hq // cfg.Hkv * cfg.HD) == (ka - cfg.QD) // cfg.HD
    for key, c in cover.items():
        assert np.all(c == 1), key


# ---------------------------------------------------------------------------
# the split decode step on the numpy oracle, two gloo ranks
# ---------------------------------------------------------------------------
def _tiny_model(seed=1):
    from oracle.qwen3 import Qwen3Shape
    s = Qwen3Shape(D=256, FF=512, Hq=4, Hkv=2, HD=64, V=1024, n_layers=2, group=32)
    rng = np.random.default_rng(seed)
    w = {"layers": []}
    QKV = (s.Hq + 2 * s.Hkv) * s.HD
    for _ in range(s.n_layers):
        L = {}
        for name, (M, K) in (("wqkv", (QKV, s.D)), ("wo", (s.D, s.Hq * s.HD)), ("wg", (s.FF, s.D)),
                             ("wu", (s.FF, s.D)), ("wd", (s.D, s.FF))):
            L[name + "_q"], L[name + "_s"] = ops.quantize_rtn(
                rng.standard_normal((M, K)).astype(np.float32) * 0.02, s.group)
        for name, n in (("norm1", s.D), ("norm2", s.D), ("qn", s.HD), ("kn", s.HD)):
            L[name] = rnd(1 + 0.1 * rng.standard_normal(n).astype(np.float32))
        w["layers"].append(L)
    w["final_norm"] = rnd(1 + 0.1 * rng.standard_normal(s.D).astype(np.float32))
    w["embed"] = rnd(0.02 * rng.standard_normal((s.V, s.D)).astype(np.float32))
    return s, w


def _tp_step(s, w, kv, x, pos, rank, world, angles):
    """One decode step of rank ``rank``: local heads / rows / columns, with the O and down
    partials and the argmax candidates exchanged over the process group."""
    cfg = Qwen3Config(D=s.D, FF=s.FF, Hq=s.Hq, Hkv=s.Hkv, HD=s.HD, V=s.V, n_layers=s.n_layers)
    lc, sr = shard_config(cfg, world), shard_ranges(cfg, rank, world)
    G = s.group

    def allsum(v):
        t = torch.from_numpy(np.asarray(v, np.float64).copy())
        dist.all_reduce(t)
        return t.numpy()

    for i, L in enumerate(w["layers"]):
        qkv_q = np.concatenate([L["wqkv_q"][a:b] for a, b in sr["qkv_rows"]])
        qkv_s = np.concatenate([L["wqkv_s"][a:b] for a, b in sr["qkv_rows"]])
        qkv = ops.qkv_head(x, L["norm1"], lambda h: ops.gemv_int8_exact(qkv_q, qkv_s, h), L["qn"], L["kn"],
                           angles[pos], s.D, s.HD, lc.Hq, lc.Hkv, s.eps)
        QD, KVD = lc.Hq * s.HD, lc.Hkv * s.HD
        kv[i, :, pos, 0] = qkv[QD:QD + KVD].reshape(lc.Hkv, s.HD)
        kv[i, :, pos, 1] = qkv[QD + KVD:].reshape(lc.Hkv, s.HD)
        ctx = ops.decode_attention(qkv[:QD].reshape(lc.Hq, s.HD), kv[i, :, :pos + 1, 0], kv[i, :, :pos + 1, 1],
                                   pos, s.HD, lc.Hq, lc.Hkv)
        c0, c1 = sr["o_cols"]
        a = rnd(allsum(ops.gemv_int8_exact(L["wo_q"][:, c0:c1], L["wo_s"][:, c0 // G:c1 // G], ctx.reshape(-1))))
        x1 = rnd(np.asarray(x, np.float32) + a)
        hf = ops.rms_norm_f32(x1, L["norm2"], s.eps)
        f0, f1 = sr["ff_rows"]
        g = rnd(ops.gemv_int8_exact(L["wg_q"][f0:f1], L["wg_s"][f0:f1], hf))
        u = rnd(ops.gemv_int8_exact(L["wu_q"][f0:f1], L["wu_s"][f0:f1], hf))
        gh = rnd(ops.silu_tanh_bf16(g) * u)
        d0, d1 = sr["d_cols"]
        d = rnd(allsum(ops.gemv_int8_exact(L["wd_q"][:, d0:d1], L["wd_s"][:, d0 // G:d1 // G], gh)))
        x = rnd(x1 + d)
    xf = ops.rms_norm_ref(x.reshape(1, -1), w["final_norm"], weighted=True, eps=s.eps).reshape(-1)
    v0, v1 = sr["vocab_rows"]
    logits = ops.gemv_bf16(w["embed"][v0:v1], xf)
    t = int(np.argmax(logits))
    pair = torch.tensor([float(logits[t]), float(t + v0)], dtype=torch.float64)
    pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(pairs, pair)
    best = max(pairs, key=lambda p: (p[0].item(), -p[1].item()))  # largest value, then lowest index
    return x, int(best[1].item())


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.qwen3 import OracleQwen3
        s, w = _tiny_model()
        max_seq = 8
        orc = OracleQwen3(s, w, max_seq)
        lc = shard_config(Qwen3Config(D=s.D, FF=s.FF, Hq=s.Hq, Hkv=s.Hkv, HD=s.HD, V=s.V), world)
        kv = np.zeros((s.n_layers, lc.Hkv, max_seq, 2, s.HD), np.float32)
        tok, res = 7, []
        for pos in range(4):
            x_tp, t_tp = _tp_step(s, w, kv, orc.embed(tok), pos, rank, world, orc.angles)
            logits, t_full = orc.step(orc.embed(tok), pos)
            # the rank's KV heads are the unsplit model's heads [rank Hkv/n, (rank+1) Hkv/n)
            k0 = rank * lc.Hkv
            res.append((t_tp, t_full, np.abs(kv[:, :, :pos + 1] - orc.kv[:, k0:k0 + lc.Hkv, :pos + 1]).max()))
            tok = t_full
        out[rank] = res
    finally:
        dist.destroy_process_group()


def test_tp_split_decode_two_gloo_ranks_matches_unsplit_oracle():
    port = 29600 + os.getpid() % 1000
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    for rank in (0, 1):
        for t_tp, t_full, kv_err in res[rank]:
            assert t_tp == t_full
            assert kv_err == 0.0
