"""GPTQ checkpoint import (iron_b200/gptq.py) on CPU tensors.

Pinned to the reference's own import (tests/golden/gptq_pack.npz: the Qwen3 runtime's
``_set_int8`` -> ``_gptq_rows`` -> ``_pack_int8``, qwen3_npu_int8.py:350-455, run on
seeded checkpoint tensors): the wire bytes must be identical in both payload domains.
The wire must also dequantise to the checkpoint's weights, (u - 128) * bf16(scale),
and a whole checkpoint must load with its shapes checked.  The loaded wires are
the plain wires the GPU kernels are tested on (quantize_to_wire's format)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from iron_b200.gptq import gptq_rows, gptq_stack_to_wire, gptq_to_wire, gptq_wo_tile_major, load_qwen3_gptq
from iron_b200.qwen3 import Qwen3Config, wire_nbytes, wire_to_numpy
from oracle import ops
from oracle.bf16 import from_bits

GOLDEN = Path(__file__).resolve().parent / "golden" / "gptq_pack.npz"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _parts(g):
    return [(torch.from_numpy(g[f"qweight_{p}"]), torch.from_numpy(g[f"scales_{p}"].view(np.float16)))
            for p in ("a", "b")]


@pytest.mark.parametrize("domain,tag", [(0, "signed"), (1, "biased")])
def test_gptq_wire_matches_reference_import(golden, domain, tag):
    wire = gptq_stack_to_wire(_parts(golden), domain)
    assert np.array_equal(wire.numpy(), golden[f"wire_{tag}"])


def test_gptq_tile_wire_matches_reference_import(golden):
    """The per-core tile wire (4-row tiles over 2 columns) of the same import, and the
    oracle's tile packer on the unpacked rows."""
    wire = gptq_stack_to_wire(_parts(golden), 0, tile_m=4, cols=2)
    assert np.array_equal(wire.numpy(), golden["wire_signed_c2_t4"])
    q, s_bits = wire_to_numpy(gptq_stack_to_wire(_parts(golden), 0), 32, 256, 128)
    assert np.array_equal(wire.numpy(), ops.pack_tile_wire(q, s_bits, 4, 2, "signed"))
    with pytest.raises(ValueError, match="do not split"):
        gptq_stack_to_wire(_parts(golden), 0, tile_m=3, cols=2)


def test_gptq_wo_tile_major_matches_reference_import(golden):
    """fuse_o's Wo wire: 2 cores of 16 rows, windows of 3 tiles x 6 rows, so rows 16-17
    appear in both cores' windows and the last window reads 2 zero pad rows."""
    qw, sc = torch.from_numpy(golden["qweight_o"]), torch.from_numpy(golden["scales_o"].view(np.float16))
    wire = gptq_wo_tile_major(qw, sc, cols=2, tile_rows=6, tiles_per_core=3)
    assert np.array_equal(wire.numpy(), golden["wire_wo_c2_t6_n3"])
    with pytest.raises(ValueError, match="do not cover"):
        gptq_wo_tile_major(qw, sc, cols=2, tile_rows=5, tiles_per_core=3)
    with pytest.raises(ValueError, match="cores"):
        gptq_wo_tile_major(qw, sc, cols=3, tile_rows=6, tiles_per_core=3)


def test_gptq_wire_dequantises_to_checkpoint_weights(golden):
    """Independently of the reference code: the GPTQ weight is (u - 128) * scale with u
    the byte k % 4 of word (k / 4, m); the signed wire must hold q = u - 128 and the
    scale rounded to bf16, and the oracle's tile packer must give the same bytes."""
    for qw, sc in _parts(golden):
        K, M = 4 * qw.shape[0], qw.shape[1]
        words = qw.numpy().view(np.uint32)
        u = np.stack([(words >> (8 * j)) & 0xFF for j in range(4)], axis=1).reshape(K, M).T
        q_want = (u.astype(np.int32) - 128).astype(np.int8)
        s_want = torch.from_numpy(sc.numpy().astype(np.float32).T.copy()).to(torch.bfloat16)
        q, s_bits = wire_to_numpy(gptq_to_wire(qw, sc, 0), M, K, 128)
        assert np.array_equal(q, q_want)
        assert np.array_equal(s_bits, s_want.view(torch.int16).numpy().view(np.uint16))
        w = q.astype(np.float32) * np.repeat(from_bits(s_bits), 128, axis=1)
        assert np.array_equal(w, q_want.astype(np.float32) * np.repeat(s_want.float().numpy(), 128, axis=1))
        assert np.array_equal(gptq_to_wire(qw, sc, 0).numpy(), ops.pack_tile_wire(q, s_bits, 1, 1, "signed"))
        payload, _ = gptq_rows(qw, sc, 1)
        assert np.array_equal(payload.numpy(), u.astype(np.uint8))


def test_gptq_rejects_bad_tensors(golden):
    qw, sc = _parts(golden)[0]
    assert gptq_to_wire(qw, torch.cat([sc, sc])).numel() == 24 * (256 + 2 * 4)  # 4 groups of 64
    with pytest.raises(ValueError, match="group 16"):
        gptq_to_wire(qw, torch.cat([sc] * 8))  # 16 groups of 16 along K = 256
    with pytest.raises(ValueError, match="do not match"):
        gptq_to_wire(qw, sc[:, :5])
    with pytest.raises(ValueError, match="32-bit"):
        gptq_to_wire(qw.to(torch.int64), sc)
    with pytest.raises(ValueError, match="domain"):
        gptq_to_wire(qw, sc, 2)


def _checkpoint(cfg: Qwen3Config, n_layers: int, group: int, seed: int = 5):
    rng = np.random.default_rng(seed)

    def proj(name, M, K):
        words = rng.integers(0, 2 ** 32, size=(K // 4, M), dtype=np.uint64).astype(np.uint32)
        return {f"{name}.qweight": torch.from_numpy(words.view(np.int32).copy()),
                f"{name}.scales": torch.from_numpy((rng.random((K // group, M)) * 0.02 + 1e-3).astype(np.float16))}

    def vec(n):
        return torch.from_numpy((1 + 0.1 * rng.standard_normal(n)).astype(np.float32)).to(torch.bfloat16)

    t = {}
    for i in range(n_layers):
        L = f"model.layers.{i}"
        t[f"{L}.input_layernorm.weight"] = vec(cfg.D)
        t[f"{L}.post_attention_layernorm.weight"] = vec(cfg.D)
        t[f"{L}.self_attn.q_norm.weight"] = vec(cfg.HD)
        t[f"{L}.self_attn.k_norm.weight"] = vec(cfg.HD)
        t.update(proj(f"{L}.self_attn.q_proj", cfg.QD, cfg.D))
        t.update(proj(f"{L}.self_attn.k_proj", cfg.Hkv * cfg.HD, cfg.D))
        t.update(proj(f"{L}.self_attn.v_proj", cfg.Hkv * cfg.HD, cfg.D))
        t.update(proj(f"{L}.self_attn.o_proj", cfg.D, cfg.QD))
        t.update(proj(f"{L}.mlp.gate_proj", cfg.FF, cfg.D))
        t.update(proj(f"{L}.mlp.up_proj", cfg.FF, cfg.D))
        t.update(proj(f"{L}.mlp.down_proj", cfg.D, cfg.FF))
    t["model.norm.weight"] = vec(cfg.D)
    t["model.embed_tokens.weight"] = torch.from_numpy(
        (0.02 * rng.standard_normal((cfg.V, cfg.D))).astype(np.float32)).to(torch.bfloat16)
    return t


def test_load_qwen3_gptq_checkpoint():
    cfg = Qwen3Config(D=256, FF=512, Hq=4, Hkv=2, HD=64, V=1024, n_layers=2)
    t = _checkpoint(cfg, 2, 128)
    w = load_qwen3_gptq(t, cfg, device="cpu")
    assert w.group == 128 and len(w.layers) == 2 and w.lm_wire is None
    L, L0 = w.layers[1], "model.layers.1"
    for name, (M, K) in (("wqkv", (cfg.QKV, cfg.D)), ("wo", (cfg.D, cfg.QD)), ("wg", (cfg.FF, cfg.D)),
                         ("wu", (cfg.FF, cfg.D)), ("wd", (cfg.D, cfg.FF))):
        assert L[name].dtype == torch.uint8 and L[name].numel() == wire_nbytes(M, K, 128), name
    # Wqkv rows: the q, k, v projections in that order (qwen3_npu_int8.py:505-509)
    parts = [(t[f"{L0}.self_attn.{p}_proj.qweight"], t[f"{L0}.self_attn.{p}_proj.scales"]) for p in "qkv"]
    assert torch.equal(L["wqkv"], torch.cat([gptq_to_wire(*p) for p in parts]))
    assert torch.equal(L["qn"], t[f"{L0}.self_attn.q_norm.weight"])
    assert torch.equal(w.embed, t["model.embed_tokens.weight"])
    # the oracle's view of the loaded model
    host = w.to_numpy()
    assert host["layers"][0]["wd_q"].shape == (cfg.D, cfg.FF)


def test_load_qwen3_gptq_checks_shapes():
    cfg = Qwen3Config(D=256, FF=512, Hq=4, Hkv=2, HD=64, V=1024, n_layers=1)
    t = _checkpoint(cfg, 1, 128)
    bad = dict(t)
    bad["model.layers.0.mlp.up_proj.qweight"] = t["model.layers.0.mlp.up_proj.qweight"][:, :-4]
    with pytest.raises(ValueError, match="up_proj.qweight"):
        load_qwen3_gptq(bad, cfg, device="cpu")
    mixed = dict(t)
    mixed.update({k: v for k, v in _checkpoint(cfg, 1, 64, seed=6).items() if "down_proj" in k})
    with pytest.raises(ValueError, match="mixes group sizes"):
        load_qwen3_gptq(mixed, cfg, device="cpu")
    with pytest.raises(ValueError, match="embed_tokens"):
        load_qwen3_gptq(t, Qwen3Config(D=256, FF=512, Hq=4, Hkv=2, HD=64, V=2048, n_layers=1), device="cpu")
