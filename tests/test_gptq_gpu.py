"""A GPTQ int8 checkpoint (iron_b200/gptq.py) decoded on the GPU against the CPU oracle.

The checkpoint holds the reference's tensors (qwen3_npu_int8.py:152-178): N(0, 0.02)
masters quantised GPTQ-style (symmetric, zero-point 128, fp16 scale = absmax / 127
per group of 128) and packed four bytes to a 32-bit word; the 2-layer model has the
Qwen3-0.6B layer shape and vocabulary.  The loaded group-128 wires run the one-launch
step kernel; the oracle reads the same wires."""

import numpy as np
import pytest
import torch

from iron_b200.gptq import load_qwen3_gptq
from iron_b200.qwen3 import Qwen3B200, Qwen3Config
from oracle.qwen3 import OracleQwen3, Qwen3Shape

from helpers import assert_close, host

pytestmark = pytest.mark.gpu


def _gptq(g, M, K, G=128):
    w = (torch.randn(M, K, generator=g) * 0.02).reshape(M, K // G, G)
    s = (w.abs().amax(dim=2) / 127).to(torch.float16)
    q = torch.round(w / s.float()[:, :, None]).clamp_(-127, 127).reshape(M, K)
    u = (q + 128).to(torch.int64)                                        # (M, K) bytes q + 128
    words = (u.reshape(M, K // 4, 4) << torch.tensor([0, 8, 16, 24])).sum(dim=2)
    words = torch.from_numpy(words.t().contiguous().numpy().astype(np.uint32).view(np.int32))
    return words, s.t().contiguous()


def test_gptq_checkpoint_decodes_like_oracle():
    cfg = Qwen3Config.qwen3_0_6b()
    g = torch.Generator().manual_seed(4)
    t = {}
    for i in range(2):
        L = f"model.layers.{i}"
        for name, (M, K) in (("self_attn.q_proj", (cfg.QD, cfg.D)), ("self_attn.k_proj", (cfg.Hkv * cfg.HD, cfg.D)),
                             ("self_attn.v_proj", (cfg.Hkv * cfg.HD, cfg.D)), ("self_attn.o_proj", (cfg.D, cfg.QD)),
                             ("mlp.gate_proj", (cfg.FF, cfg.D)), ("mlp.up_proj", (cfg.FF, cfg.D)),
                             ("mlp.down_proj", (cfg.D, cfg.FF))):
            t[f"{L}.{name}.qweight"], t[f"{L}.{name}.scales"] = _gptq(g, M, K)
        for name, n in (("input_layernorm", cfg.D), ("post_attention_layernorm", cfg.D),
                        ("self_attn.q_norm", cfg.HD), ("self_attn.k_norm", cfg.HD)):
            t[f"{L}.{name}.weight"] = 1 + 0.1 * torch.randn(n, generator=g)
    t["model.norm.weight"] = 1 + 0.1 * torch.randn(cfg.D, generator=g)
    t["model.embed_tokens.weight"] = (torch.randn(cfg.V, cfg.D, generator=g) * 0.02).to(torch.bfloat16)
    w = load_qwen3_gptq(t, cfg, device="cuda", n_layers=2)
    assert w.group == 128
    S = 32
    dec = Qwen3B200(w, max_seq=S, keep_logits=True)
    orc = OracleQwen3(Qwen3Shape(n_layers=2, group=128), w.to_numpy(), S, angles=host(dec.angles))
    tok = 11
    for pos in range(2):
        got = int(dec.step_tokens([tok], pos)[0])
        logits, want = orc.step(orc.embed(tok), pos)
        assert_close(host(dec.logits[0]), logits, what=f"logits pos {pos}")
        assert got == want
        tok = want
