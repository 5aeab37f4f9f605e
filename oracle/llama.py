"""CPU oracle of Llama-3.2-1B-shaped bf16 decode (TEST INFRASTRUCTURE ONLY).

Restates the reference's CPU Llama path, iron/applications/llama_3.2_1b/
llama_cpu.py, for single-token decode of one stream, with every torch bf16 op's
rounding applied by ``rnd``:

* ``rms_norm_forward`` (llama_cpu.py:41-46): ``x * rsqrt(mean(x^2) + eps)`` then
  ``* weight``, eps = 1e-5 -- each torch op on the bf16 tensors rounds;
* ``grouped_query_attention_forward`` (:49-148): q/k/v projections (bf16 linear:
  float accumulation, one rounding), ``rope_forward`` (:14-38) on q and k with the
  interleaved ``[cos, sin]`` angle row of the position (angles as
  ``llama_inference_harness.compute_rope_angles``, :109-123, theta 5e5; a caller may
  pass the exact table the device uses), the new K/V
  appended to the cache, GQA softmax attention (``repeat_interleave`` of the KV
  heads), the output projection;
* ``transformer_block_forward`` (:170-218): x + attention, post-attention norm,
  ``swiglu_ffn_forward`` (:151-167, SiLU = ``torch.nn.functional.silu``), x + FFN;
* ``llama_forward_pass`` (:221-289): embedding, blocks, final norm, tied lm_head.

Float64 accumulation stands for torch's float32 accumulation inside each bf16 op
(the two round to the same bf16 value except at rare ties); numpy's exp/sqrt stand
for torch's.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import ops
from .bf16 import rnd

F32 = np.float32


@dataclass(frozen=True)
class LlamaShape:
    D: int = 2048
    FF: int = 8192
    Hq: int = 32
    Hkv: int = 8
    HD: int = 64
    V: int = 128256
    n_layers: int = 16
    eps: float = 1e-5
    theta: float = 5e5


def rms_norm(x, w, eps):
    """llama_cpu.py:41-46 on bf16 tensors."""
    x = np.asarray(x, F32)
    var = rnd((rnd(x * x).astype(np.float64).mean(axis=-1, keepdims=True)).astype(F32))
    r = rnd((1.0 / np.sqrt(rnd(var + F32(eps)).astype(np.float64))).astype(F32))
    return rnd(np.asarray(w, F32) * rnd(x * r))


def linear(w, x):
    """torch.nn.functional.linear on bf16: float accumulation, one bf16 rounding."""
    return rnd((np.asarray(w, np.float64) @ np.asarray(x, np.float64)).astype(F32))


def rope(x, ang):
    """llama_cpu.py:14-38: ``[x1*c - x2*s, x1*s + x2*c]``.  The reference's angle table is
    float32, so the bf16 x times the float32 cos/sin runs in float32 and rounds once
    when stored into the bf16 result: ``ops.rope_two_halves`` (given the same table)."""
    return ops.rope_two_halves(x, ang)


class OracleLlama:
    """One stream of Llama decode over bf16 weights.

    ``weights``: per layer ``layers[i]`` with ``norm1 (D)``, ``wqkv ((Hq+2Hkv)*HD, D)``
    (the q, k, v projections stacked), ``wo (D, Hq*HD)``, ``norm2 (D)``, ``wg``, ``wu``
    ``(FF, D)``, ``wd (D, FF)``; ``final_norm (D)``, ``embed (V, D)`` (tied lm_head).
    All bf16 values as float32."""

    def __init__(self, shape: LlamaShape, weights: dict, max_seq: int, angles=None,
                 exact_attention: bool = False, norm_form: str = "llama"):
        """``exact_attention``: softmax and context in float64, rounded once -- the
        quantity the reference's bf16 op chain approximates (its scores and
        probabilities are rounded to bf16); the float32 flash attention of the GPU
        path is checked against this form.  ``norm_form``: "llama" is
        ``rms_norm_forward`` of llama_cpu.py:41-46; "golden" is the RMSNorm operator's
        golden (rms_norm/reference.py:8-17, ``ops.rms_norm_ref``), the form of the
        ``RMSNorm`` operators in the NPU decode runlist (llama_npu.py:385-392)."""
        if norm_form not in ("llama", "golden"):
            raise ValueError(f"norm_form {norm_form!r}")
        self.s, self.w, self.exact_attention = shape, weights, exact_attention
        self.norm = rms_norm if norm_form == "llama" else (
            lambda x, w, eps: ops.rms_norm_ref(x, w, weighted=True, eps=eps))
        self.kv = np.zeros((shape.n_layers, shape.Hkv, max_seq, 2, shape.HD), F32)
        self.angles = (ops.rope_angle_table(max_seq, shape.HD, shape.theta) if angles is None
                       else np.asarray(angles, F32))

    def layer(self, i: int, x, pos: int):
        s, L = self.s, self.w["layers"][i]
        QD, KVD = s.Hq * s.HD, s.Hkv * s.HD
        h = self.norm(x, L["norm1"], s.eps)
        qkv = linear(L["wqkv"], h)
        q = rope(qkv[:QD].reshape(s.Hq, s.HD), self.angles[pos])
        k = rope(qkv[QD:QD + KVD].reshape(s.Hkv, s.HD), self.angles[pos])
        self.kv[i, :, pos, 0] = k
        self.kv[i, :, pos, 1] = qkv[QD + KVD:].reshape(s.Hkv, s.HD)
        # llama_cpu.py:119-141 on bf16 tensors: scores = bf16(q @ K^T), bf16(/ sqrt(d)),
        # p = bf16(softmax) (float32 inside), context = bf16(p @ V)
        ctx = np.zeros((s.Hq, s.HD), F32)
        for hh in range(s.Hq):
            kvh = hh * s.Hkv // s.Hq  # repeat_interleave: query head hh reads KV head hh // group
            K = self.kv[i, kvh, :pos + 1, 0].astype(np.float64)
            V = self.kv[i, kvh, :pos + 1, 1].astype(np.float64)
            if self.exact_attention:
                sc = (K @ q[hh].astype(np.float64)) / math.sqrt(s.HD)
                e = np.exp(sc - sc.max())
                ctx[hh] = rnd(((e @ V) / e.sum()).astype(F32))
                continue
            sc = rnd((K @ q[hh].astype(np.float64)).astype(F32))
            sc = rnd((sc / F32(math.sqrt(s.HD))).astype(F32))
            e = np.exp(sc.astype(np.float64) - float(sc.max()))
            p = rnd((e / e.sum()).astype(F32))
            ctx[hh] = rnd((p.astype(np.float64) @ V).astype(F32))
        a = linear(L["wo"], ctx.reshape(-1))
        x1 = ops.add_ref(x, a)
        h2 = self.norm(x1, L["norm2"], s.eps)
        g = linear(L["wg"], h2)
        u = linear(L["wu"], h2)
        gh = ops.mul_ref(ops.silu_ref(g), u)
        return ops.add_ref(x1, linear(L["wd"], gh))

    def step(self, token: int, pos: int):
        """Embedding of ``token`` at ``pos`` through every layer -> (logits, argmax)."""
        x = np.asarray(self.w["embed"][token], F32)
        for i in range(self.s.n_layers):
            x = self.layer(i, x, pos)
        xf = self.norm(x, self.w["final_norm"], self.s.eps)
        logits = linear(self.w["embed"], xf)
        return logits, int(np.argmax(logits))
