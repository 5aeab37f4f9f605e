"""Composed CPU oracle of one Qwen3 decode step (TEST INFRASTRUCTURE ONLY).

The reference ships no whole-model CPU golden for Qwen3; its decode runtime
(iron/applications/qwen3_0.6b/qwen3_npu_int8.py:249-281, 594-621) chains one
fused QKV head, one decode attention and one fused (``fuse_o``) SwiGLU MLP per
layer, then the final RMSNorm and the lm_head GEMV, then a host argmax.  This
module composes the per-operator golden restatements of ``oracle.ops`` in
exactly that order:

* every int8 projection is the operator's ``reference()`` arithmetic, the exact
  dequantised matvec ``(q*s) @ x`` in float (``GEMVInt8.reference``,
  gemv_int8/op.py:173-178; ``SwiGLUMLPDataParallelOurs.reference``,
  swiglu_mlp_dp/op_ours.py:543-570); ``matvec="premul"`` selects instead the
  kernel-faithful golden ``gemv_int8/reference.py:25-40`` that rounds
  ``bf16(x*s)`` before the multiply-accumulate;
* QKV head: ``qkv_head_dp/reference.py:13-33`` with that matvec as its projection;
* K_t, V_t appended to the per-layer cache at position ``seq_pos``
  (qwen3_npu_int8.py:596-600, 608);
* attention: ``decode_attn/reference.py:26-38`` with ``seq_pos`` inclusive
  (``S_kv_eff = seq_pos + 1``, qwen3_npu_int8.py:609);
* MLP: the kernel-faithful golden ``swiglu_mlp_dp/test.py:79-91`` with
  ``a = bf16(Wo @ cx)`` (the ``fuse_o`` arm, swiglu_mlp_dp/reference.py:54-67);
* final RMSNorm: ``rms_norm/reference.py:8-17``; lm_head: bf16 tied embedding
  (``gemv/reference.py:9-11``) or the int8 RTN wire (premul GEMV);
* argmax over the logits (qwen3_npu_int8.py:615-621).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ops
from .bf16 import rnd


@dataclass
class Qwen3Shape:
    D: int = 1024
    FF: int = 3072
    Hq: int = 16
    Hkv: int = 8
    HD: int = 128
    V: int = 151936
    n_layers: int = 28
    eps: float = 1e-6
    theta: float = 1e6
    group: int = 32


class OracleQwen3:
    """Numpy Qwen3 decoder over int8 group-quantised weights.

    ``weights`` layout (numpy): per layer ``layers[i]`` a dict with ``norm1 (D)``,
    ``wqkv_q (QD+2KVD, D) int8``, ``wqkv_s (.., D/G) uint16``, ``qn``, ``kn`` (HD),
    ``wo_q (D, QD)``, ``wo_s``, ``norm2 (D)``, ``wg_q``/``wu_q`` (FF, D), ``wd_q`` (D, FF)
    and their ``_s`` scale bits; globals ``final_norm (D)``, ``embed (V, D)`` bf16
    values and optionally ``lm_q``/``lm_s`` (int8 lm_head).
    """

    def __init__(self, shape: Qwen3Shape, weights: dict, max_seq: int, int8_lm_head=False,
                 matvec: str = "exact", angles=None):
        self.s = shape
        self.w = weights
        self.max_seq = max_seq
        self.int8_lm_head = int8_lm_head
        if matvec not in ("exact", "premul"):
            raise ValueError("matvec must be 'exact' or 'premul'")
        self.mv = ops.gemv_int8_exact if matvec == "exact" else ops.gemv_int8_premul
        s = shape
        self.kv = np.zeros((s.n_layers, s.Hkv, max_seq, 2, s.HD), np.float32)
        # the RoPE row table is an input of the decode step (qwen3_npu_int8.py:603-604),
        # computed on the host; a caller may pass the exact table the device uses
        self.angles = (ops.rope_angle_table(max_seq, s.HD, s.theta) if angles is None
                       else np.asarray(angles, np.float32))

    def layer(self, i: int, x, pos: int):
        s, L = self.s, self.w["layers"][i]
        QD, KVD = s.Hq * s.HD, s.Hkv * s.HD
        qkv = ops.qkv_head(
            x, L["norm1"], lambda hn: self.mv(L["wqkv_q"], L["wqkv_s"], hn),
            L["qn"], L["kn"], self.angles[pos], s.D, s.HD, s.Hq, s.Hkv, s.eps)
        q = qkv[:QD].reshape(s.Hq, s.HD)
        self.kv[i, :, pos, 0] = qkv[QD:QD + KVD].reshape(s.Hkv, s.HD)
        self.kv[i, :, pos, 1] = qkv[QD + KVD:].reshape(s.Hkv, s.HD)
        ctx = ops.decode_attention(q, self.kv[i, :, :pos + 1, 0], self.kv[i, :, :pos + 1, 1],
                                   pos, s.HD, s.Hq, s.Hkv)
        a = rnd(self.mv(L["wo_q"], L["wo_s"], ctx.reshape(-1)))

        def mv(name):
            return lambda v: self.mv(L[name + "_q"], L[name + "_s"], v)

        return ops.swiglu_mlp_kernel_form(x, a, L["norm2"], mv("wg"), mv("wu"), mv("wd"), s.eps)

    def step(self, x, pos: int, n_layers: int | None = None):
        """One decode step for hidden state ``x`` (D,) at ``pos``.

        Returns ``(logits (V,) bf16 values, argmax token)``."""
        x = rnd(np.asarray(x, np.float32))
        for i in range(self.s.n_layers if n_layers is None else n_layers):
            x = self.layer(i, x, pos)
        xf = ops.rms_norm_ref(x.reshape(1, -1), self.w["final_norm"], weighted=True,
                              eps=self.s.eps).reshape(-1)
        if self.int8_lm_head:
            logits = rnd(self.mv(self.w["lm_q"], self.w["lm_s"], xf))
        else:
            logits = ops.gemv_bf16(self.w["embed"], xf)
        return logits, int(np.argmax(logits))

    def embed(self, token: int):
        return self.w["embed"][token]
