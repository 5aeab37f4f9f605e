"""IRON's Llama-3.2-1B decode runlist as an ``OperatorSequence`` of the B200 operators.

The reference builds one fused operator for a whole decode token out of its bf16
NPU operators (iron/applications/llama_3.2_1b/llama_npu.py:279-580) and drives it
per token (``llama_forward_pass_decode``, :1154-1198).  ``LlamaDecodeSequence``
builds the same runlist with the same operator constructors, buffer names, slices
and runtime parameters from ``iron_b200.operators``; the sequence runs it as one
CUDA graph.  Per layer:

  RMSNorm -> q / k / v GEMVs -> RoPE of q and k (one angle row) -> StridedCopy of the
  new key and value into the layer's caches at the ``cache_offset`` parameter ->
  Repeat of the KV heads to the query heads -> batched GEMV of the scores -> scale
  (ElementwiseMul) -> Softmax over the ``softmax_vector_size`` first positions ->
  one Transpose of the values per head (byte slices of one buffer) -> batched GEMV of
  the context -> O GEMV -> residual add -> RMSNorm -> gate and up GEMVs -> SiLU ->
  multiply -> down GEMV -> residual add;

then the final RMSNorm and the tied lm_head GEMV into ``logits``.  ``prompt_len`` is
the context capacity (the reference sizes its caches and score rows by it).

It is the operator-level showcase of the reference's Llama path; the fast batched
Llama decoder of this library is ``iron_b200.llama.LlamaB200``.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import call as abi, ptr
from .llama import LlamaWeights
from .operators import (GEMV, ElementwiseAdd, ElementwiseMul, Repeat, RMSNorm, RoPE, SiLU, Softmax,
                        StridedCopy, Transpose)
from .qwen3 import rope_angle_table
from .sequence import OperatorSequence


def decode_runlist(c, prompt_len: int, n_layers: int):
    """The operators, runlist and explicit buffer sizes of the fused decode operator
    (llama_npu.py:279-580) for config ``c`` (``LlamaConfig``), context capacity
    ``prompt_len`` and ``n_layers`` layers: (runlist, buffer_sizes, strided_copy_op)."""
    H, KV, HD, D, FF = c.Hq, c.Hkv, c.HD, c.D, c.FF
    gemv_attn_query_op = GEMV(M=H * HD, K=D, num_aie_columns=8, tile_size_input=4,
                              tile_size_output=HD // 2)
    gemv_attn_key_value_op = GEMV(M=KV * HD, K=D, num_aie_columns=8, tile_size_input=4,
                                  tile_size_output=HD // 2)
    rope_queries_op = RoPE(rows=H, cols=HD, angle_rows=1)
    rope_keys_op = RoPE(rows=KV, cols=HD, angle_rows=1)
    strided_copy_cache_op = StridedCopy(
        input_sizes=(KV, HD), input_strides=(HD, 1), input_offset=0,
        output_sizes=(1, KV, HD), output_strides=(0, prompt_len * HD, 1), output_offset=0,
        input_buffer_size=KV * HD, output_buffer_size=KV * prompt_len * HD, num_aie_channels=1,
        output_offset_parameter="cache_offset")
    gemv_attn_scores_op = GEMV(M=prompt_len, K=HD, num_aie_columns=8, tile_size_input=4,
                               tile_size_output=prompt_len // 8, num_batches=H)
    attn_scale_op = ElementwiseMul(size=H * prompt_len, tile_size=prompt_len // 8, num_aie_columns=8)
    softmax_op = Softmax(rows=H, cols=prompt_len, num_aie_columns=1, num_channels=1,
                         rtp_vector_size=prompt_len, vector_size_parameter="softmax_vector_size")
    transpose_values_op = Transpose(M=prompt_len, N=HD, num_aie_columns=2, num_channels=1, m=256, n=32, s=8)
    gemv_attn_context_op = GEMV(M=HD, K=prompt_len, num_aie_columns=8, tile_size_input=4,
                                tile_size_output=4, num_batches=H)
    gemv_attn_output_op = GEMV(M=D, K=H * HD, num_aie_columns=8, tile_size_input=4, tile_size_output=D // 8)
    rms_norm_op = RMSNorm(size=D, num_aie_columns=1, num_channels=1, tile_size=D, weighted=True)
    gemv_ffn_up_gate_op = GEMV(M=FF, K=D, num_aie_columns=8, tile_size_input=4, tile_size_output=FF // 8)
    gemv_ffn_down_op = GEMV(M=D, K=FF, num_aie_columns=8, tile_size_input=1, tile_size_output=D // 8)
    silu_ffn_op = SiLU(size=FF, tile_size=FF // 8, num_aie_columns=8)
    eltwise_mul_ffn_op = ElementwiseMul(size=FF, tile_size=FF // 8, num_aie_columns=8)
    residual_add_op = ElementwiseAdd(size=D, tile_size=D // 8)
    repeat_interleave_op = Repeat(rows=KV, cols=prompt_len * HD, repeat=H // KV, transfer_size=HD)
    gemv_out_head_op = GEMV(M=c.V, K=D, num_aie_columns=8, tile_size_input=4, tile_size_output=32)

    cache_buffer_size = KV * prompt_len * HD * 2
    vph = prompt_len * HD * 2  # bytes of one head's values
    values_buffer_size = H * vph
    runlist = []
    for i in range(n_layers):
        runlist += [
            (rms_norm_op, "x", f"W_norm1_{i}", "x_norm"),
            (gemv_attn_query_op, f"W_attn_query_{i}", "x_norm", "queries"),
            (gemv_attn_key_value_op, f"W_attn_key_{i}", "x_norm", "keys"),
            (gemv_attn_key_value_op, f"W_attn_value_{i}", "x_norm", "values"),
            (rope_queries_op, "queries", "rope_angles", "queries"),
            (rope_keys_op, "keys", "rope_angles", "keys"),
            (strided_copy_cache_op, "keys", f"keys_cache_{i}"),
            (strided_copy_cache_op, "values", f"values_cache_{i}"),
            (repeat_interleave_op, f"keys_cache_{i}", "attn_scores_keys"),
            (repeat_interleave_op, f"values_cache_{i}", "attn_scores_values"),
            (gemv_attn_scores_op, "attn_scores_keys", "queries", "attn_scores"),
            (attn_scale_op, "attn_scores", "attn_scale_factor", "attn_scores"),
            (softmax_op, "attn_scores", "attn_weights"),
        ]
        runlist += [(transpose_values_op, f"attn_scores_values[{h * vph}:{(h + 1) * vph}]",
                     f"attn_scores_values_transposed[{h * vph}:{(h + 1) * vph}]") for h in range(H)]
        runlist += [
            (gemv_attn_context_op, "attn_scores_values_transposed", "attn_weights", "attn_context"),
            (gemv_attn_output_op, f"W_attn_output_decode_{i}", "attn_context", "attn_output"),
            (residual_add_op, "x", "attn_output", "x"),
            (rms_norm_op, "x", f"W_norm2_{i}", "x_norm"),
            (gemv_ffn_up_gate_op, f"W_ffn_gate_{i}", "x_norm", "ffn_gate"),
            (gemv_ffn_up_gate_op, f"W_ffn_up_{i}", "x_norm", "ffn_up"),
            (silu_ffn_op, "ffn_gate", "ffn_gate"),
            (eltwise_mul_ffn_op, "ffn_gate", "ffn_up", "ffn_hidden"),
            (gemv_ffn_down_op, f"W_ffn_down_{i}", "ffn_hidden", "ffn_output"),
            (residual_add_op, "x", "ffn_output", "x"),
        ]
    runlist += [(rms_norm_op, "x", "W_final_norm", "x"), (gemv_out_head_op, "W_out_head", "x", "logits")]
    sizes = {**{f"keys_cache_{i}": cache_buffer_size for i in range(n_layers)},
             **{f"values_cache_{i}": cache_buffer_size for i in range(n_layers)},
             "attn_scores_values": values_buffer_size, "attn_scores_values_transposed": values_buffer_size}
    return runlist, sizes, strided_copy_cache_op


class LlamaDecodeSequence:
    """One stream of Llama decode through the reference's fused decode runlist.

    ``step(token, pos)`` writes the runtime parameters, the RoPE row of ``pos`` and the
    token's embedding into the sequence's buffers, calls the sequence and returns the
    logits (a device view of the ``logits`` buffer)."""

    def __init__(self, weights: LlamaWeights, prompt_len: int, n_layers: int | None = None):
        c = weights.cfg
        self.cfg, self.w, self.prompt_len = c, weights, prompt_len
        self.n_layers = len(weights.layers) if n_layers is None else n_layers
        runlist, sizes, self.strided_copy_cache_op = decode_runlist(c, prompt_len, self.n_layers)
        H, KV, HD = c.Hq, c.Hkv, c.HD
        self.fused_op = OperatorSequence("fused_op", runlist, input_args=["x", "rope_angles"],
                                         output_args=["logits"], buffer_sizes=sizes).compile()
        self.fused = self.fused_op.get_callable()
        f = self.fused
        QD, KVD = H * HD, KV * HD
        for i in range(self.n_layers):
            L = weights.layers[i]
            for name, t in ((f"W_norm1_{i}", L["norm1"]), (f"W_attn_query_{i}", L["wqkv"][:QD]),
                            (f"W_attn_key_{i}", L["wqkv"][QD:QD + KVD]),
                            (f"W_attn_value_{i}", L["wqkv"][QD + KVD:]),
                            (f"W_attn_output_decode_{i}", L["wo"]), (f"W_norm2_{i}", L["norm2"]),
                            (f"W_ffn_gate_{i}", L["wg"]), (f"W_ffn_up_{i}", L["wu"]), (f"W_ffn_down_{i}", L["wd"])):
                f.get_buffer(name).torch_view()[:] = t.flatten()
        f.get_buffer("attn_scale_factor").fill_(1.0 / math.sqrt(HD))
        f.get_buffer("W_final_norm").torch_view()[:] = weights.final_norm.flatten()
        f.get_buffer("W_out_head").torch_view()[:] = weights.embed.flatten()
        dev = f.arena.device
        self.angles = rope_angle_table(prompt_len, HD, c.theta).to(dev)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)

    def step(self, token: int, pos: int) -> torch.Tensor:
        """One decode token at position ``pos`` (llama_forward_pass_decode,
        llama_npu.py:1154-1198) -> the logits buffer (device view, V bf16 values).

        The runtime parameters are the new key's element offset in a KV head's cache
        row (``cache_offset`` = pos * head_dim) and the count of positions the softmax
        keeps (``softmax_vector_size`` = pos + 1, the context length: positions past it
        hold no keys yet).  The reference's driver writes a running sum of the context
        lengths there (llama_npu.py:1161-1167), whose meaning depends on its mask
        kernel, which is not part of the reference's sources."""
        c = self.cfg
        if not 0 <= pos < self.prompt_len:
            raise ValueError(f"position {pos} outside the context capacity {self.prompt_len}")
        f = self.fused
        f.params.write("cache_offset", pos * c.HD)
        f.params.write("softmax_vector_size", pos + 1)
        s = f.stream
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            f.params.sync(s)
            f.get_buffer("rope_angles").torch_view()[:c.HD] = self.angles[pos]
            self.tok.fill_(int(token))
            x = f.get_buffer("x").torch_view()
            abi("iron_embedding", ptr(self.w.embed), c.V, ptr(self.tok), 1, c.D, ptr(x), s.cuda_stream)
        f()
        err = self.strided_copy_cache_op.status()
        if err:
            raise _lib.IronError("StridedCopy: a cache write fell outside its buffer")
        return f.get_buffer("logits").torch_view()[:c.V]

    @property
    def kv(self):
        """Layer i's key and value caches as (KV, prompt_len, HD) device views."""
        c = self.cfg
        shape = (c.Hkv, self.prompt_len, c.HD)
        return [(self.fused.get_buffer(f"keys_cache_{i}").torch_view().view(shape),
                 self.fused.get_buffer(f"values_cache_{i}").torch_view().view(shape))
                for i in range(self.n_layers)]
