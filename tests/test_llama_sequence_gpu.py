"""The Llama decode runlist's operators and the runlist itself on the GPU.

Operators (through ``get_callable()``): RoPE (two halves and interleaved, angle rows
serving consecutive rows, in place), StridedCopy (channel splits, runtime offset
parameters), Repeat, Softmax (with and without the runtime vector size) and Transpose,
against the reference's own golden generators (tests/golden/seqops.npz): data movement
bit for bit, RoPE bit for bit (float32, no fused multiply-add, one rounding), softmax
within one bf16 ulp.

The runlist (``LlamaDecodeSequence``, llama_npu.py:279-580 driven as
llama_forward_pass_decode, :1154-1198): a 2-layer Llama-3.2-1B-shaped model from an
empty 256-position cache, against the oracle's bf16 op chain (``OracleLlama``, the
reference's llama_cpu.py, with the RMSNorm operator's golden form the runlist's
``RMSNorm`` operators compute), teacher-forced with the sequence's tokens and caches."""

import json

import numpy as np
import pytest
import torch

from iron_b200.llama import LlamaConfig, LlamaWeights
from iron_b200.llama_sequence import LlamaDecodeSequence
from iron_b200.operators import Repeat, RoPE, Softmax, StridedCopy, Transpose
from oracle import ops
from oracle.bf16 import from_bits
from oracle.llama import LlamaShape, OracleLlama

from helpers import assert_close, assert_ulps, bits, host, logit_gate

pytestmark = pytest.mark.gpu


def _u16(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).copy()).view(torch.bfloat16).cuda()


def test_rope_rows_golden(golden):
    g = golden("seqops")
    for i in range(4):
        rows, cols, arows, method = (int(v) for v in g[f"rope{i}_dims"])
        op = RoPE(rows=rows, cols=cols, angle_rows=arows, method_type=method)
        x, ang = _u16(g[f"rope{i}_x"]), _u16(g[f"rope{i}_ang"])
        y = torch.zeros_like(x)
        call = op.get_callable()
        call(x, ang, y)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y).reshape(-1), g[f"rope{i}_y"].reshape(-1)), f"rope case {i}"
        call(x, ang, x)  # in place
        torch.cuda.synchronize()
        assert torch.equal(x, y)


def test_strided_copy_golden(golden):
    g = golden("seqops")
    for i in range(8):
        kw = json.loads(str(g[f"sc{i}_kw"]))
        ia, oa = kw.pop("input_offset_addend", 0), kw.pop("output_offset_addend", 0)
        op = StridedCopy(**kw, input_offset_parameter="in_off" if ia else None,
                         output_offset_parameter="out_off" if oa else None)
        call = op.get_callable()
        if call.params is not None:
            if ia:
                call.params.write("in_off", ia)
            if oa:
                call.params.write("out_off", oa)
            call.params.sync()
        src = _u16(g[f"sc{i}_in"])
        dst = torch.zeros(kw["output_buffer_size"], dtype=torch.bfloat16, device="cuda")
        call(src, dst)
        torch.cuda.synchronize()
        assert np.array_equal(bits(dst), g[f"sc{i}_out"]), f"strided copy case {i}"
        assert op.status() == 0
    # an addend that moves the pattern past the buffer's end: the elements outside are
    # skipped (the others land) and the error word says so
    op = StridedCopy(input_sizes=[64], input_strides=[1], input_offset=0, output_sizes=[64], output_strides=[1],
                     output_offset=0, input_buffer_size=64, output_buffer_size=96, output_offset_parameter="o")
    call = op.get_callable()
    call.params.write("o", 48)
    call.params.sync()
    src = torch.arange(64, dtype=torch.float32, device="cuda").to(torch.bfloat16)
    dst = torch.zeros(96, dtype=torch.bfloat16, device="cuda")
    call(src, dst)
    torch.cuda.synchronize()
    assert torch.equal(dst[48:], src[:48]) and op.status() == 1 and op.status() == 0


def test_repeat_softmax_transpose_golden(golden):
    g = golden("seqops")
    for i in range(3):
        rows, cols, r = (int(v) for v in g[f"rep{i}_dims"])
        x = _u16(g[f"rep{i}_in"]).view(rows, cols)
        y = torch.zeros(rows * r, cols, dtype=torch.bfloat16, device="cuda")
        Repeat(rows=rows, cols=cols, repeat=r).get_callable()(x, y)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y).reshape(-1), g[f"rep{i}_out"].reshape(-1))
    for i, (rows, cols) in enumerate(((32, 256), (16, 1024))):
        x = _u16(g[f"smx{i}_in"]).reshape(-1)
        y = torch.zeros_like(x)
        Softmax(rows=rows, cols=cols).get_callable()(x, y)
        torch.cuda.synchronize()
        assert_ulps(host(y), from_bits(g[f"smx{i}_out"]).reshape(-1), max_ulp=1, frac_exact=0.97,
                    what=f"softmax {rows}x{cols}")
        # the runtime vector size: the first n entries of each row, the rest zero
        op = Softmax(rows=rows, cols=cols, vector_size_parameter="n")
        call = op.get_callable()
        for n in (1, 77, cols):
            call.params.write("n", n)
            call.params.sync()
            call(x, y)
            torch.cuda.synchronize()
            want = ops.softmax_rows(from_bits(g[f"smx{i}_in"]).reshape(rows, cols), n)
            assert_ulps(host(y), want.reshape(-1), max_ulp=1, frac_exact=0.97, what=f"masked softmax n={n}")
            assert not host(y).reshape(rows, cols)[:, n:].any()
    for i in range(2):
        M, N, b = (int(v) for v in g[f"tr{i}_dims"])
        x = _u16(g[f"tr{i}_in"]).reshape(-1)
        y = torch.zeros_like(x)
        Transpose(M=M, N=N, num_aie_columns=2, num_channels=1, m=64, n=32, s=8,
                  num_batches=b).get_callable()(x.view(b, -1) if b > 1 else x, y.view(b, -1) if b > 1 else y)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y).reshape(-1), g[f"tr{i}_out"].reshape(-1))


def test_llama_decode_sequence_matches_oracle():
    """Six tokens from position 0 of an empty cache.  Each step: the logits within the
    whole-model gate of the oracle's bf16 chain; the greedy token equal or a near-tie
    within the step's measured noise; the first layer's new key and value rows within
    one bf16 ulp of the oracle's, the second's within the bf16 gate.  The oracle then continues from the sequence's caches.
    The second and later calls replay the captured graph with new runtime parameters."""
    cfg = LlamaConfig.llama_3_2_1b()
    w = LlamaWeights.synthetic(cfg, seed=5, n_layers=2)
    P = 256
    seq = LlamaDecodeSequence(w, prompt_len=P)
    orc = OracleLlama(LlamaShape(n_layers=2), w.to_numpy(), P, angles=host(seq.angles), norm_form="golden")
    tok, agree = 1234, 0
    for pos in range(6):
        logits = host(seq.step(tok, pos))
        want, want_tok = orc.step(tok, pos)
        logit_gate(logits, want, f"step {pos}", max_outside=0.05)
        got_tok = int(np.argmax(logits))
        if got_tok == want_tok:
            agree += 1
        else:
            noise = float(np.abs(logits - want).max())
            assert abs(want[got_tok] - want[want_tok]) <= noise, f"step {pos}: not a near-tie"
        for i, (k, v) in enumerate(seq.kv):
            for name, got, want in (("key", k, orc.kv[i, :, pos, 0]), ("value", v, orc.kv[i, :, pos, 1])):
                what = f"layer {i} {name} row {pos}"
                if i == 0:  # float32 against float64 sums: a rounding flip at most
                    assert_ulps(host(got[:, pos]), want, max_ulp=1, frac_exact=0.9, what=what)
                else:  # one flip in the layer's input can move the RMSNorm scale by an ulp
                    assert_close(host(got[:, pos]), want, what=what)
            assert not host(k[:, pos + 1:]).any()  # positions past the context stay empty
            orc.kv[i, :, :P, 0] = host(k)
            orc.kv[i, :, :P, 1] = host(v)
        tok = got_tok
    assert agree >= 5
