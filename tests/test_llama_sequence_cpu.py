"""The Llama decode runlist (iron/applications/llama_3.2_1b/llama_npu.py:279-580) as
an ``OperatorSequence`` of the B200 operators, on the host: its buffer layout (sizes,
byte slices of the per-head value buffers, explicit cache sizes) and runtime
parameters, and the constructor checks the new operators keep from the reference's
(rope/op.py:36-54, strided_copy/op.py:53-65, softmax/op.py:37-45, transpose/op.py:49-83)."""

import pytest

from iron_b200.llama import LlamaConfig
from iron_b200.llama_sequence import decode_runlist
from iron_b200.operators import Repeat, RoPE, Softmax, StridedCopy, Transpose
from iron_b200.sequence import OperatorSequence


def test_llama_decode_runlist_layout():
    c = LlamaConfig.llama_3_2_1b()
    P, L = 256, 2
    runlist, sizes, sc = decode_runlist(c, P, L)
    # per layer: 13 entries, one Transpose per query head, 10 entries; then norm + head
    assert len(runlist) == L * (13 + c.Hq + 10) + 2
    seq = OperatorSequence("fused_op", runlist, input_args=["x", "rope_angles"], output_args=["logits"],
                           buffer_sizes=sizes)
    layout, total = seq.calculate_buffer_layout()
    vph = P * c.HD * 2
    assert layout["keys_cache_1"][1] == c.Hkv * P * c.HD * 2
    assert layout["attn_scores_values"][1] == c.Hq * vph
    base = layout["attn_scores_values_transposed"][0]
    for h in (0, 5, c.Hq - 1):
        off, n = layout[f"attn_scores_values_transposed[{h * vph}:{(h + 1) * vph}]"]
        assert (off, n) == (base + h * vph, vph)
    assert layout["logits"][1] == c.V * 2
    assert layout["W_attn_query_0"][1] == c.QD * c.D * 2
    assert total >= sum(n for k, (o, n) in layout.items() if "[" not in k)
    params = set()
    for op, *_ in runlist:
        params |= set(op.get_params_used())
    assert params == {"cache_offset", "softmax_vector_size"}
    assert sc.get_params_used() == ("cache_offset",)


def test_runlist_operator_checks():
    with pytest.raises(ValueError, match="multiple of 32"):
        RoPE(rows=8, cols=48)
    with pytest.raises(ValueError, match="angle_rows must divide rows"):
        RoPE(rows=8, cols=64, angle_rows=3)
    with pytest.raises(ValueError, match="method_type"):
        RoPE(rows=8, cols=64, method_type=2)
    with pytest.raises(ValueError, match="same length"):
        StridedCopy(input_sizes=[2, 4], input_strides=[4], input_offset=0, output_sizes=[8], output_strides=[1],
                    output_offset=0, input_buffer_size=8, output_buffer_size=8)
    with pytest.raises(ValueError, match="multiple of 16"):
        Softmax(rows=15, cols=64)
    with pytest.raises(ValueError, match="multiple of 256"):
        Transpose(M=100, N=64, num_aie_columns=2, num_channels=1, m=256, n=32, s=8)
    with pytest.raises(ValueError, match="exceeds N/n"):
        Transpose(M=512, N=64, num_aie_columns=4, num_channels=1, m=256, n=32, s=8)
    r = Repeat(rows=8, cols=64, repeat=4)
    assert [s.shape for s in r.get_arg_spec()] == [(8, 64), (32, 64)]
    t = Transpose(M=256, N=64, num_aie_columns=2, num_channels=1, m=256, n=32, s=8, num_batches=3)
    assert [s.shape for s in t.get_arg_spec()] == [(3, 256 * 64), (3, 64 * 256)]
    s = Softmax(rows=32, cols=256, vector_size_parameter="n")
    assert s.get_params_used() == ("n",) and s.get_arg_spec()[0].shape == (32 * 256,)
