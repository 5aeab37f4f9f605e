"""The sequence runtime on the GPU: ``OperatorSequence`` runlists and ``SwiGLUDecode``
run through ``get_callable()()`` -- the first call eager and captured, later calls
graph replays that read runtime parameters written with ``params.write`` + ``sync()``
(iron/common/sequence.py:596-626, 684-711) -- against the oracle."""

import numpy as np
import pytest
import torch

from iron_b200.operators import DecodeAttention, QKVHeadDataParallelOurs, SwiGLUMLPDataParallelOurs
from iron_b200.sequence import OperatorSequence, SwiGLUDecode
from oracle import ops
from oracle.bf16 import rnd

from helpers import assert_close, assert_ulps, dev_bf16, dev_u8, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("embedding_dim,hidden_dim", [(2048, 2048), (1024, 3584)])
def test_swiglu_decode_sequence(embedding_dim, hidden_dim):
    """SwiGLUDecode (swiglu_decode/op.py:13-70) as its test drives it
    (swiglu_decode/test.py): weights written into the persistent buffers in (M, K)
    layout, a warm-up call, a second call, then the stages checked.  Each stage is held
    to the oracle's bf16 form of that stage on the sequence's own inputs (the reference
    isolates its stages the same way: intermediate from the observed left_swished and
    right, out from the observed intermediate, to its rel 0.04 / abs 0.4)."""
    K, N = embedding_dim, hidden_dim
    g = torch.Generator().manual_seed(42)
    x = (torch.randn(K, generator=g) * 4).to(torch.bfloat16)
    wg = (torch.randn(N, K, generator=g) * 4).to(torch.bfloat16)
    wu = (torch.randn(N, K, generator=g) * 4).to(torch.bfloat16)
    wd = (torch.randn(K, N, generator=g) * 4).to(torch.bfloat16)
    op = SwiGLUDecode(embedding_dim=K, hidden_dim=N)
    op.compile()
    fc = op.get_callable()
    for name, t in (("w_gate", wg), ("w_up", wu), ("w_down", wd)):
        fc.get_buffer(name).torch_view()[:] = t.reshape(-1).cuda()
        fc.get_buffer(name).to("npu")
    fc.get_buffer("in").torch_view()[:] = x.cuda()
    fc()  # eager run + capture
    fc.get_buffer("in").torch_view()[:] = x.cuda()
    fc()  # graph replay
    for name in ("left", "right", "left_swished", "intermediate", "out"):
        fc.get_buffer(name).to("cpu")
    buf = {n: host(fc.get_buffer(n).torch_view()[:sz])
           for n, sz in (("left", N), ("right", N), ("left_swished", N), ("intermediate", N), ("out", K))}
    xn, wgn, wun, wdn = (host(t) for t in (x, wg, wu, wd))
    assert_ulps(buf["left"], ops.gemv_bf16(wgn, xn), max_ulp=1, frac_exact=0.95, what="left")
    assert_ulps(buf["right"], ops.gemv_bf16(wun, xn), max_ulp=1, frac_exact=0.95, what="right")
    # float32 x * sigmoid(x): CUDA's and numpy's exp differ in the last float32 bits, and
    # for large negative inputs both are tiny values (or zero) many ulps apart
    ls_want = ops.silu_ref(buf["left"])
    assert_close(buf["left_swished"], ls_want, what="left_swished")
    assert np.mean(buf["left_swished"] == ls_want) >= 0.99
    assert np.array_equal(buf["intermediate"], ops.mul_ref(buf["left_swished"], buf["right"]))
    assert_ulps(buf["out"], ops.gemv_bf16(wdn, buf["intermediate"]), max_ulp=1, frac_exact=0.9, what="out")
    # the reference test's own check of the output: against intermediate @ w_down in
    # float32 with rel 0.04 / abs 0.4 (swiglu_decode/test.py).  A float64 chain from x is
    # no gate at this scale (|out| ~ 1e7 from cancelling sums of bf16-rounded stages).
    ref_out = (torch.from_numpy(buf["intermediate"]).float() @ torch.from_numpy(wdn).float().T).numpy()
    assert np.all(np.abs(buf["out"] - ref_out) <= 0.4 + 0.04 * np.abs(ref_out))


def _layer_weights(D, FF, Hq, Hkv, HD, group, rng):
    QKV, QD = (Hq + 2 * Hkv) * HD, Hq * HD
    W = {}
    for name, (M, K) in (("wqkv", (QKV, D)), ("wo", (D, QD)), ("wg", (FF, D)), ("wu", (FF, D)), ("wd", (D, FF))):
        W[name] = ops.quantize_rtn(rnd(rng.standard_normal((M, K)).astype(np.float32) * 0.02), group)
    norms = {k: rnd(1 + 0.1 * rng.standard_normal(n).astype(np.float32))
             for k, n in (("n_in", D), ("n_qn", HD), ("n_kn", HD), ("n_pf", D))}
    return W, norms


def test_operator_sequence_decoder_layer_graph_replay():
    """A Qwen3 decoder layer as an OperatorSequence runlist in the order of
    qwen3_npu_int8.py:249-281 (fused QKV head -> decode attention -> SwiGLU MLP with the
    O projection fused), driven like Qwen3NPU.__call__ (:594-613): per token the host
    writes the input and the RoPE row into their buffers and the k_cache_offset and
    S_kv_eff parameters, syncs them, and calls.  Four tokens: the first call runs eagerly
    and captures, the rest replay the graph; each matches the oracle's layer on the same
    inputs, and the cache keeps every earlier position."""
    D, FF, Hq, Hkv, HD, S, G = 1024, 3072, 16, 8, 128, 64, 32
    QD = Hq * HD
    rng = np.random.default_rng(7)
    W, nm = _layer_weights(D, FF, Hq, Hkv, HD, G, rng)
    qkv = QKVHeadDataParallelOurs(D=D, HD=HD, Hq=Hq, Hkv=Hkv, max_seq=S, tile_size_input=4,
                                  kernel_source="mv_int8_signed.cc", kv_offset_parameter="k_cache_offset",
                                  group_size=G)
    attn = DecodeAttention(num_heads=Hq, num_kv_heads=Hkv, head_dim=HD, seq_len_kv=S, use_runtime_seq_len=True)
    mlp = SwiGLUMLPDataParallelOurs(D=D, FF=FF, num_aie_columns=8, epsilon=1e-6, QD=QD, fuse_o=True,
                                    kernel_source="mv_int8_signed.cc", group_size=G)
    runlist = [
        (qkv, "x", "n_in", "wqkv", "n_qn", "n_kn", "rope_angles", "q", "kv"),
        (attn, "q", "kv", "attn_out"),
        (mlp, "x", "attn_out", "n_pf", "wo", "wg", "wu", "wd", "gh", "a_scratch", "x_next"),
    ]
    seq = OperatorSequence("qwen3_layer", runlist, input_args=["x", "rope_angles"], output_args=["x_next"])
    seq.compile()
    fc = seq.get_callable()
    n, n_o, tsi_o, _ = mlp._wo_tiling()
    wires = {"wqkv": ops.pack_tile_wire(*W["wqkv"], 4, 8, "signed"),
             "wo": ops.pack_wo_tiled(*W["wo"], cols=n, tsi_o=tsi_o, n_o_tiles=n_o),
             "wg": ops.pack_tile_wire(*W["wg"], 12, n, "signed"),
             "wu": ops.pack_tile_wire(*W["wu"], 12, n, "signed"),
             "wd": ops.pack_tile_wire(*W["wd"], 4, n, "signed")}
    for name, wire in wires.items():
        fc.get_buffer(name).torch_view(torch.uint8)[:wire.size] = dev_u8(wire)
    for name in ("n_in", "n_qn", "n_kn", "n_pf"):
        fc.get_buffer(name).torch_view()[:nm[name].size] = dev_bf16(nm[name])
    angles = ops.rope_angle_table(S, HD, 1e6)
    mv = {k: (lambda v, k=k: ops.gemv_int8_exact(*W[k], v)) for k in W}
    Kc = np.zeros((Hkv, S, HD), np.float32)
    Vc = np.zeros((Hkv, S, HD), np.float32)
    for pos in range(4):
        x = rnd(rng.standard_normal(D).astype(np.float32))
        fc.get_buffer("x").torch_view()[:D] = dev_bf16(x)
        fc.get_buffer("rope_angles").torch_view()[:HD] = dev_bf16(angles[pos])
        fc.params.write("k_cache_offset", pos * 2 * HD)
        fc.params.write("S_kv_eff", pos + 1)
        fc.params.sync()
        fc()
        got = host(fc.get_buffer("x_next").torch_view()[:D])
        # the oracle layer on the same input
        r = ops.qkv_head(x, nm["n_in"], mv["wqkv"], nm["n_qn"], nm["n_kn"], angles[pos], D, HD, Hq, Hkv, 1e-6)
        Kc[:, pos], Vc[:, pos] = r[QD:QD + Hkv * HD].reshape(Hkv, HD), r[QD + Hkv * HD:].reshape(Hkv, HD)
        ctx = ops.decode_attention(r[:QD].reshape(Hq, HD), Kc[:, :pos + 1], Vc[:, :pos + 1], pos, HD, Hq, Hkv)
        want = ops.swiglu_mlp_kernel_form(x, rnd(mv["wo"](ctx.reshape(-1))), nm["n_pf"], mv["wg"], mv["wu"],
                                          mv["wd"], 1e-6)
        assert_close(got, want, what=f"token {pos}")
        assert np.mean(got == want) >= 0.95, f"token {pos}: {np.mean(got == want):.3f} bit-exact"
        kv = host(fc.get_buffer("kv").torch_view()[:Hkv * S * 2 * HD]).reshape(Hkv, S, 2, HD)
        assert_close(kv[:, :pos + 1, 0], Kc[:, :pos + 1], what=f"K cache after token {pos}")
        assert_close(kv[:, :pos + 1, 1], Vc[:, :pos + 1], what=f"V cache after token {pos}")
        assert not kv[:, pos + 1:].any(), "a position past the token was written"
    assert fc._graph is not None  # calls after the first replayed the captured graph
