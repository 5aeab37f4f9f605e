"""Pin the numpy oracle against vectors produced by IRON's own golden code.

The fixtures come from ``tests/golden/make_golden.py`` (the reference's golden
functions, run unchanged).  Integer / byte outputs (quantiser, wire packer) must
match bit for bit.  Float outputs must match bit for bit on at least 99% of the
elements and within one bf16 ulp everywhere: the reference sums in float32 in
an order numpy cannot reproduce, so a rounding tie can land one ulp apart.
"""

import math

import numpy as np
import pytest

from oracle import ops
from oracle.bf16 import from_bits, rnd, round_bits


def assert_bf16_pinned(got, want_bits, min_exact=0.99):
    got_bits = round_bits(got).astype(np.int32).reshape(-1)
    want = np.asarray(want_bits, np.uint16).astype(np.int32).reshape(-1)
    exact = np.mean(got_bits == want)
    # bf16 patterns of same-signed values are ordered: one ulp = a step of 1.
    ulp = np.abs(got_bits - want)
    assert exact >= min_exact, f"only {exact:.4f} bit-exact"
    assert ulp.max() <= 1, f"max ulp distance {ulp.max()}"


def test_bf16_rounding_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 1000
    x[:4] = [np.inf, -np.inf, 0.0, -0.0]
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.uint16).numpy()
    assert np.array_equal(round_bits(x), want)


def test_gemv_int8_premul_g128(golden):
    g = golden("gemv_int8")
    y = ops.gemv_int8_premul(g["w_int8"], g["scales"], from_bits(g["x"]))
    assert_bf16_pinned(y, g["y"])


def test_gemv_int8_premul_g32(golden):
    g = golden("gemv_int8")
    y = ops.gemv_int8_premul(g["w_int8"], g["scales_g32"], from_bits(g["x"]))
    assert_bf16_pinned(y, g["y_g32"])


def test_tile_wire_packer_bit_exact(golden):
    g = golden("gemv_int8")
    w = g["w_int8"][:16]
    s = g["scales"][:16]
    signed = ops.pack_tile_wire(w, s, tile_m=4, cols=2, domain="signed")
    biased = ops.pack_tile_wire(w, s, tile_m=2, cols=1, domain="biased")
    assert np.array_equal(signed.view(np.uint16), g["wire_signed_c2_t4"])
    assert np.array_equal(biased.view(np.uint16), g["wire_biased_c1_t2"])
    q, sb = ops.unpack_tile_wire(biased, 16, 1024, 128, tile_m=2, domain="biased")
    assert np.array_equal(q, w) and np.array_equal(sb, s)


def test_rtn_quantiser_and_packer_bit_exact(golden):
    g = golden("rtn_pack")
    w = from_bits(g["w"]).reshape(64, 256)
    q, s = ops.quantize_rtn(w, group=128)
    assert np.array_equal(ops.pack_tile_wire(q, s, 4, 1, "signed").view(np.uint16), g["wire_signed_t4"])
    assert np.array_equal(ops.pack_tile_wire(q, s, 2, 2, "biased").view(np.uint16), g["wire_biased_c2_t2"])
    assert from_bits(s)[5, 0] == 1.0  # the all-zero group keeps s = 1


def test_rope_angle_table(golden):
    g = golden("rtn_pack")
    table = ops.rope_angle_table(1200, 128, 1e6)
    assert_bf16_pinned(table, g["angle_table"], min_exact=0.999)


def test_rms_norm(golden):
    g = golden("rms_norm")
    for xk, wk, yk in (("x_gen", "w_gen", "y_gen"), ("x", "w", "y")):
        y = ops.rms_norm_ref(from_bits(g[xk]), from_bits(g[wk]), weighted=True, eps=1e-6)
        assert_bf16_pinned(y, g[yk])


def test_rope(golden):
    g = golden("rope")
    y = ops.rope_two_halves(from_bits(g["x"]), from_bits(g["ang"]).reshape(-1))
    assert_bf16_pinned(y, g["y"], min_exact=1.0)


def test_qkv_head(golden):
    g = golden("qkv_head")
    D, HD, Hq, Hkv = (int(v) for v in g["dims"])
    W = from_bits(g["wqkv"]).reshape(-1, D).astype(np.float64)
    out = ops.qkv_head(from_bits(g["cur"]), from_bits(g["n_in"]), lambda hn: W @ hn,
                       from_bits(g["n_qn"]), from_bits(g["n_kn"]), from_bits(g["ang"]),
                       D, HD, Hq, Hkv, eps=1e-6)
    assert_bf16_pinned(out, g["out"])


@pytest.mark.parametrize("sp", [0, 1, 31, 32, 33, 100, 255])
def test_decode_attention(golden, sp):
    g = golden("decode_attn")
    Q, K, V = (from_bits(g[k]) for k in ("Q", "K", "V"))
    o = ops.decode_attention(Q, K, V, sp, 128, 16, 8)
    assert_bf16_pinned(o, g[f"O_{sp}"])
    if sp == 255:
        # decode_attn/reference.py:83-88 computes O_gen from the float32 V *before* it
        # is rounded into the bf16 KV buffer, so only a tolerance check applies to it.
        want = from_bits(g["O_gen"])
        assert np.abs(o - want).max() < 2e-2


@pytest.mark.parametrize("tag", ["causal", "noncausal"])
def test_decode_attention_batch_verify_mode(golden, tag):
    """DecodeAttention's multi-query verify mode (decode_attn/test_batch.py:31-46): 16
    new tokens after 192 cached positions.  The golden is float32: the oracle's bf16
    output must be its rounding -- bit-exact at >= 99.9 %, one ulp where a float32 sum
    rounds the other way, and more only for outputs so near zero that float32's
    absolute summation error (256 terms) spans several of their ulps.  A causal query
    m must equal the single-query oracle at position 192 + m."""
    g = golden("decode_attn_batch")
    N, H, KV, D, S, base = (int(v) for v in g["dims"])
    Q, K, V = (from_bits(g[k]) for k in ("Q", "K", "V"))
    o = ops.decode_attention_batch(Q, K, V, base, tag == "causal", D, H, KV)
    assert o.shape == (N, H, D)
    want = g[f"O_{tag}"]
    ulp = np.abs(round_bits(o).astype(np.int32) - round_bits(want).astype(np.int32))
    assert np.mean(ulp == 0) >= 0.999
    far = ulp > 1
    assert np.all(np.abs(o.astype(np.float64) - want)[far] <= 2e-5), np.abs(o - want)[far].max()
    if tag == "causal":
        for m in (0, 7, N - 1):
            assert np.array_equal(o[m], ops.decode_attention(Q[m], K, V, base + m, D, H, KV))


@pytest.mark.parametrize("S", [128, 96])
def test_mha_prefill(golden, S):
    """The prefill MHA golden (mha/reference.py:26-93: torch's causal SDPA on bf16
    tensors, GQA by repeat_interleave), a 128- and a 96-token prompt (the generator pads
    the latter to 128 with zeros).  Torch's bf16 kernel rounds intermediates the oracle
    keeps exact, so ~6 % of the outputs land one bf16 ulp away; none further."""
    g = golden("mha_prefill")
    Q, K, V = (from_bits(g[f"{k}_{S}"])[:, :S] for k in "QKV")
    o = ops.mha_prefill(Q, K, V, 64, 4, 2)
    assert_bf16_pinned(o, g[f"O_{S}"][:, :S], min_exact=0.90)
    assert not g[f"O_{S}"][:, S:].any()
    # position i sees only [0, i]: the first query row attends to the first key alone
    assert np.array_equal(o[:, 0], rnd(from_bits(g[f"V_{S}"])[[0, 0, 1, 1], 0]))


def test_swiglu_f32_goldens(golden):
    g = golden("swiglu")
    f = {k[4:]: from_bits(v) for k, v in g.items() if k.startswith("f32_")}
    y = ops.swiglu_mlp(f["cur"], f["a"], f["n_pf"], f["Wg"], f["Wu"], f["Wd"], 128, 384)
    assert_bf16_pinned(y, g["f32_nxt"])
    o = {k[3:]: from_bits(v) for k, v in g.items() if k.startswith("fo_")}
    y = ops.swiglu_mlp_fused_o(o["cur"], o["cx"], o["n_pf"], o["Wo"], o["Wg"], o["Wu"], o["Wd"],
                               128, 384, 256)
    assert_bf16_pinned(y, g["fo_nxt"])


def test_swiglu_kernel_form_and_silu(golden):
    g = golden("swiglu")
    assert_bf16_pinned(ops.silu_tanh_bf16(from_bits(g["silu_in"])), g["silu_tanh_out"], min_exact=0.995)

    def mv(name):
        q = (g[f"k_{name}_q"].astype(np.int16) - 128).astype(np.int8)
        return lambda v: ops.gemv_int8_premul(q, g[f"k_{name}_s"], v)

    y = ops.swiglu_mlp_kernel_form(from_bits(g["k_cur"]), from_bits(g["k_a"]), g["k_npf"],
                                   mv("wg"), mv("wu"), mv("wd"), eps=1e-6)
    assert_bf16_pinned(y, g["k_nxt"])


def test_elementwise(golden):
    g = golden("elementwise")
    a, b = from_bits(g["a"]), from_bits(g["b"])
    assert_bf16_pinned(ops.add_ref(a, b), g["add"], min_exact=1.0)
    assert_bf16_pinned(ops.mul_ref(a, b), g["mul"], min_exact=1.0)
    assert_bf16_pinned(ops.silu_ref(a), g["silu"])


def test_gemv_bf16(golden):
    g = golden("gemv_bf16")
    A = from_bits(g["A"]).reshape(256, 512)
    assert_bf16_pinned(ops.gemv_bf16(A, from_bits(g["B"])), g["C"])


def test_quantiser_error_bound():
    """|w - q*s| <= s/2 per group (qwen3_npu_int8.py:466-467)."""
    w = np.random.default_rng(1).standard_normal((32, 256)).astype(np.float32) * 0.02
    q, s = ops.quantize_rtn(w, group=32)
    deq = ops.dequant_f32(q, s)
    half = np.repeat(from_bits(s), 32, axis=1) / 2
    assert np.all(np.abs(w - deq) <= half * (1 + 2 ** -7))
    assert math.isclose(float(np.abs(q).max()), 127)


def test_llama_block_matches_reference_cpu_path(golden):
    """oracle/llama.py against llama_cpu.transformer_block_forward run unchanged (one
    decode token over a 5-position cache, bf16 weights, the harness's float32 RoPE
    table).  The new K (RMSNorm, projection, RoPE) and V rows and every attention op are
    pinned bit for bit.  torch's CPU bf16 rsqrt is not correctly rounded for about 0.5 %
    of inputs (measured: rsqrt(bf16 1.0546875) = 0.9765625, the correctly rounded value
    is 0.97265625), and the post-attention RMSNorm of this fixture meets such an input:
    its scale lands one bf16 ulp apart, which moves every later value by ~0.4 %.  The
    block output is therefore checked within the bf16 gate (rtol 2e-2, atol 1e-2)."""
    from oracle.llama import LlamaShape, OracleLlama
    g = golden("llama_block")
    D, H, KVH, HD, FF, T = (int(v) for v in g["dims"])
    f = from_bits
    L = {"norm1": f(g["norm1"]), "wqkv": np.concatenate([f(g["wq"]), f(g["wk"]), f(g["wv"])]),
         "wo": f(g["wo"]), "norm2": f(g["norm2"]), "wg": f(g["wg"]), "wu": f(g["wu"]), "wd": f(g["wd"])}
    shape = LlamaShape(D=D, FF=FF, Hq=H, Hkv=KVH, HD=HD, V=8, n_layers=1)
    orc = OracleLlama(shape, {"layers": [L]}, g["angles"].shape[0], angles=g["angles"])
    orc.kv[0, :, :T, 0] = f(g["kc"])
    orc.kv[0, :, :T, 1] = f(g["vc"])
    out = orc.layer(0, f(g["x"]), T)
    # the new K (RoPE) and V rows are single projections: pinned like the other goldens
    assert_bf16_pinned(orc.kv[0, :, T, 0], g["k_new"])
    assert_bf16_pinned(orc.kv[0, :, T, 1], g["v_new"])
    want = from_bits(g["out"])
    assert np.all(np.abs(out - want) <= 1e-2 + 2e-2 * np.abs(want))


def test_llama_runlist_data_movement(golden):
    """The oracle's RoPE (both methods, angle rows serving consecutive rows), strided copy
    (channel splits, runtime addends), repeat-interleave, softmax and transpose against
    the reference's own golden generators (tests/golden/make_golden.py ``seqops``)."""
    import json
    g = golden("seqops")
    for i in range(4):
        rows, cols, arows, method = (int(v) for v in g[f"rope{i}_dims"])
        x = from_bits(g[f"rope{i}_x"]).reshape(rows, cols)
        ang = np.repeat(from_bits(g[f"rope{i}_ang"]).reshape(arows, cols), rows // arows, axis=0)
        y = ops.rope_two_halves(x, ang) if method == 0 else ops.rope_interleaved(x, ang)
        assert_bf16_pinned(y, g[f"rope{i}_y"], min_exact=1.0)
    i = 0
    while f"sc{i}_in" in g:
        kw = json.loads(str(g[f"sc{i}_kw"]))
        src = g[f"sc{i}_in"]
        out = ops.strided_copy(src, np.zeros(kw["output_buffer_size"], np.uint16), kw["input_sizes"],
                               kw["input_strides"], kw["input_offset"], kw["output_sizes"], kw["output_strides"],
                               kw["output_offset"], kw.get("num_aie_channels", 1),
                               kw.get("input_offset_addend", 0), kw.get("output_offset_addend", 0))
        assert np.array_equal(out, g[f"sc{i}_out"]), f"strided copy case {i}"
        i += 1
    assert i == 8
    for i in range(3):
        rows, cols, r = (int(v) for v in g[f"rep{i}_dims"])
        assert np.array_equal(np.repeat(g[f"rep{i}_in"].reshape(rows, cols), r, axis=0),
                              g[f"rep{i}_out"].reshape(rows * r, cols))
    for i in range(2):
        x = from_bits(g[f"smx{i}_in"])
        assert_bf16_pinned(ops.softmax_rows(x), g[f"smx{i}_out"])
    for i in range(2):
        M, N, b = (int(v) for v in g[f"tr{i}_dims"])
        assert np.array_equal(g[f"tr{i}_in"].reshape(b, M, N).transpose(0, 2, 1), g[f"tr{i}_out"].reshape(b, N, M))
