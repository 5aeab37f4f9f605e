"""GPU parity of RMSNorm, elementwise ops, the fused QKV head, decode attention and the
fused SwiGLU MLP block, each through its IRON-compatible operator class."""

import numpy as np
import pytest
import torch

from iron_b200.operators import (DecodeAttention, ElementwiseAdd, ElementwiseMul, QKVHeadDataParallelOurs,
                                 RMSNorm, SiLU, SwiGLUMLPDataParallel, SwiGLUMLPDataParallelOurs)
from iron_b200.test_utils import verify_buffer
from oracle import ops
from oracle.bf16 import from_bits, rnd, round_bits

from helpers import assert_close, assert_ulps, dev_bf16, dev_u8, host

pytestmark = pytest.mark.gpu


def _out(n):
    return torch.zeros(n, dtype=torch.bfloat16, device="cuda")


def test_rmsnorm_against_reference_golden(golden):
    g = golden("rms_norm")
    for xk, wk, yk, rows in (("x_gen", "w_gen", "y_gen", 4), ("x", "w", "y", 3)):
        x2d = dev_bf16(g[xk]).reshape(rows, 1024)
        # golden arithmetic (every torch op rounds to bf16): the golden's bits
        op = RMSNorm(size=rows * 1024, num_aie_columns=1, num_channels=1, tile_size=1024, weighted=True,
                     epsilon=1e-6)
        y = _out(rows * 1024)
        op.get_callable()(x2d, dev_bf16(g[wk]), y.reshape(rows, 1024))
        torch.cuda.synchronize()
        assert_ulps(host(y), from_bits(g[yk]), max_ulp=1, frac_exact=0.99, what="rmsnorm golden form")
        # kernel arithmetic (float32, one rounding, rms_norm.cc): within the reference
        # test's tolerance of the golden (rms_norm/test.py: rel 0.04, abs 1e-6)
        op = RMSNorm(size=rows * 1024, num_aie_columns=1, num_channels=1, tile_size=1024, weighted=True,
                     epsilon=1e-6, golden_rounding=False)
        op.get_callable()(x2d, dev_bf16(g[wk]), y.reshape(rows, 1024))
        torch.cuda.synchronize()
        assert not verify_buffer(host(y), "y", from_bits(g[yk]), rel_tol=0.04, abs_tol=1e-6)
        want = ops.rms_norm_f32(from_bits(g[xk]).reshape(rows, 1024), from_bits(g[wk]), 1e-6)
        assert_ulps(host(y), want, max_ulp=1, frac_exact=0.99, what="rmsnorm f32 form")


def test_rmsnorm_llama_form_matches_oracle():
    """iron_rmsnorm mode 2 (llama_cpu.py:41-46 on bf16 tensors) against oracle.llama.rms_norm."""
    from iron_b200 import _lib
    from oracle.llama import rms_norm as llama_norm
    torch.manual_seed(21)
    rows, cols = 7, 2048
    x = (torch.randn(rows, cols, device="cuda") * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(cols, device="cuda")).to(torch.bfloat16)
    y = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_rmsnorm", x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, cols, 1e-5, 2, _lib.stream_ptr())
    torch.cuda.synchronize()
    assert_ulps(host(y), llama_norm(host(x), host(w), 1e-5), max_ulp=1, frac_exact=0.99, what="llama norm")


def test_elementwise_against_reference_golden(golden):
    g = golden("elementwise")
    a, b = dev_bf16(g["a"]), dev_bf16(g["b"])
    for cls, key in ((ElementwiseAdd, "add"), (ElementwiseMul, "mul")):
        c = _out(2048)
        cls(size=2048, tile_size=256).get_callable()(a, b, c)
        torch.cuda.synchronize()
        assert np.array_equal(host(c), from_bits(g[key])), key
    y = _out(2048)
    SiLU(size=2048, num_aie_columns=8, tile_size=256).get_callable()(a, y)
    torch.cuda.synchronize()
    assert_ulps(host(y), from_bits(g["silu"]), max_ulp=1, frac_exact=0.99, what="silu")


def test_silu_tanh_form_against_kernel_golden(golden):
    g = golden("swiglu")
    x = dev_bf16(g["silu_in"])
    y = _out(x.numel())
    SiLU(size=x.numel(), num_aie_columns=8, tile_size=512, tanh_form=True).get_callable()(x, y)
    torch.cuda.synchronize()
    assert_ulps(host(y), from_bits(g["silu_tanh_out"]), max_ulp=1, frac_exact=0.99, what="silu tanh")


def _qkv_case(D, Hq, Hkv, HD, group, tile_m, max_seq, pos, seed=0):
    rng = np.random.default_rng(seed)
    QKV = (Hq + 2 * Hkv) * HD
    w = rng.standard_normal((QKV, D)).astype(np.float32) * 0.02
    q8, s8 = ops.quantize_rtn(rnd(w), group)
    cur = rnd(rng.standard_normal(D).astype(np.float32))
    n_in = rnd(1 + 0.1 * rng.standard_normal(D).astype(np.float32))
    n_qn = rnd(1 + 0.1 * rng.standard_normal(HD).astype(np.float32))
    n_kn = rnd(1 + 0.1 * rng.standard_normal(HD).astype(np.float32))
    ang = ops.rope_angle_table(max_seq, HD, 1e6)[pos]
    return q8, s8, cur, n_in, n_qn, n_kn, ang


@pytest.mark.parametrize("group,tile_m,pos", [(128, 4, 0), (32, 1, 77), (128, 4, 511)])
def test_qkv_head_op(group, tile_m, pos):
    """QKVHeadDataParallelOurs vs qkv_head_dp/reference.py:13-33 with the premul int8 matvec;
    K_t, V_t land at k_cache_offset = pos*2*HD of every head region; nothing else changes."""
    D, Hq, Hkv, HD, S = 1024, 16, 8, 128, 512
    q8, s8, cur, n_in, n_qn, n_kn, ang = _qkv_case(D, Hq, Hkv, HD, group, tile_m, S, pos)
    op = QKVHeadDataParallelOurs(D=D, HD=HD, Hq=Hq, Hkv=Hkv, max_seq=S, tile_size_input=tile_m,
                                 kernel_source="mv_int8_signed.cc", kv_offset_parameter="k_cache_offset",
                                 group_size=group)
    call = op.get_callable()
    call.params.write("k_cache_offset", pos * 2 * HD)
    call.params.sync()
    wire = dev_u8(ops.pack_tile_wire(q8, s8, tile_m, 8, "signed")).view(torch.bfloat16)
    q = _out(Hq * HD)
    kv = torch.full((Hkv * S * HD * 2,), 7.0, dtype=torch.bfloat16, device="cuda")
    call(dev_bf16(cur), dev_bf16(n_in), wire, dev_bf16(n_qn), dev_bf16(n_kn), dev_bf16(ang), q, kv)
    torch.cuda.synchronize()
    want = ops.qkv_head(cur, n_in, lambda hn: ops.gemv_int8_premul(q8, s8, hn), n_qn, n_kn, ang,
                        D, HD, Hq, Hkv, 1e-6)
    QD, KVD = Hq * HD, Hkv * HD
    assert_close(host(q), want[:QD], what="q")
    kvh = host(kv).reshape(Hkv, S, 2, HD)
    assert_close(kvh[:, pos, 0], want[QD:QD + KVD].reshape(Hkv, HD), what="K_t")
    assert_close(kvh[:, pos, 1], want[QD + KVD:].reshape(Hkv, HD), what="V_t")
    untouched = np.ones((Hkv, S), bool)
    untouched[:, pos] = False
    assert np.all(kvh[untouched] == 7.0)


@pytest.mark.parametrize("sp", [0, 1, 31, 32, 33, 100, 255])
def test_decode_attention_against_reference_golden(golden, sp):
    """decode_attn/reference.py golden vectors (H=16, KV=8, D=128), [K half | V half] buffer."""
    g = golden("decode_attn")
    S = 256
    op = DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=S,
                         use_runtime_seq_len=True, kv_halves=True)
    call = op.get_callable()
    call.params.write("S_kv_eff", sp + 1)
    call.params.sync()
    kv = np.concatenate([from_bits(g["K"]), from_bits(g["V"])], axis=1)  # (KV, 2S, D)
    o = _out(16 * 128)
    call(dev_bf16(g["Q"]), dev_bf16(kv).reshape(8, 2 * S * 128), o.reshape(16, 128))
    torch.cuda.synchronize()
    want = from_bits(g[f"O_{sp}"])  # the float64 result rounded to bf16, to within one ulp
    assert_close(host(o), want, what=f"seq_pos {sp}")
    # float32 sums in another order: the golden's rounding almost everywhere; outputs
    # that nearly cancel (down to ~1e-6 here) may sit several of their ulps away
    _near_rounding(host(o), want, f"seq_pos {sp}")


@pytest.mark.parametrize("layout", ["token", "block"])
@pytest.mark.parametrize("L", [1, 33, 64, 65, 130, 511, 512])
def test_decode_attention_layouts_and_unaligned_lengths(layout, L):
    """seq_pos values of decode_attn/test_seqpos_unaligned.py:80 over both cache layouts."""
    rng = np.random.default_rng(L)
    H, KV, D, S, B = 16, 8, 128, 512, 64
    Q = rnd(rng.standard_normal((H, D)).astype(np.float32))
    K = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    V = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    if layout == "token":
        kv = np.stack([K, V], axis=2).reshape(KV, 2 * S * D)
        op = DecodeAttention(num_heads=H, num_kv_heads=KV, head_dim=D, seq_len_kv=S, use_runtime_seq_len=True)
    else:
        kv = np.concatenate([K.reshape(KV, S // B, B, D), V.reshape(KV, S // B, B, D)], axis=2).reshape(KV, -1)
        op = DecodeAttention(num_heads=H, num_kv_heads=KV, head_dim=D, seq_len_kv=S, block_kv=B,
                             use_runtime_seq_len=True, kv_token_interleaved=False)
    call = op.get_callable()
    call.params.write("S_kv_eff", L)
    call.params.sync()
    o = _out(H * D)
    call(dev_bf16(Q), dev_bf16(kv), o.reshape(H, D))
    torch.cuda.synchronize()
    want = ops.decode_attention(Q, K, V, L - 1, D, H, KV)
    assert_close(host(o).reshape(H, D), want, what=f"L={L}")
    assert not np.isnan(host(o)).any()


def _pack_kv(K, V, layout, block=32):
    """One stream's cache (KV, 2*S*D) from K, V (KV, S, D) in the three layouts."""
    KV, S, D = K.shape
    if layout == "token":
        return np.stack([K, V], axis=2).reshape(KV, 2 * S * D)
    if layout == "block":
        return np.concatenate([K.reshape(KV, S // block, block, D), V.reshape(KV, S // block, block, D)],
                              axis=2).reshape(KV, -1)
    return np.concatenate([K, V], axis=1).reshape(KV, -1)


def _near_rounding(got, want, what):
    """bf16 outputs against a float reference: the float32 sums of the kernel differ
    from the reference's only in order, so almost every output is the reference's
    rounding and the rest one ulp off -- except values so near zero that the absolute
    summation error spans several of their ulps, held to 1e-4 absolute instead."""
    got = np.asarray(got, np.float32).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    g = round_bits(got).astype(np.int32)
    w = round_bits(rnd(want.astype(np.float32))).astype(np.int32)
    d = np.abs(np.where(g >= 0x8000, 0x8000 - g, g) - np.where(w >= 0x8000, 0x8000 - w, w))
    assert np.mean(d == 0) >= 0.9, f"{what}: only {np.mean(d == 0):.4f} bit-exact"
    assert np.mean(d <= 1) >= 0.995, f"{what}: {np.mean(d <= 1):.4f} within one ulp"
    far = d > 2
    assert np.all(np.abs(got[far] - want[far]) <= 1e-4), f"{what}: {np.abs(got[far] - want[far]).max()}"


@pytest.mark.parametrize("HD,GQ", [(128, 4), (128, 2), (128, 8), (64, 4)])
def test_decode_attention_tensor_pipe_matches_lane_kernel(HD, GQ):
    """Both pass-1 kernels of iron_decode_attn on the same ragged streams: the tensor-pipe
    one (16-byte aligned queries) and the lane-load one (the same queries 4 bytes off a
    16-byte boundary, which the tensor-pipe kernel does not take).  Both are float32
    flash decoding over the same positions and differ only in summation order."""
    from iron_b200 import _lib

    B, KV, S = 5, 8, 700
    H = KV * GQ
    g = torch.Generator(device="cuda").manual_seed(HD * 10 + GQ)
    qa = torch.randn(B * H * HD, generator=g, device="cuda").to(torch.bfloat16)
    qbuf = torch.zeros(B * H * HD + 2, dtype=torch.bfloat16, device="cuda")
    qb = qbuf[2:]  # 4 bytes past the allocation's aligned start
    qb.copy_(qa)
    assert qa.data_ptr() % 16 == 0 and qb.data_ptr() % 16 == 4
    kv = torch.randn(B, KV, 2 * S * HD, generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.tensor([S, S // 2 + 3, 1, 65, 64], dtype=torch.int32, device="cuda")
    nws = _lib.lib().iron_decode_attn_workspace_bytes(B, H, HD, S)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    outs = []
    for q in (qa, qb):
        out = torch.zeros(B, H, HD, dtype=torch.bfloat16, device="cuda")
        _lib.call("iron_decode_attn", q.data_ptr(), kv.data_ptr(), out.data_ptr(), B, H, KV, HD, S, 0, 0, 0,
                  lens.data_ptr(), ws.data_ptr(), nws, _lib.stream_ptr())
        torch.cuda.synchronize()
        outs.append(host(out))
    _near_rounding(outs[0], outs[1], f"HD {HD} GQ {GQ}")
    kvr = kv.float().view(B, KV, S, 2, HD)
    for b in range(B):
        Lb = int(lens[b])
        K = kvr[b, :, :Lb, 0].repeat_interleave(GQ, 0)
        V = kvr[b, :, :Lb, 1].repeat_interleave(GQ, 0)
        p = torch.softmax(torch.einsum("hd,hjd->hj", qa.view(B, H, HD)[b].float(), K) / HD ** 0.5, -1)
        assert_close(outs[0][b], host(torch.einsum("hj,hjd->hd", p, V)), what=f"stream {b}")


def _verify_op(H, KV, D, S, T, causal, layout, block=32, **kw):
    return DecodeAttention(num_heads=H, num_kv_heads=KV, head_dim=D, seq_len_kv=S, block_kv=block,
                           use_runtime_seq_len=True, batch_queries=T if T % 8 else 8, num_new_tokens=T,
                           causal=causal, kv_token_interleaved=layout != "block", kv_halves=layout == "halves",
                           **kw)


@pytest.mark.parametrize("layout", ["token", "block", "halves"])
@pytest.mark.parametrize("tag", ["causal", "noncausal"])
def test_decode_attention_verify_mode_against_reference_golden(golden, tag, layout):
    """The multi-query verify mode (decode_attn/op.py:40-56) on the batch test's golden
    (decode_attn/test_batch.py:31-46): 16 new tokens at positions 192..207 of a 256-position
    cache; causal (query m sees [0, 192 + m]) and over the whole cache.  The golden is
    float32; the bf16 output is held to the decode gate and to its rounding."""
    g = golden("decode_attn_batch")
    N, H, KV, D, S, base = (int(v) for v in g["dims"])
    Q, K, V = (from_bits(g[k]) for k in ("Q", "K", "V"))
    op = _verify_op(H, KV, D, S, N, tag == "causal", layout)
    call = op.get_callable()
    call.params.write("S_kv_base", base)
    call.params.sync()
    o = _out(N * H * D)
    call(dev_bf16(Q).reshape(N * H, D), dev_bf16(_pack_kv(K, V, layout)), o.reshape(N * H, D))
    torch.cuda.synchronize()
    want = g[f"O_{tag}"]
    got = host(o).reshape(N, H, D)
    assert_close(got, want, what=f"verify {tag} {layout}")
    _near_rounding(got, want, f"verify {tag} {layout}")
    _near_rounding(got, ops.decode_attention_batch(Q, K, V, base, tag == "causal", D, H, KV), "vs oracle")


def test_decode_attention_verify_mask_matters():
    """Causal and whole-cache outputs differ (decode_attn/test_batch.py main: the mask
    must do something), and a runtime base written later takes effect without a rebuild."""
    rng = np.random.default_rng(3)
    H, KV, D, S, T = 16, 8, 128, 256, 16
    Q = rnd(rng.standard_normal((T, H, D)).astype(np.float32))
    K = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    V = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    kv = dev_bf16(_pack_kv(K, V, "token"))
    outs = {}
    for causal in (True, False):
        call = _verify_op(H, KV, D, S, T, causal, "token").get_callable()
        for base in (192, 40):
            call.params.write("S_kv_base", base)
            call.params.sync()
            o = _out(T * H * D)
            call(dev_bf16(Q).reshape(T * H, D), kv, o.reshape(T * H, D))
            torch.cuda.synchronize()
            outs[causal, base] = host(o).reshape(T, H, D)
            want = ops.decode_attention_batch(Q, K, V, base, causal, D, H, KV)
            assert_close(outs[causal, base], want, what=f"causal={causal} base={base}")
    assert not np.array_equal(outs[True, 192], outs[False, 192])
    assert not np.array_equal(outs[True, 192], outs[True, 40])
    assert np.array_equal(outs[False, 192], outs[False, 40])


@pytest.mark.parametrize("T,H,KV,D,S,base,causal", [
    (1, 16, 8, 128, 512, 300, True), (5, 16, 8, 128, 512, 507, True), (37, 32, 8, 128, 640, 100, True),
    (100, 16, 8, 64, 256, 0, True), (33, 8, 8, 128, 320, 77, False), (64, 16, 4, 128, 1024, 960, True)])
def test_attn_mq_shapes_against_oracle(T, H, KV, D, S, base, causal):
    """iron_attn_mq over ragged token counts (row blocks past the last row), GQA 1..8,
    head_dim 64, prompts from position 0 and blocks ending at the cache's end, against
    the oracle's per-query decode attention."""
    from iron_b200 import _lib
    rng = np.random.default_rng(T * 1000 + S)
    Q = rnd(rng.standard_normal((T, H, D)).astype(np.float32))
    K = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    V = rnd(rng.standard_normal((KV, S, D)).astype(np.float32))
    kv = dev_bf16(_pack_kv(K, V, "token"))
    o = torch.full((T, H, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(_lib.lib().iron_attn_mq_workspace_bytes(T, H, KV, D, S), dtype=torch.uint8, device="cuda")
    _lib.call("iron_attn_mq", dev_bf16(Q).data_ptr(), kv.data_ptr(), o.data_ptr(), T, H, KV, D, S, 0, 0, base,
              None, S, int(causal), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
    torch.cuda.synchronize()
    want = ops.decode_attention_batch(Q, K, V, base, causal, D, H, KV)
    got = host(o)
    assert not np.isnan(got).any()
    assert_close(got, want, what=f"T{T} H{H} KV{KV} D{D}")
    _near_rounding(got, want, f"T{T} H{H} KV{KV} D{D}")


def test_mlp_kernel_golden_biased_wire(golden):
    """The kernel-faithful golden of swiglu_mlp_dp/test.py (biased q+128 wire, tiles 12/4)."""
    g = golden("swiglu")
    D, FF = 256, 768
    op = SwiGLUMLPDataParallelOurs(D=D, FF=FF, num_aie_columns=2, epsilon=1e-6)
    wire = {}
    for name, K, tm in (("wg", D, 12), ("wu", D, 12), ("wd", FF, 4)):
        q = (g[f"k_{name}_q"].astype(np.int16) - 128).astype(np.int8)
        wire[name] = dev_u8(ops.pack_tile_wire(q, g[f"k_{name}_s"], tm, 2, "biased")).view(torch.bfloat16)
        assert wire[name].numel() == op.get_arg_spec()[{"wg": 3, "wu": 4, "wd": 5}[name]].shape[0]
    nxt = _out(D)
    gh = _out(FF)
    npf = rnd(g["k_npf"])
    op.get_callable()(dev_bf16(g["k_cur"]), dev_bf16(g["k_a"]), dev_bf16(npf), wire["wg"],
                      wire["wu"], wire["wd"], gh, nxt)
    torch.cuda.synchronize()
    W = {n: ((g[f"k_{n}_q"].astype(np.int16) - 128).astype(np.int8), g[f"k_{n}_s"]) for n in ("wg", "wu", "wd")}
    cur, a = from_bits(g["k_cur"]), from_bits(g["k_a"])
    exact = ops.swiglu_mlp_kernel_form(cur, a, npf, *(lambda v, n=n: ops.gemv_int8_exact(*W[n], v)
                                                      for n in ("wg", "wu", "wd")), eps=1e-6)
    premul = ops.swiglu_mlp_kernel_form(cur, a, npf, *(lambda v, n=n: ops.gemv_int8_premul(*W[n], v)
                                                       for n in ("wg", "wu", "wd")), eps=1e-6)
    _check_mlp(host(nxt), exact, premul, from_bits(g["k_nxt"]))


def _check_mlp(got, exact_chain, premul_chain, golden, rel=0.05, abs_=0.05):
    """The kernels compute every int8 matvec as the exact dequantised sum (the
    operators' reference(), swiglu_mlp_dp/op_ours.py:543-570) with float64
    accumulation, so they are held to the kernel-faithful chain with exact matvecs on
    the device's own inputs: the bf16 gate and >= 99% bit-exact.  Against the
    reference golden (swiglu_mlp_dp/test.py:53-91) the reference test's tolerance
    (test.py:190-191) applies, widened by how far that golden moves when only its
    matvec rounding changes (|premul chain - exact chain|) and by the golden's own
    inputs (a float32 n_pf the device holds in bf16: |premul chain - golden|)."""
    assert_close(got, exact_chain, what="vs exact-matvec chain")
    assert_ulps(got, exact_chain, max_ulp=1 << 15, frac_exact=0.99, what="vs exact-matvec chain")
    drift = np.abs(np.asarray(premul_chain, np.float64) - np.asarray(exact_chain, np.float64))
    inputs = np.abs(np.asarray(premul_chain, np.float64) - np.asarray(golden, np.float64))
    tol = np.maximum(abs_, rel * (np.abs(got) + np.abs(golden))) + 2 * drift + inputs
    assert np.all(np.abs(got - golden) <= tol), np.max(np.abs(got - golden) / tol)


@pytest.mark.parametrize("group", [128, 32])
def test_mlp_fuse_o_tile_major_wo(group):
    """fuse_o arm at the Qwen3-0.6B shape: Wo in the per-core tile-major wire with pad rows
    (qwen3_npu_int8.py:407-436), gate/up 12-row tiles, down 4-row tiles, signed payload."""
    D, FF, QD = 1024, 3072, 2048
    rng = np.random.default_rng(group)
    W = {}
    for name, (M, K) in (("wg", (FF, D)), ("wu", (FF, D)), ("wd", (D, FF)), ("wo", (D, QD))):
        W[name] = ops.quantize_rtn(rnd(rng.standard_normal((M, K)).astype(np.float32) * 0.02), group)
    cur = rnd(rng.standard_normal(D).astype(np.float32))
    cx = rnd(rng.standard_normal(QD).astype(np.float32))
    npf = rnd(1 + 0.1 * rng.standard_normal(D).astype(np.float32))
    op = SwiGLUMLPDataParallelOurs(D=D, FF=FF, num_aie_columns=8, epsilon=1e-6, QD=QD, fuse_o=True,
                                   kernel_source="mv_int8_signed.cc", group_size=group)
    n, n_o, tsi_o, _ = op._wo_tiling()
    spec = op.get_arg_spec()
    wo = ops.pack_wo_tiled(*W["wo"], cols=n, tsi_o=tsi_o, n_o_tiles=n_o)
    assert wo.size // 2 == spec[3].shape[0]
    bufs = [dev_bf16(cur), dev_bf16(cx), dev_bf16(npf), dev_u8(wo).view(torch.bfloat16)]
    for name, tm in (("wg", 12), ("wu", 12), ("wd", 4)):
        bufs.append(dev_u8(ops.pack_tile_wire(*W[name], tm, n, "signed")).view(torch.bfloat16))
    nxt = _out(D)
    bufs += [_out(FF), _out(D), nxt]
    op.get_callable()(*bufs)
    torch.cuda.synchronize()
    out = host(nxt)
    chains = {}
    for mode, f in (("exact", ops.gemv_int8_exact), ("premul", ops.gemv_int8_premul)):
        mv = {k: (lambda v, k=k, f=f: f(*W[k], v)) for k in W}
        chains[mode] = ops.swiglu_mlp_kernel_form(cur, rnd(mv["wo"](cx)), npf, mv["wg"], mv["wu"], mv["wd"], 1e-6)
    _check_mlp(out, chains["exact"], chains["premul"], chains["premul"])
    # the float32 golden of swiglu_mlp_dp/reference.py:54-67 within the reference's tolerance
    deq = {k: ops.dequant_f32(*W[k]) for k in W}
    f32 = ops.swiglu_mlp_fused_o(cur, cx, npf, deq["wo"], deq["wg"], deq["wu"], deq["wd"], D, FF, QD, 1e-6)
    assert not verify_buffer(out, "nxt", f32, rel_tol=0.05, abs_tol=0.05)


def test_mlp_bf16_arm():
    D, FF = 512, 1536
    rng = np.random.default_rng(4)
    Wg, Wu, Wd = (rnd(rng.standard_normal(s).astype(np.float32) * 0.05) for s in ((FF, D), (FF, D), (D, FF)))
    cur, a = (rnd(rng.standard_normal(D).astype(np.float32)) for _ in range(2))
    npf = rnd(rng.random(D).astype(np.float32) + 0.5)
    nxt = _out(D)
    SwiGLUMLPDataParallel(D=D, FF=FF, num_aie_columns=2, epsilon=1e-6).get_callable()(
        dev_bf16(cur), dev_bf16(a), dev_bf16(npf), dev_bf16(Wg).reshape(-1), dev_bf16(Wu).reshape(-1),
        dev_bf16(Wd).reshape(-1), _out(FF), nxt)
    torch.cuda.synchronize()
    want = ops.swiglu_mlp_kernel_form(cur, a, npf, lambda v: Wg.astype(np.float64) @ v,
                                      lambda v: Wu.astype(np.float64) @ v, lambda v: Wd.astype(np.float64) @ v,
                                      1e-6)
    assert_close(host(nxt), want, what="bf16 arm")


@pytest.mark.parametrize("S", [128, 96])
def test_attn_mq_prefill_against_mha_golden(golden, S):
    """Prompt attention (iron_attn_mq from position 0, causal) on the prefill MHA golden
    (mha/reference.py:26-93: torch's causal SDPA in bf16, GQA 4/2, head_dim 64), a 128-
    and a 96-token prompt; torch rounds intermediates to bf16, so a few percent of the
    golden's outputs sit one ulp from the float32 result."""
    from iron_b200 import _lib
    g = golden("mha_prefill")
    Q, K, V = (from_bits(g[f"{k}_{S}"])[:, :S] for k in "QKV")
    H, KV, D = 4, 2, 64
    kv = dev_bf16(_pack_kv(np.ascontiguousarray(K), np.ascontiguousarray(V), "token"))
    q = dev_bf16(np.ascontiguousarray(Q.transpose(1, 0, 2)))
    o = torch.empty(S, H, D, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(_lib.lib().iron_attn_mq_workspace_bytes(S, H, KV, D, S), dtype=torch.uint8, device="cuda")
    _lib.call("iron_attn_mq", q.data_ptr(), kv.data_ptr(), o.data_ptr(), S, H, KV, D, S, 0, 0, 0, None, S, 1,
              ws.data_ptr(), ws.numel(), _lib.stream_ptr())
    torch.cuda.synchronize()
    got = host(o).transpose(1, 0, 2)
    want = from_bits(g[f"O_{S}"])[:, :S]
    assert_close(got, want, what=f"prefill S={S}")
    assert_ulps(got, want, max_ulp=2, frac_exact=0.85, what=f"prefill S={S}")
    _near_rounding(got, ops.mha_prefill(Q, K, V, D, H, KV), f"prefill S={S} vs oracle")
