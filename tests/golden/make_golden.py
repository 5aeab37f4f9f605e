"""Generate the golden fixtures in this folder by running IRON's own golden code.

Run where the IRON source tree is available (it is NOT needed afterwards):

    python tests/golden/make_golden.py /path/to/IRON [--only NAME ...]

(``--only gptq_pack`` writes just that fixture and leaves the others as committed.)

The reference package ``__init__``s import the NPU toolchain (``aie``), which is
not installable off-NPU, so the golden modules are loaded by file path with a
one-symbol stand-in for ``iron.common.test_utils.torch_dtype_map``.  Functions
that live inside modules importing ``aie`` at top level (the Qwen3 runtime's
packers and rope table, the fused-MLP test's kernel-faithful golden) are
extracted with ``ast`` and executed unchanged in a small namespace.

Outputs (numpy ``.npz``; bf16 stored as uint16 bit patterns):
  gemv_int8.npz, rtn_pack.npz, rms_norm.npz, rope.npz, qkv_head.npz,
  decode_attn.npz, swiglu.npz, elementwise.npz, gemv_bf16.npz, llama_block.npz,
  gptq_pack.npz, decode_attn_batch.npz, mha_prefill.npz, seqops.npz
"""

from __future__ import annotations

import ast
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().to(torch.bfloat16).view(torch.uint16).numpy().copy()


def setup_shim(ref: Path):
    iron = types.ModuleType("iron")
    iron.__path__ = []
    common = types.ModuleType("iron.common")
    common.__path__ = []
    tu = types.ModuleType("iron.common.test_utils")
    tu.torch_dtype_map = {"bf16": torch.bfloat16, "f32": torch.float32, "i8": torch.int8,
                          "ui8": torch.uint8, "i16": torch.int16, "i32": torch.int32}
    ops = types.ModuleType("iron.operators")
    ops.__path__ = []
    for m in (iron, common, tu, ops):
        sys.modules[m.__name__] = m


def load(ref: Path, rel: str, modname: str):
    spec = importlib.util.spec_from_file_location(modname, ref / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[modname] = mod
    spec.loader.exec_module(mod)
    return mod


def extract(ref: Path, rel: str, names: list[str], cls: str | None = None, extra_globals=None):
    """Exec selected top-level (or class-level) function defs of a file unchanged."""
    src = (ref / rel).read_text()
    tree = ast.parse(src)
    body = tree.body
    if cls is not None:
        body = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls).body
    fns = [n for n in body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {f.name for f in fns}
    if missing:
        raise KeyError(f"{rel}: {missing}")
    mod = ast.Module(body=fns, type_ignores=[])
    g = {"np": np, "torch": torch, **(extra_globals or {})}
    exec(compile(mod, str(ref / rel), "exec"), g)
    return {n: g[n] for n in names}


def gptq_pack(ref: Path):
    """The Qwen3 runtime's GPTQ import (``_set_int8`` -> ``_gptq_rows`` -> ``_pack_int8``)
    on seeded random checkpoint tensors: two projections stacked along M (as q/k/v),
    K = 256 in groups of 128 (the packer's fixed group), every byte value 0..255 in the
    words, fp16 scales including an fp16 subnormal; both payload domains with one row
    per tile and one column (the plain wire), the signed wire in tiles of 4 rows over
    2 columns, and fuse_o's tile-major Wo wire (``_set_wo_tiled``) with overlapping
    per-core windows and pad rows."""
    app = "iron/applications/qwen3_0.6b/qwen3_npu_int8.py"
    fns = extract(ref, app, ["_set_int8", "_gptq_rows", "_pack_int8", "_set_wo_tiled"], cls="Qwen3NPU")
    captured = {}

    class FakeSelf:
        def _set(self, name, t):
            captured[name] = t

        def _gptq_rows(self, *a, **k):
            return fns["_gptq_rows"](self, *a, **k)

        def _pack_int8(self, *a):
            return fns["_pack_int8"](self, *a)

    rng = np.random.default_rng(23)
    K, Ms = 256, (24, 8)
    qws, scs = [], []
    for M in Ms:
        words = rng.integers(0, 2 ** 32, size=(K // 4, M), dtype=np.uint64).astype(np.uint32)
        words[0, 0], words[1, 0] = 0x00000000, 0xFFFFFFFF  # q = -128 and q = 127 everywhere in a word
        qws.append(torch.from_numpy(words.view(np.int32).copy()))
        sc = (rng.random((K // 128, M)) * 0.05 + 1e-4).astype(np.float16)
        sc[0, 1] = np.float16(6e-8)  # an fp16 subnormal
        scs.append(torch.from_numpy(sc))
    out = {}
    for signed, tag in ((True, "signed"), (False, "biased")):
        fns["_set_int8"](FakeSelf(), tag, qws, scs, sum(Ms), K, 1, 1, signed=signed)
        out[f"wire_{tag}"] = captured[tag].view(torch.uint8).numpy()
    # per-core tiles as the fused ops take them: 2 columns, 4 rows per tile
    fns["_set_int8"](FakeSelf(), "tiles", qws, scs, sum(Ms), K, 2, 4, signed=True)
    out["wire_signed_c2_t4"] = captured["tiles"].view(torch.uint8).numpy()
    # fuse_o's Wo: 2 cores of 16 rows, windows of 3 tiles x 6 rows (rows 16-17 twice, 2 pad rows)
    words = rng.integers(0, 2 ** 32, size=(K // 4, 32), dtype=np.uint64).astype(np.uint32)
    qwo = torch.from_numpy(words.view(np.int32).copy())
    sco = torch.from_numpy((rng.random((K // 128, 32)) * 0.05 + 1e-4).astype(np.float16))
    w_q, s_mg = fns["_gptq_rows"](FakeSelf(), qwo, sco, signed=True)
    fns["_set_wo_tiled"](FakeSelf(), "wo", w_q, s_mg, 32, K, 2, 6, 3)
    out.update(qweight_o=qwo.numpy(), scales_o=sco.numpy().view(np.uint16),
               wire_wo_c2_t6_n3=captured["wo"].view(torch.uint8).numpy())
    np.savez_compressed(OUT / "gptq_pack.npz", qweight_a=qws[0].numpy(), qweight_b=qws[1].numpy(),
                        scales_a=scs[0].numpy().view(np.uint16), scales_b=scs[1].numpy().view(np.uint16),
                        **out)


def decode_attn_batch(ref: Path):
    """DecodeAttention's multi-query verify mode: the batch test's CPU golden
    (``cpu_reference_batch``, float32 out) on N(0, 1) data, 16 new tokens after 192
    cached positions of a 256-position cache, causal and non-causal (16 query heads,
    8 KV heads, head_dim 128)."""
    fns = extract(ref, "iron/operators/decode_attn/test_batch.py", ["cpu_reference_batch"],
                  extra_globals={"math": __import__("math")})
    g = torch.Generator().manual_seed(29)
    N, H, KV, D, S, base = 16, 16, 8, 128, 256, 192
    Q = torch.randn(N, H, D, generator=g).to(torch.bfloat16)
    K = torch.randn(KV, S, D, generator=g).to(torch.bfloat16)
    V = torch.randn(KV, S, D, generator=g).to(torch.bfloat16)
    out = {f"O_{tag}": fns["cpu_reference_batch"](Q, K, V, base, N, S, causal, head_dim=D, GQA=H // KV).numpy()
           for causal, tag in ((True, "causal"), (False, "noncausal"))}
    np.savez_compressed(OUT / "decode_attn_batch.npz", Q=bits(Q), K=bits(K), V=bits(V),
                        dims=np.array([N, H, KV, D, S, base]), **out)


def mha_prefill(ref: Path):
    """The prefill MHA golden (torch's causal SDPA in bf16, GQA by repeat_interleave)
    from its own generator: 4 query heads over 2 KV heads, head_dim 64, a 128-token
    prompt and a 96-token one (padded by the generator to 128 with zeros)."""
    m = load(ref, "iron/operators/mha/reference.py", "ref_mha")
    out = {}
    for S in (128, 96):
        g = m.generate_golden_reference(heads=4, S_q=S, S_kv=S, d=64, num_kv_heads=2)
        out.update({f"{k}_{S}": bits(g[k]) for k in ("Q", "K", "V", "O")})
    np.savez_compressed(OUT / "mha_prefill.npz", **out)


def seqops(ref: Path):
    """The data-movement and softmax operators of the Llama decode runlist, from their
    own golden generators: RoPE (``rope/reference.py``; the exact target from the bf16
    angle buffer: ``reference`` for the two halves, ``apply_rope`` with the buffer's
    cos/sin for the interleaved method; rows laid out as the rope test lays them,
    ``(seq_len, n_heads, cols)``), StridedCopy (the cases of ``strided_copy/test.py``
    plus runtime offset addends), Repeat, Softmax and Transpose."""
    import json
    rope = load(ref, "iron/operators/rope/reference.py", "ref_rope_seq")
    sc = load(ref, "iron/operators/strided_copy/reference.py", "ref_strided_copy")
    rep = load(ref, "iron/operators/repeat/reference.py", "ref_repeat")
    smx = load(ref, "iron/operators/softmax/reference.py", "ref_softmax")
    tr = load(ref, "iron/operators/transpose/reference.py", "ref_transpose")
    out = {}
    for i, (rows, cols, arows, method) in enumerate(((32, 512, 8, 0), (32, 128, 16, 1), (64, 128, 32, 1),
                                                     (64, 128, 8, 0))):
        g = rope.generate_golden_reference(rows=rows, cols=cols, context_len=arows, method_type=method)
        x = g["A"].transpose(0, 1).contiguous().reshape(rows, cols)
        ang = g["B"]
        if method == 0:
            y = rope.reference(x, ang, 0, rows, cols)
        else:
            cos, sin = ang[:, 0::2].float(), ang[:, 1::2].float()
            y = rope.apply_rope(g["A"], cos, sin, 1).transpose(0, 1).contiguous().reshape(rows, cols)
        out.update({f"rope{i}_x": bits(x), f"rope{i}_ang": bits(ang), f"rope{i}_y": bits(y),
                    f"rope{i}_dims": np.array([rows, cols, arows, method])})

    def kv_slot(seq, slot, ch=1):
        return dict(input_sizes=[8, 64], input_strides=[64, 1], input_offset=0, input_buffer_size=8 * 64,
                    output_sizes=[1, 8, 64], output_strides=[0, seq * 64, 1], output_offset=slot * 64,
                    output_buffer_size=8 * seq * 64, num_aie_channels=ch)

    def flat(n, ch=1):
        return dict(input_sizes=[n], input_strides=[1], input_offset=0, input_buffer_size=n,
                    output_sizes=[n], output_strides=[1], output_offset=0, output_buffer_size=n,
                    num_aie_channels=ch)

    cases = [flat(1024), flat(1024, 2), flat(1024, 4), kv_slot(128, 5), kv_slot(128, 5, 2), kv_slot(128, 5, 4),
             dict(kv_slot(128, 0), output_offset_addend=37 * 64),
             dict(input_sizes=[4, 16, 8], input_strides=[8, 32, 1], input_offset=3, input_buffer_size=600,
                  output_sizes=[16, 32], output_strides=[40, 1], output_offset=0, output_buffer_size=700,
                  num_aie_channels=2, input_offset_addend=5, output_offset_addend=11)]
    for i, kw in enumerate(cases):
        g = sc.generate_golden_reference(**kw)
        out.update({f"sc{i}_in": bits(g["input"]), f"sc{i}_out": bits(g["output"]),
                    f"sc{i}_kw": np.array(json.dumps(kw))})
    for i, (rows, cols, r) in enumerate(((8, 64, 4), (8, 512, 4), (4, 1024, 2))):
        g = rep.generate_golden_reference(rows=rows, cols=cols, repeat=r)
        out.update({f"rep{i}_in": bits(g["input"]), f"rep{i}_out": bits(g["output"]),
                    f"rep{i}_dims": np.array([rows, cols, r])})
    for i, (rows, cols) in enumerate(((32, 256), (16, 1024))):
        g = smx.generate_golden_reference(rows=rows, cols=cols)
        out.update({f"smx{i}_in": bits(g["input"]), f"smx{i}_out": bits(g["output"])})
    for i, (M, N, b) in enumerate(((256, 64, 1), (64, 128, 4))):
        g = tr.generate_golden_reference(rows=M, cols=N, num_batches=b)
        out.update({f"tr{i}_in": bits(g["input"]), f"tr{i}_out": bits(g["output"]),
                    f"tr{i}_dims": np.array([M, N, b])})
    np.savez_compressed(OUT / "seqops.npz", **out)


def main(ref: Path, only: list[str] | None = None):
    setup_shim(ref)
    if only:
        for name in only:
            {"gptq_pack": gptq_pack, "decode_attn_batch": decode_attn_batch, "mha_prefill": mha_prefill,
             "seqops": seqops}[name](ref)
        print("wrote", ", ".join(only), "to", OUT)
        return
    rms = load(ref, "iron/operators/rms_norm/reference.py", "iron.operators.rms_norm.reference")
    rope = load(ref, "iron/operators/rope/reference.py", "iron.operators.rope.reference")
    qkv = load(ref, "iron/operators/qkv_head_dp/reference.py", "iron.operators.qkv_head_dp.reference")
    attn = load(ref, "iron/operators/decode_attn/reference.py", "ref_decode_attn")
    g8 = load(ref, "iron/operators/gemv_int8/reference.py", "ref_gemv_int8")
    mlp = load(ref, "iron/operators/swiglu_mlp_dp/reference.py", "ref_swiglu_mlp_dp")
    gemv = load(ref, "iron/operators/gemv/reference.py", "ref_gemv")
    silu = load(ref, "iron/operators/silu/reference.py", "ref_silu")
    add = load(ref, "iron/operators/elementwise_add/reference.py", "ref_add")
    mul = load(ref, "iron/operators/elementwise_mul/reference.py", "ref_mul")

    # ---- int8 GEMV: the reference's own generator + a group-32 variant ----
    g = g8.generate_golden_reference(M=256, K=1024)
    rng = np.random.default_rng(7)
    s32 = torch.from_numpy((rng.random((256, 1024 // 32)) * 0.05 + 0.01).astype(np.float32)).to(torch.bfloat16)
    c32 = g8.reference(torch.from_numpy(g["w_int8"]), s32, g["B"]).to(torch.bfloat16)
    wire_signed = g8.pack_payload(g["w_int8"][:16], g["scales"][:16], 2, 4, "signed")
    wire_biased = g8.pack_payload(g["w_int8"][:16], g["scales"][:16], 1, 2, "biased")
    np.savez_compressed(
        OUT / "gemv_int8.npz", w_int8=g["w_int8"], scales=bits(g["scales"]), x=bits(g["B"]),
        y=bits(g["C"]), scales_g32=bits(s32), y_g32=bits(c32),
        wire_signed_c2_t4=wire_signed.view(torch.uint16).numpy(),
        wire_biased_c1_t2=wire_biased.view(torch.uint16).numpy())

    # ---- RTN quantiser + tile packer + rope table from the Qwen3 runtime ----
    app = "iron/applications/qwen3_0.6b/qwen3_npu_int8.py"
    fns = extract(ref, app, ["_set_int8_rtn", "_pack_int8", "_precompute_rope_angles"], cls="Qwen3NPU")
    captured = {}

    class FakeSelf:
        def _set(self, name, t):
            captured[name] = t

        def _pack_int8(self, *a):
            return fns["_pack_int8"](self, *a)

    w = (torch.randn(64, 256, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)
    w[5, :128] = 0  # an all-zero group exercises the s=1 branch
    fns["_set_int8_rtn"](FakeSelf(), "W", w, 64, 256, 1, 4, signed=True)
    wire128 = captured["W"].view(torch.uint16).numpy()
    fns["_set_int8_rtn"](FakeSelf(), "W2", w, 64, 256, 2, 2, signed=False)
    wire128b = captured["W2"].view(torch.uint16).numpy()
    ns = types.SimpleNamespace()
    rope_mod = extract(ref, app, ["_precompute_rope_angles"], cls="Qwen3NPU",
                       extra_globals={"head_dim": 128, "rope_theta": 1e6, "max_seq_len": 1200})
    rope_mod["_precompute_rope_angles"](ns)
    np.savez_compressed(OUT / "rtn_pack.npz", w=bits(w), wire_signed_t4=wire128,
                        wire_biased_c2_t2=wire128b, angle_table=bits(ns.angle_table))

    # ---- RMSNorm: reference generator (weighted, eps 1e-6) + N(0,1) rows ----
    gr = rms.generate_golden_reference(rows=4, cols=1024, weighted=True, eps=1e-6)
    gen = torch.Generator().manual_seed(11)
    x = torch.randn(3, 1024, generator=gen).to(torch.bfloat16)
    wv = (1 + 0.1 * torch.randn(1024, generator=gen)).to(torch.bfloat16)
    y = rms.reference(x, wv, weighted=True, eps=1e-6)
    np.savez_compressed(OUT / "rms_norm.npz", x_gen=bits(gr["input"]), w_gen=bits(gr["weight"]),
                        y_gen=bits(gr["output"]), x=bits(x), w=bits(wv), y=bits(y))

    # ---- RoPE two-halves from an angle row ----
    xr = torch.randn(16, 1, 128, generator=gen).to(torch.bfloat16)
    ang = ns.angle_table[777].reshape(1, 128)
    yr = rope.reference(xr, ang, method_type=0, rows=1, cols=128)
    np.savez_compressed(OUT / "rope.npz", x=bits(xr.reshape(16, 128)), ang=bits(ang), y=bits(yr))

    # ---- fused QKV head (float weights, Qwen3-0.6B head geometry, D=256) ----
    D, HD, Hq, Hkv = 256, 128, 4, 2
    cur = torch.randn(D, generator=gen).to(torch.bfloat16)
    n_in = (1 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    wqkv = (0.05 * torch.randn((Hq + 2 * Hkv) * HD, D, generator=gen)).to(torch.bfloat16)
    n_qn = (1 + 0.1 * torch.randn(HD, generator=gen)).to(torch.bfloat16)
    n_kn = (1 + 0.1 * torch.randn(HD, generator=gen)).to(torch.bfloat16)
    angq = ns.angle_table[345]
    out = qkv.reference(cur, n_in, wqkv, n_qn, n_kn, angq, D, HD, Hq, Hkv, eps=1e-6)
    np.savez_compressed(OUT / "qkv_head.npz", cur=bits(cur), n_in=bits(n_in), wqkv=bits(wqkv),
                        n_qn=bits(n_qn), n_kn=bits(n_kn), ang=bits(angq), out=bits(out),
                        dims=np.array([D, HD, Hq, Hkv]))

    # ---- decode attention: reference generator + several causal boundaries ----
    ga = attn.generate_golden_reference(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=256)
    kv = ga["kv_in"].reshape(8, 2 * 256, 128)
    K, V = kv[:, :256], kv[:, 256:]
    outs = {}
    for sp in (0, 1, 31, 32, 33, 100, 255):
        outs[f"O_{sp}"] = bits(attn.reference(ga["Q"], K, V, sp, 128, 16, 8))
    np.savez_compressed(OUT / "decode_attn.npz", Q=bits(ga["Q"]), K=bits(K), V=bits(V),
                        O_gen=bits(ga["O"]), **outs)

    # ---- SwiGLU MLP: f32 goldens (plain and fuse_o) + the kernel-faithful golden ----
    gm = mlp.generate_golden_reference(D=128, FF=384)
    gf = mlp.generate_golden_reference_fused_o(D=128, FF=384, QD=256)
    tf = extract(ref, "iron/operators/swiglu_mlp_dp/test.py",
                 ["matvec_int8", "silu_bf16_inplace", "reference", "quantize_weights"],
                 extra_globals={"GROUP": 128})
    torch.manual_seed(42)
    Dk, FFk = 256, 768
    wg_q, wg_s = tf["quantize_weights"](torch.randn(FFk, Dk) * 0.1)
    wu_q, wu_s = tf["quantize_weights"](torch.randn(FFk, Dk))
    wd_q, wd_s = tf["quantize_weights"](torch.randn(Dk, FFk))
    qg = torch.from_numpy(wg_q.astype(np.int16) - 128).float()
    qu = torch.from_numpy(wu_q.astype(np.int16) - 128).float()
    qd = torch.from_numpy(wd_q.astype(np.int16) - 128).float()
    mv = tf["matvec_int8"]
    kcur = torch.randn(Dk).to(torch.bfloat16) * 0.2
    ka = torch.randn(Dk).to(torch.bfloat16) * 0.2
    kn = torch.rand(Dk) + 0.5
    knxt = tf["reference"](kcur, ka, kn,
                           lambda v: mv(qg, wg_s, v).to(torch.bfloat16),
                           lambda v: mv(qu, wu_s, v).to(torch.bfloat16),
                           lambda v: mv(qd, wd_s, v).to(torch.bfloat16), eps=1e-6)
    sil_in = (torch.randn(4096, generator=gen) * 4).to(torch.bfloat16)
    np.savez_compressed(
        OUT / "swiglu.npz",
        **{f"f32_{k}": v.view(np.uint16) for k, v in gm.items()},
        **{f"fo_{k}": v.view(np.uint16) for k, v in gf.items()},
        k_wg_q=wg_q, k_wg_s=wg_s, k_wu_q=wu_q, k_wu_s=wu_s, k_wd_q=wd_q, k_wd_s=wd_s,
        k_cur=bits(kcur), k_a=bits(ka), k_npf=kn.numpy(), k_nxt=bits(knxt),
        silu_in=bits(sil_in), silu_tanh_out=bits(tf["silu_bf16_inplace"](sil_in)))

    # ---- elementwise + SiLU goldens ----
    ea = (torch.randn(2048, generator=gen) * 3).to(torch.bfloat16)
    eb = (torch.randn(2048, generator=gen) * 3).to(torch.bfloat16)
    np.savez_compressed(OUT / "elementwise.npz", a=bits(ea), b=bits(eb),
                        add=bits(add.reference(ea, eb)), mul=bits(mul.reference(ea, eb)),
                        silu=bits(silu.reference(ea)))

    # ---- bf16 GEMV golden (reference generator) ----
    gb = gemv.generate_golden_reference(M=256, K=512)
    np.savez_compressed(OUT / "gemv_bf16.npz", A=bits(gb["A"]), B=bits(gb["B"]), C=bits(gb["C"]))
    # ---- Llama decode block (llama_cpu.py, the C5 CPU path) ----
    import math
    lf = extract(ref, "iron/applications/llama_3.2_1b/llama_cpu.py",
                 ["rope_forward", "rms_norm_forward", "grouped_query_attention_forward", "swiglu_ffn_forward",
                  "transformer_block_forward"], extra_globals={"math": math})
    hf = extract(ref, "iron/applications/llama_3.2_1b/llama_inference_harness.py", ["compute_rope_angles"])
    lg = torch.Generator().manual_seed(51)
    D, H, KVH, HD, FF, T = 256, 4, 2, 64, 512, 5  # T cached positions, one new token
    bf = torch.bfloat16

    def lw(*shape, std=0.02, mean=0.0):
        return (torch.randn(*shape, generator=lg) * std + mean).to(bf)

    x = lw(1, 1, D, std=1.0)
    wts = {"norm1": lw(D, std=0.1, mean=1.0), "wq": lw(H * HD, D), "wk": lw(KVH * HD, D), "wv": lw(KVH * HD, D),
           "wo": lw(D, H * HD), "norm2": lw(D, std=0.1, mean=1.0), "wg": lw(FF, D), "wu": lw(FF, D),
           "wd": lw(D, FF)}
    kc, vc = lw(1, KVH, T, HD, std=1.0), lw(1, KVH, T, HD, std=1.0)
    angles = hf["compute_rope_angles"](HD, 64, 500000.0)
    out, k2, v2 = lf["transformer_block_forward"](x, kc, vc, H, KVH, wts["norm1"], wts["wq"], wts["wk"], wts["wv"],
                                                  wts["wo"], wts["norm2"], wts["wg"], wts["wu"], wts["wd"],
                                                  angles, None)
    np.savez_compressed(OUT / "llama_block.npz", x=bits(x.reshape(D)), kc=bits(kc[0]), vc=bits(vc[0]),
                        angles=angles.numpy(), out=bits(out.reshape(D)), k_new=bits(k2[0, :, T]),
                        v_new=bits(v2[0, :, T]), dims=np.array([D, H, KVH, HD, FF, T]),
                        **{k: bits(v) for k, v in wts.items()})
    gptq_pack(ref)
    decode_attn_batch(ref)
    mha_prefill(ref)
    seqops(ref)
    print("wrote fixtures to", OUT)


if __name__ == "__main__":
    if len(sys.argv) < 2 or (len(sys.argv) > 2 and sys.argv[2] != "--only"):
        sys.exit("usage: make_golden.py <path to the IRON source tree> [--only NAME ...]")
    main(Path(sys.argv[1]), sys.argv[3:] if len(sys.argv) > 2 else None)
