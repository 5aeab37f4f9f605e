"""numpy restatement of the IRON golden functions on the Qwen3 decode path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function names
the reference file:line it restates.  Conventions:

* bf16 tensors are float32 arrays holding exactly-representable bf16 values
  (``oracle.bf16.rnd``) unless a name ends in ``_bits`` (uint16 patterns).
* Where the reference computes with torch bf16 tensors, every torch op rounds
  its float32 result to bf16; the restatement rounds at the same points.
* Where the reference sums in float32 (matmul / ``sum``), the restatement sums
  in float64 and rounds once: torch's summation order is not reproducible in
  numpy, and the float64 sum is at least as close to the exact value.
"""

from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .bf16 import from_bits, rnd, round_bits

F32 = np.float32

_POOL: ThreadPoolExecutor | None = None
_THREADS = 1


def set_threads(n: int) -> int:
    """Spread the row blocks of the int8 GEMV over ``n`` host threads (numpy releases
    the GIL inside its array loops).  Returns the thread count in use."""
    global _POOL, _THREADS
    n = max(1, int(n))
    if _POOL is not None:
        _POOL.shutdown()
    _POOL = ThreadPoolExecutor(n) if n > 1 else None
    _THREADS = n
    return n


# ---------------------------------------------------------------------------
# int8 group quantisation and wire packing
# ---------------------------------------------------------------------------

def quantize_rtn(w, group: int = 128, zero_scale: str = "one"):
    """Symmetric per-(row, group) int8 RTN quantiser.

    Restates ``Qwen3NPU._set_int8_rtn`` (iron/applications/qwen3_0.6b/
    qwen3_npu_int8.py:477-490): ``s = absmax/127`` in float32, ``s = 1`` where the
    group is all zero, the wire scale is ``bf16(s)``, and ``q = round(w / f32(bf16 s))``
    (round-half-even) clamped to [-127, 127].  ``zero_scale="clamp"`` instead follows
    ``swiglu_mlp_dp/test.py:120-125`` (``clamp(min=1e-8)``).

    Returns ``(q int8 (M, K), scale_bits uint16 (M, K/group))``.
    """
    w = np.asarray(w, dtype=F32)
    m, k = w.shape
    if k % group:
        raise ValueError(f"K={k} is not a multiple of group={group}")
    ng = k // group
    blk = w.reshape(m, ng, group)
    s = (np.abs(blk).max(axis=2) / F32(127.0)).astype(F32)
    if zero_scale == "one":
        s = np.where(s > 0, s, F32(1.0)).astype(F32)
    else:
        s = np.maximum(s, F32(1e-8)).astype(F32)
    s_bits = round_bits(s)
    s_wire = from_bits(s_bits)
    q = np.rint(blk / s_wire[:, :, None]).astype(F32)
    q = np.clip(q, -127, 127).astype(np.int8).reshape(m, k)
    return q, s_bits


def pack_tile_wire(q, scale_bits, tile_m: int, cols: int = 1, domain: str = "signed"):
    """Reference int8 tile wire: per ``tile_m``-row block ``[tile_m*K payload | tile_m*G bf16]``.

    Restates ``gemv_int8/reference.py:59-80`` and ``Qwen3NPU._pack_int8``
    (qwen3_npu_int8.py:381-405).  ``domain="biased"`` stores ``q+128``
    (gemv_int8/reference.py:63-64), ``"signed"`` two's complement (:65-66).
    Returns the wire as a flat uint8 array.
    """
    q = np.asarray(q, dtype=np.int8)
    m, k = q.shape
    ng = np.asarray(scale_bits).shape[1]
    if domain == "biased":
        wb = (q.astype(np.int16) + 128).astype(np.uint8)
    elif domain == "signed":
        wb = q.view(np.uint8)
    else:
        raise ValueError(f"unknown payload domain: {domain}")
    sb = np.ascontiguousarray(np.asarray(scale_bits, dtype=np.uint16)).view(np.uint8).reshape(m, ng * 2)
    per_col = m // cols
    chunks = []
    for c in range(cols):
        for r0 in range(c * per_col, (c + 1) * per_col, tile_m):
            chunks.append(wb[r0:r0 + tile_m].reshape(-1))
            chunks.append(sb[r0:r0 + tile_m].reshape(-1))
    return np.concatenate(chunks).astype(np.uint8)


def unpack_tile_wire(wire, m: int, k: int, group: int, tile_m: int, domain: str = "signed"):
    """Inverse of :func:`pack_tile_wire` -> ``(q int8 (M,K), scale_bits (M,G))``."""
    b = np.asarray(wire, dtype=np.uint8).reshape(-1)
    ng = k // group
    tb = tile_m * (k + 2 * ng)
    q = np.empty((m, k), np.uint8)
    s = np.empty((m, ng * 2), np.uint8)
    for t in range(m // tile_m):
        blk = b[t * tb:(t + 1) * tb]
        q[t * tile_m:(t + 1) * tile_m] = blk[:tile_m * k].reshape(tile_m, k)
        s[t * tile_m:(t + 1) * tile_m] = blk[tile_m * k:].reshape(tile_m, 2 * ng)
    if domain == "biased":
        qi = (q.astype(np.int16) - 128).astype(np.int8)
    else:
        qi = q.view(np.int8)
    return qi, s.view(np.uint16).reshape(m, ng)


def dequant_f32(q, scale_bits):
    """Dequantised weight ``q * s`` in float32 (exact: 8-bit x 8-bit significands).

    Restates ``GEMVInt8.reference`` (gemv_int8/op.py:177) and
    ``swiglu_mlp_dp/op_ours.py:_payload_to_q`` followed by the scale multiply."""
    q = np.asarray(q, dtype=np.int8).astype(F32)
    s = from_bits(scale_bits)
    g = q.shape[1] // s.shape[1]
    return (q * np.repeat(s, g, axis=1)).astype(F32)


# ---------------------------------------------------------------------------
# GEMV
# ---------------------------------------------------------------------------

def gemv_int8_premul(q, scale_bits, x, chunk_rows: int = 0):
    """int8 GEMV with the kernel's premultiplied activations, float32 result.

    Restates ``gemv_int8/reference.py:25-40`` (the kernel of
    ``aie_kernels/aie2p/mv_int8_signed.cc:70-100``): ``xs = bf16(x * s)`` per
    (row, group), ``y = sum(q * xs)`` accumulated in float (float64 here).
    ``x`` may be (K,) or (B, K); the result is (M,) or (B, M) float32.
    """
    q = np.asarray(q, dtype=np.int8)
    s = from_bits(scale_bits)
    x = np.asarray(x, dtype=F32)
    squeeze = x.ndim == 1
    xb = x[None, :] if squeeze else x
    m, k = q.shape
    g = k // s.shape[1]
    out = np.empty((xb.shape[0], m), np.float64)
    if chunk_rows <= 0:
        chunk_rows = max(128, min(8192, -(-m // (4 * _THREADS))))

    def block(r0):
        qs = q[r0:r0 + chunk_rows].astype(np.float64)
        se = np.repeat(s[r0:r0 + chunk_rows], g, axis=1)
        for b in range(xb.shape[0]):
            xs = rnd(xb[b][None, :] * se)
            out[b, r0:r0 + chunk_rows] = (qs * xs).sum(axis=1)

    starts = range(0, m, chunk_rows)
    if _POOL is not None and len(starts) > 1:
        list(_POOL.map(block, starts))
    else:
        for r0 in starts:
            block(r0)
    out = out.astype(F32)
    return out[0] if squeeze else out


def gemv_int8_exact(q, scale_bits, x):
    """Exact-dequant int8 GEMV: ``y = sum_k q*s*x`` in float64, returned as float32."""
    w = dequant_f32(q, scale_bits).astype(np.float64)
    x = np.asarray(x, dtype=np.float64)
    return (x @ w.T).astype(F32) if x.ndim == 2 else (w @ x).astype(F32)


def gemv_bf16(a, x):
    """bf16 GEMV ``C = A @ B`` (gemv/reference.py:9-11), float accumulation, bf16 result."""
    a = np.asarray(a, dtype=np.float64)
    x = np.asarray(x, dtype=np.float64)
    return rnd((x @ a.T) if x.ndim == 2 else (a @ x))


# ---------------------------------------------------------------------------
# RMSNorm, RoPE, elementwise
# ---------------------------------------------------------------------------

def rms_norm_ref(x, w=None, weighted: bool = False, eps: float = 1e-5):
    """rms_norm/reference.py:8-17 applied to bf16 tensors (torch bf16 op semantics).

    ``rms = sqrt(mean(x**2) + eps)``, ``out = x / rms`` (``* w`` if weighted); each torch
    op on a bf16 tensor rounds its float32 result to bf16, reduced along the last axis.
    """
    x = np.asarray(x, dtype=F32)
    x2 = rnd(x * x)
    mean = rnd((x2.astype(np.float64).sum(axis=-1, keepdims=True) / x.shape[-1]).astype(F32))
    ms = rnd(mean + F32(eps))
    rms = rnd(np.sqrt(ms))
    out = rnd(x / rms)
    if weighted:
        out = rnd(out * np.asarray(w, dtype=F32))
    return out


def rms_norm_f32(x, w=None, eps: float = 1e-6):
    """Kernel-form weighted RMSNorm: float32 math, one bf16 rounding.

    Restates ``aie_kernels/aie2p/rms_norm.cc:9-53`` (``sum_sq/cols + eps``, ``invsqrt``,
    ``x*inv*w`` in float32) -- the same math ``swiglu_mlp_dp/test.py:85-86`` uses
    (there ``x1 / rms * n_pf``).  Float64 here, rounded once.
    """
    x = np.asarray(x, dtype=np.float64)
    ms = (x * x).mean(axis=-1, keepdims=True) + eps
    y = x / np.sqrt(ms)
    if w is not None:
        y = y * np.asarray(w, dtype=np.float64)
    return rnd(y.astype(F32))


def rope_two_halves(x, ang):
    """RoPE, two-halves method, from the interleaved ``[cos, sin, ...]`` angle row.

    Restates ``rope/reference.py:118-154`` (kernel ``aie_kernels/generic/rope.cc:41-72``):
    float32 ``y1 = x1*c - x2*s``, ``y2 = x2*c + x1*s``, one bf16 rounding.
    ``x`` is (..., HD); ``ang`` is (HD,) or broadcastable (..., HD).
    """
    x = np.asarray(x, dtype=F32)
    ang = np.asarray(ang, dtype=F32)
    half = x.shape[-1] // 2
    c = ang[..., 0::2]
    s = ang[..., 1::2]
    x1, x2 = x[..., :half], x[..., half:]
    y1 = (x1 * c).astype(F32) - (x2 * s).astype(F32)
    y2 = (x2 * c).astype(F32) + (x1 * s).astype(F32)
    return rnd(np.concatenate([y1, y2], axis=-1))


def rope_angle_table(max_seq: int, head_dim: int, theta: float):
    """Interleaved half-dim ``[cos0, sin0, cos1, sin1, ...]`` rows, bf16 (float32 values).

    Restates ``Qwen3NPU._precompute_rope_angles`` (qwen3_npu_int8.py:580-591):
    ``inv_freq = 1/theta**(arange(half)/half)``, angle = pos*inv_freq in float32,
    cos/sin rounded to bf16.
    """
    half = head_dim // 2
    inv_freq = (1.0 / (np.float32(theta) ** (np.arange(half, dtype=F32) / F32(half)))).astype(F32)
    t = np.arange(max_seq, dtype=F32)
    freqs = np.outer(t, inv_freq).astype(F32)
    cos = rnd(np.cos(freqs.astype(np.float64)).astype(F32))
    sin = rnd(np.sin(freqs.astype(np.float64)).astype(F32))
    return np.stack([cos, sin], axis=-1).reshape(max_seq, head_dim)


def add_ref(a, b):
    """elementwise_add/reference.py: ``a + b`` on bf16 tensors (float add, bf16 store)."""
    return rnd(np.asarray(a, F32) + np.asarray(b, F32))


def mul_ref(a, b):
    """elementwise_mul/reference.py: ``a * b`` on bf16 tensors (float mul, bf16 store)."""
    return rnd(np.asarray(a, F32) * np.asarray(b, F32))


def silu_ref(x):
    """silu/reference.py:8-10: ``torch.nn.functional.silu`` on a bf16 tensor (float math,
    one bf16 rounding).  Float64 here."""
    x = np.asarray(x, dtype=np.float64)
    return rnd((x / (1.0 + np.exp(-x))).astype(F32))


def silu_tanh_bf16(g):
    """Kernel-form SiLU: sigmoid via tanh, every vector op rounding to bf16.

    Restates ``swiglu_mlp_dp/test.py:70-76`` (``silu_bf16_inplace``), the arithmetic of
    ``aie_kernels/aie2p/silu.cc:11-97``."""
    g = np.asarray(g, dtype=F32)
    half = (g * F32(0.5)).astype(F32)
    th = rnd(np.tanh(half.astype(np.float64)).astype(F32))
    one_plus = rnd(th + F32(1.0))
    sig = rnd(one_plus * F32(0.5))
    return rnd(g * sig)


# ---------------------------------------------------------------------------
# Fused operators
# ---------------------------------------------------------------------------

def qkv_head(cur, n_in, matvec, n_qn, n_kn, ang, D, HD, Hq, Hkv, eps=1e-6):
    """Fused QKV head golden -> concatenated ``[q | k | v]`` (bf16 values).

    Restates ``qkv_head_dp/reference.py:13-33``: ``hn = rms_norm_ref(cur, n_in)``;
    ``raw = bf16(W @ hn)``; q, k = per-head ``rms_norm_ref`` with ``n_qn``/``n_kn`` then
    RoPE two-halves; v = raw.  ``matvec`` maps the bf16 ``hn`` (D,) to the float
    (QD+2*KVD,) projection (e.g. premul int8 or a float weight matrix product).
    """
    QD, KVD = Hq * HD, Hkv * HD
    hn = rms_norm_ref(np.asarray(cur, F32).reshape(1, D), n_in, weighted=True, eps=eps).reshape(D)
    raw = rnd(np.asarray(matvec(hn), dtype=F32))
    q = rms_norm_ref(raw[:QD].reshape(Hq, HD), n_qn, weighted=True, eps=eps)
    k = rms_norm_ref(raw[QD:QD + KVD].reshape(Hkv, HD), n_kn, weighted=True, eps=eps)
    q = rope_two_halves(q, ang).reshape(QD)
    k = rope_two_halves(k, ang).reshape(KVD)
    return np.concatenate([q, k, raw[QD + KVD:]])


def decode_attention(Q, K, V, seq_pos: int, head_dim: int, num_heads: int, num_kv_heads: int,
                     causal: bool = True):
    """Single-query GQA decode attention, base-2 softmax.

    Restates ``decode_attn/reference.py:26-38``: ``s = (q . K^T) * log2(e)/sqrt(D)``,
    positions ``> seq_pos`` masked, ``p = exp2(s - max)``, ``o = (p @ V)/sum(p)``, bf16 out.
    Q: (H, D); K, V: (KV, S, D).  Head ``h`` reads KV head ``h*KV//H``.
    """
    scale = math.log2(math.e) / math.sqrt(head_dim)
    Q = np.asarray(Q, np.float64)
    out = np.zeros((num_heads, head_dim), np.float64)
    for h in range(num_heads):
        kv = h * num_kv_heads // num_heads
        Kh = np.asarray(K[kv], np.float64)
        Vh = np.asarray(V[kv], np.float64)
        s = (Kh @ Q[h]) * scale
        if causal:
            s = np.where(np.arange(s.shape[0]) <= seq_pos, s, -np.inf)
        p = np.exp2(s - s.max())
        out[h] = (p @ Vh) / p.sum()
    return rnd(out.astype(F32))


def decode_attention_batch(Q, K, V, s_kv_base: int, causal: bool, head_dim: int, num_heads: int,
                           num_kv_heads: int):
    """Multi-query (verify-mode) decode attention over one KV stream.

    Restates ``cpu_reference_batch`` (decode_attn/test_batch.py:31-46), the golden of
    DecodeAttention's ``batch_queries`` / ``num_new_tokens`` mode: the N new tokens sit
    at positions ``s_kv_base .. s_kv_base + N - 1``; with ``causal`` query m attends
    positions ``[0, s_kv_base + m]``, otherwise every position of K/V.  Each query is
    ``decode_attention`` at its own boundary.  Q: (N, H, D); K, V: (KV, S, D); bf16 out
    (N, H, D)."""
    Q = np.asarray(Q)
    S = np.asarray(K).shape[1]
    return np.stack([decode_attention(Q[m], K, V, (s_kv_base + m) if causal else S - 1, head_dim, num_heads,
                                      num_kv_heads, causal=True) for m in range(Q.shape[0])])


def mha_prefill(Q, K, V, head_dim: int, num_heads: int, num_kv_heads: int):
    """Causal GQA self-attention over a prompt (the prefill MHA golden).

    Restates ``mha/reference.py:26-93``: ``scaled_dot_product_attention`` with
    ``is_causal=True`` and scale ``1/sqrt(d)`` after ``repeat_interleave`` of the KV heads,
    so query head h reads KV head ``h // (H/KV)`` and position i attends ``[0, i]`` --
    ``decode_attention_batch`` with the new tokens starting at position 0.
    Q: (H, S, D); K, V: (KV, S, D); bf16 out (H, S, D)."""
    Qt = np.asarray(Q).transpose(1, 0, 2)
    return decode_attention_batch(Qt, K, V, 0, True, head_dim, num_heads, num_kv_heads).transpose(1, 0, 2)


def swiglu_mlp(cur, a, n_pf, Wg, Wu, Wd, D, FF, epsilon=1e-5):
    """Float32 SwiGLU MLP block golden (swiglu_mlp_dp/reference.py:8-38).

    ``x1 = cur + a``; ``hf = x1/sqrt(mean(x1^2)+eps) * n_pf``;
    ``nxt = x1 + Wd @ (silu(Wg@hf) * (Wu@hf))`` with the exact logistic; bf16 out.
    Float64 here.
    """
    cur = np.asarray(cur, np.float64)
    a = np.asarray(a, np.float64)
    n_pf = np.asarray(n_pf, np.float64)
    Wg = np.asarray(Wg, np.float64).reshape(FF, D)
    Wu = np.asarray(Wu, np.float64).reshape(FF, D)
    Wd = np.asarray(Wd, np.float64).reshape(D, FF)
    x1 = cur + a
    hf = x1 / np.sqrt(np.mean(x1 * x1) + epsilon) * n_pf
    g = Wg @ hf
    gh = g / (1.0 + np.exp(-g)) * (Wu @ hf)
    return rnd((x1 + Wd @ gh).astype(F32))


def swiglu_mlp_fused_o(cur, cx, n_pf, Wo, Wg, Wu, Wd, D, FF, QD, epsilon=1e-5):
    """swiglu_mlp_dp/reference.py:54-67: ``a = bf16(Wo[:D] @ cx)`` then :func:`swiglu_mlp`."""
    Wo = np.asarray(Wo, np.float64).reshape(-1, QD)[:D]
    a = rnd((Wo @ np.asarray(cx, np.float64)).astype(F32))
    return swiglu_mlp(cur, a, n_pf, Wg, Wu, Wd, D, FF, epsilon)


def swiglu_mlp_kernel_form(cur, a, n_pf, matvec_g, matvec_u, matvec_d, eps=1e-5):
    """Kernel-faithful SwiGLU MLP golden (swiglu_mlp_dp/test.py:79-91).

    ``x1 = bf16(cur + a)``; ``hf = bf16(x1/rms*n_pf)`` (float32 rms);
    ``g = bf16(matvec_g(hf))``; ``gh = bf16(silu_tanh_bf16(g) * bf16(matvec_u(hf)))``;
    ``nxt = bf16(x1 + bf16(matvec_d(gh)))``.  ``matvec_*`` return float results.
    """
    x1 = rnd(np.asarray(cur, F32) + np.asarray(a, F32))
    hf = rms_norm_f32(x1, n_pf, eps)
    g = rnd(matvec_g(hf))
    u = rnd(matvec_u(hf))
    gh = rnd(silu_tanh_bf16(g) * u)
    d = rnd(matvec_d(gh))
    return rnd(x1 + d)


def pack_wo_tiled(q, scale_bits, cols: int, tsi_o: int, n_o_tiles: int, domain: str = "signed"):
    """The fuse_o Wo wire: per core, ``n_o_tiles`` tiles of ``tsi_o`` rows covering the
    core's window, rows past the matrix end zero (payload and scale).

    Restates ``Qwen3NPU._set_wo_tiled`` (qwen3_npu_int8.py:407-436)."""
    q = np.asarray(q, dtype=np.int8)
    m, k = q.shape
    ng = np.asarray(scale_bits).shape[1]
    rows_per_col = m // cols
    pad = n_o_tiles * tsi_o - rows_per_col
    if pad < 0:
        raise ValueError("tiles do not cover the per-core window")
    wb = (q.astype(np.int16) + 128).astype(np.uint8) if domain == "biased" else q.view(np.uint8)
    W = np.zeros((m + pad, k), np.uint8)
    S = np.zeros((m + pad, ng * 2), np.uint8)
    W[:m] = wb
    S[:m] = np.ascontiguousarray(np.asarray(scale_bits, np.uint16)).view(np.uint8).reshape(m, ng * 2)
    chunks = []
    for g in range(cols):
        for j in range(n_o_tiles):
            r0 = g * rows_per_col + j * tsi_o
            chunks.append(W[r0:r0 + tsi_o].reshape(-1))
            chunks.append(S[r0:r0 + tsi_o].reshape(-1))
    return np.concatenate(chunks)


# ---------------------------------------------------------------------------
# data movement and softmax of the Llama decode runlist
# ---------------------------------------------------------------------------

def rope_interleaved(x, ang):
    """RoPE, interleaved method: columns (2j, 2j + 1) rotate by pair j of the angle row.

    Restates ``rope/reference.py:94-113`` (``x_even*cos - x_odd*sin``,
    ``x_even*sin + x_odd*cos``) in float32 with one bf16 rounding."""
    x = np.asarray(x, dtype=F32)
    ang = np.asarray(ang, dtype=F32)
    c, s = ang[..., 0::2], ang[..., 1::2]
    xe, xo = x[..., 0::2], x[..., 1::2]
    y = np.empty_like(x)
    y[..., 0::2] = (xe * c).astype(F32) - (xo * s).astype(F32)
    y[..., 1::2] = (xo * c).astype(F32) + (xe * s).astype(F32)
    return rnd(y)


def _tap_offsets(sizes, strides, offset):
    grids = np.meshgrid(*[np.arange(s) for s in sizes], indexing="ij")
    flat = np.full(grids[0].shape, offset, dtype=np.int64)
    for g, st in zip(grids, strides):
        flat = flat + g * st
    return flat.reshape(-1)


def _channel_offsets(sizes, strides, offset, channels):
    sizes = [1] * (4 - len(sizes)) + list(sizes)
    strides = [0] * (4 - len(strides)) + list(strides)
    hi = max(i for i, s in enumerate(sizes) if s >= 1)
    per = sizes[hi] // channels
    split = sizes[:hi] + [per] + sizes[hi + 1:]
    return [_tap_offsets(split, strides, offset + c * per * strides[hi]) for c in range(channels)]


def strided_copy(inp, out, in_sizes, in_strides, in_offset, out_sizes, out_strides, out_offset,
                 channels=1, in_addend=0, out_addend=0):
    """Gather by the input access pattern, scatter by the output one, channel by channel,
    into a copy of ``out`` (elements the pattern does not visit keep their values).

    Restates ``strided_copy/reference.py`` (``_pad_to_4d``, ``_tap_offsets``,
    ``_channel_offsets``, ``reference``); the addends are the runtime offset
    parameters, in elements."""
    out = np.array(out, copy=True)
    src = _channel_offsets(in_sizes, in_strides, in_offset + in_addend, channels)
    dst = _channel_offsets(out_sizes, out_strides, out_offset + out_addend, channels)
    for s, d in zip(src, dst):
        if len(s) != len(d):
            raise ValueError("tap element counts differ")
        out[d] = np.asarray(inp)[s]
    return out


def softmax_rows(x, n=None):
    """Row softmax over the first ``n`` entries (all when None), the rest zero, in float64
    and rounded once to bf16.  Restates ``softmax/reference.py`` (``torch.softmax`` over
    the last dim) with the runtime vector-size mask of ``softmax/design.py:86-103``."""
    x = np.asarray(x, dtype=np.float64)
    cols = x.shape[-1]
    n = cols if n is None else max(0, min(int(n), cols))
    out = np.zeros_like(x)
    if n:
        v = x[..., :n]
        e = np.exp(v - v.max(axis=-1, keepdims=True))
        out[..., :n] = e / e.sum(axis=-1, keepdims=True)
    return rnd(out.astype(F32))
