"""GPTQ int8 checkpoints -> the library's int8 wires.

The reference's Qwen3 int8 application decodes from a GPTQ checkpoint: symmetric
int8 with zero-point 128 and one fp16 scale per (group of K, output row); the tied
lm_head stays bf16 (iron/applications/qwen3_0.6b/qwen3_npu_int8.py:144-181 names the
tensors).  It repacks every projection on the host: ``_gptq_rows`` (:350-379) unpacks
``qweight`` -- (K/4, M) 32-bit words, the byte j of word (r, m) (least significant
first) holding u = q + 128 for column k = 4r + j of row m -- into row-major payload
bytes, either as u itself (the biased domain) or as q in two's complement (the signed
domain, byte = u ^ 0x80), and rounds the fp16 scales to bf16 through float32;
``_set_int8`` (:438-455) stacks q/k/v (and gate/up) along M before packing.

Here the same unpacking runs with torch ops on the tensors' device (one-time
conversion) and writes the plain wire the kernels stream (tile_m = 1: per row
``[K payload bytes | K/G bf16 scales]``, ``quantize_to_wire``'s format), so a loaded
checkpoint runs every decode path unchanged: the weight integers are the
checkpoint's, no re-quantisation.  The reference's other two wires come out too, for
callers of the IRON-shaped operators that pass them: the per-core tile wire
(``gptq_stack_to_wire`` with tile_m > 1) and fuse_o's tile-major Wo
(``gptq_wo_tile_major``).
"""

from __future__ import annotations

import torch

from .qwen3 import Qwen3Config, Qwen3Weights, quantize_to_wire, wire_nbytes

GROUPS = (32, 64, 128)


def gptq_group(qweight: torch.Tensor, scales: torch.Tensor) -> int:
    """Group size along K of a GPTQ tensor pair (K = 4 x qweight rows)."""
    K = 4 * qweight.shape[0]
    if scales.dim() != 2 or scales.shape[1] != qweight.shape[1] or scales.shape[0] == 0 or K % scales.shape[0]:
        raise ValueError(f"gptq: scales {tuple(scales.shape)} do not match qweight {tuple(qweight.shape)}")
    G = K // scales.shape[0]
    if G not in GROUPS:
        raise ValueError(f"gptq: group {G} not in {GROUPS}")
    return G


def gptq_rows(qweight: torch.Tensor, scales: torch.Tensor, domain: int = 0):
    """(K/4, M) packed words + (K/G, M) fp16 scales -> ((M, K) uint8 payload bytes,
    (M, K/G) bf16 scales).  domain 0: signed bytes (q); 1: biased bytes (q + 128)."""
    if qweight.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"gptq: qweight must be 32-bit words, got {qweight.dtype}")
    if domain not in (0, 1):
        raise ValueError(f"gptq: domain must be 0 (signed) or 1 (biased), got {domain}")
    gptq_group(qweight, scales)
    K4, M = qweight.shape
    qw = qweight.view(torch.int32)
    shifts = torch.tensor([0, 8, 16, 24], dtype=torch.int32, device=qw.device)
    u = ((qw[:, :, None] >> shifts) & 0xFF).to(torch.uint8)   # (K/4, M, 4): byte j of each word
    payload = u.permute(1, 0, 2).reshape(M, 4 * K4)           # row m, column 4r + j
    if domain == 0:
        payload = payload ^ 0x80                               # (u - 128) mod 256
    sc = scales.to(torch.float32).to(torch.bfloat16).t().contiguous()
    return payload.contiguous(), sc


def gptq_to_wire(qweight: torch.Tensor, scales: torch.Tensor, domain: int = 0) -> torch.Tensor:
    """One GPTQ projection as a plain wire (uint8, M x (K + 2K/G) bytes, on the tensors' device)."""
    payload, sc = gptq_rows(qweight, scales, domain)
    M = payload.shape[0]
    return torch.cat([payload, sc.view(torch.uint8).reshape(M, -1)], dim=1).reshape(-1)


def gptq_stack_to_wire(parts, domain: int = 0, tile_m: int = 1, cols: int = 1) -> torch.Tensor:
    """Projections sharing K stacked along M (q, k, v; as ``_set_int8``) into one wire.

    tile_m = 1: the plain wire (rows are independent, so the wire of the stack is the
    wires in order).  tile_m > 1: the per-core tile wire the fused operators take
    (``_pack_int8``, qwen3_npu_int8.py:381-405): each column's rows in tiles of tile_m
    rows, a tile being its rows' payload bytes then their scales.  The columns cover
    consecutive row ranges, so the tiles run in row order; M must split into cols
    equal ranges of whole tiles."""
    parts = list(parts)
    Ks = {4 * qw.shape[0] for qw, _ in parts}
    Gs = {gptq_group(qw, sc) for qw, sc in parts}
    if len(Ks) != 1 or len(Gs) != 1:
        raise ValueError(f"gptq: stacked projections need one K and one group, got K {Ks}, group {Gs}")
    if tile_m == 1:
        return torch.cat([gptq_to_wire(qw, sc, domain) for qw, sc in parts])
    rows = [gptq_rows(qw, sc, domain) for qw, sc in parts]
    payload = torch.cat([p for p, _ in rows])
    sc = torch.cat([s for _, s in rows])
    M = payload.shape[0]
    if tile_m < 1 or cols < 1 or M % cols or (M // cols) % tile_m:
        raise ValueError(f"gptq: {M} rows do not split into {cols} columns of {tile_m}-row tiles")
    n = M // tile_m
    return torch.cat([payload.reshape(n, -1), sc.view(torch.uint8).reshape(n, -1)], dim=1).reshape(-1)


def gptq_wo_tile_major(qweight: torch.Tensor, scales: torch.Tensor, cols: int, tile_rows: int,
                       tiles_per_core: int, domain: int = 0) -> torch.Tensor:
    """fuse_o's Wo in the per-core tile-major wire (``_set_wo_tiled``,
    qwen3_npu_int8.py:407-436): core c streams ``tiles_per_core`` tiles of
    ``tile_rows`` rows from row c * M/cols on, each tile its payload bytes then its
    scales.  A window that runs past the core's rows repeats the next core's rows, and
    past the matrix end reads pad rows with payload and scale bytes 0 (weight 0 in
    either payload domain)."""
    payload, sc = gptq_rows(qweight, scales, domain)
    M, K = payload.shape
    if cols < 1 or tile_rows < 1 or M % cols:
        raise ValueError(f"gptq: {M} rows do not split into {cols} cores")
    rpc = M // cols
    pad = tiles_per_core * tile_rows - rpc
    if pad < 0:
        raise ValueError(f"gptq: {tiles_per_core} tiles of {tile_rows} rows do not cover a core's {rpc} rows")
    sb = sc.view(torch.uint8).reshape(M, -1)
    W = torch.cat([payload, payload.new_zeros(pad, K)])
    S = torch.cat([sb, sb.new_zeros(pad, sb.shape[1])])
    dev = payload.device
    starts = (torch.arange(cols, device=dev)[:, None] * rpc
              + torch.arange(tiles_per_core, device=dev)[None, :] * tile_rows).reshape(-1)
    rows = starts[:, None] + torch.arange(tile_rows, device=dev)[None, :]  # (tiles, tile_rows)
    n = rows.shape[0]
    return torch.cat([W[rows].reshape(n, -1), S[rows].reshape(n, -1)], dim=1).reshape(-1)


def _getter(tensors):
    if hasattr(tensors, "get_tensor"):  # a safetensors safe_open handle
        return tensors.get_tensor
    return tensors.__getitem__


def load_qwen3_gptq(tensors, cfg: Qwen3Config, device="cuda", int8_lm_head: bool = False,
                    n_layers: int | None = None) -> Qwen3Weights:
    """Qwen3Weights from a GPTQ int8 checkpoint's tensors (the names of
    qwen3_npu_int8.py:152-178; ``tensors``: a safetensors handle or a name -> tensor
    mapping).  Projections become signed plain wires; norms and the tied embedding
    bf16.  ``int8_lm_head`` RTN-quantises the embedding for the int8 lm_head (on CUDA).
    Shapes are checked against ``cfg``; ValueError on a mismatch."""
    get = _getter(tensors)
    nl = cfg.n_layers if n_layers is None else n_layers

    def bf16(name, n):
        t = get(name)
        if t.numel() != n:
            raise ValueError(f"gptq: {name} has {t.numel()} values, expected {n}")
        return t.to(device=device).to(torch.bfloat16).reshape(n).contiguous()

    def proj(name, M, K):
        qw, sc = get(f"{name}.qweight"), get(f"{name}.scales")
        if tuple(qw.shape) != (K // 4, M):
            raise ValueError(f"gptq: {name}.qweight {tuple(qw.shape)}, expected {(K // 4, M)}")
        return qw.to(device), sc.to(device)

    layers, group = [], None
    for i in range(nl):
        L = f"model.layers.{i}"
        qkv = [proj(f"{L}.self_attn.{p}_proj", M, cfg.D)
               for p, M in (("q", cfg.QD), ("k", cfg.Hkv * cfg.HD), ("v", cfg.Hkv * cfg.HD))]
        o = proj(f"{L}.self_attn.o_proj", cfg.D, cfg.QD)
        g = proj(f"{L}.mlp.gate_proj", cfg.FF, cfg.D)
        u = proj(f"{L}.mlp.up_proj", cfg.FF, cfg.D)
        d = proj(f"{L}.mlp.down_proj", cfg.D, cfg.FF)
        groups = {gptq_group(*t) for t in (*qkv, o, g, u, d)}
        if len(groups) != 1 or (group is not None and groups != {group}):
            raise ValueError(f"gptq: layer {i} mixes group sizes {groups} (model group {group})")
        group = groups.pop()
        layers.append({
            "norm1": bf16(f"{L}.input_layernorm.weight", cfg.D),
            "wqkv": gptq_stack_to_wire(qkv),
            "qn": bf16(f"{L}.self_attn.q_norm.weight", cfg.HD),
            "kn": bf16(f"{L}.self_attn.k_norm.weight", cfg.HD),
            "wo": gptq_to_wire(*o),
            "norm2": bf16(f"{L}.post_attention_layernorm.weight", cfg.D),
            "wg": gptq_to_wire(*g),
            "wu": gptq_to_wire(*u),
            "wd": gptq_to_wire(*d),
        })
        assert layers[-1]["wqkv"].numel() == wire_nbytes(cfg.QKV, cfg.D, group)
    final_norm = bf16("model.norm.weight", cfg.D)
    embed = get("model.embed_tokens.weight")
    if tuple(embed.shape) != (cfg.V, cfg.D):
        raise ValueError(f"gptq: model.embed_tokens.weight {tuple(embed.shape)}, expected {(cfg.V, cfg.D)}")
    embed = embed.to(device=device).to(torch.bfloat16).contiguous()
    lm = quantize_to_wire(embed, group) if int8_lm_head else None
    return Qwen3Weights(cfg, group, layers, final_norm, embed, lm)
