"""Qwen3 decode runtime on the B200 (the counterpart of IRON's ``Qwen3NPU``).

IRON's runtime (iron/applications/qwen3_0.6b/qwen3_npu_int8.py:129-621) packs
int8 weights into tile wires, builds one OperatorSequence of
``[QKV head, decode attention, fused MLP] x 28 + RMSNorm + lm_head`` and, per
token, writes ``x``, the RoPE row, ``k_cache_offset`` and ``S_kv_eff`` then
dispatches once and argmaxes the logits on the host.  Here the same chain is
launched through the C ABI and captured in one CUDA graph per step shape; the
positions live in device memory (advanced on the device after each step), the
RoPE row is selected on the device from the angle table, and the greedy argmax
runs in the lm_head epilogue, so a decode step needs no host traffic beyond
the 4-byte token it returns.

Weights use the native wire (row-interleaved ``[K int8 | K/G bf16]``, signed
payload) with quant group ``group`` (32 by default; the reference's checkpoint uses 128).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import call as abi, ptr


@dataclass(frozen=True)
class Qwen3Config:
    D: int = 1024
    FF: int = 3072
    Hq: int = 16
    Hkv: int = 8
    HD: int = 128
    V: int = 151936
    n_layers: int = 28
    eps: float = 1e-6
    theta: float = 1e6

    @property
    def QD(self) -> int:
        return self.Hq * self.HD

    @property
    def QKV(self) -> int:
        return (self.Hq + 2 * self.Hkv) * self.HD

    @classmethod
    def qwen3_0_6b(cls):
        return cls()

    @classmethod
    def qwen3_8b(cls):
        return cls(D=4096, FF=12288, Hq=32, Hkv=8, HD=128, V=151936, n_layers=36)


def wire_nbytes(M: int, K: int, group: int) -> int:
    return M * (K + 2 * (K // group))


def quantize_to_wire(w_bf16: torch.Tensor, group: int, tile_m: int = 1, domain: int = 0) -> torch.Tensor:
    """RTN int8 quantise a (M, K) bf16 CUDA tensor into a plain wire (uint8 CUDA tensor)."""
    M, K = w_bf16.shape
    out = torch.empty(wire_nbytes(M, K, group), dtype=torch.uint8, device=w_bf16.device)
    abi("iron_quantize_rtn", ptr(w_bf16.contiguous()), M, K, group, tile_m, domain, ptr(out),
        _lib.stream_ptr())
    return out


def wire_to_numpy(wire: torch.Tensor, M: int, K: int, group: int):
    """(q int8 (M,K), scale_bits uint16 (M,K/G)) host copies of a tile_m=1 signed wire."""
    b = wire.cpu().numpy().reshape(M, K + 2 * (K // group))
    return b[:, :K].view(np.int8).copy(), b[:, K:].copy().view(np.uint16)


def rope_angle_table(max_seq: int, head_dim: int, theta: float) -> torch.Tensor:
    """Interleaved half-dim [cos, sin] rows, bf16 (Qwen3NPU._precompute_rope_angles,
    qwen3_npu_int8.py:580-591): float32 angles, cos/sin rounded to bf16."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    t = torch.arange(max_seq, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos().to(torch.bfloat16)
    sin = freqs.sin().to(torch.bfloat16)
    return torch.stack([cos, sin], dim=-1).reshape(max_seq, head_dim)


class Qwen3Weights:
    """Device-resident Qwen3 weights in the native int8 wire (tile_m = 1, signed)."""

    def __init__(self, cfg: Qwen3Config, group: int, layers: list, final_norm, embed, lm_wire=None):
        self.cfg, self.group = cfg, group
        self.layers, self.final_norm, self.embed, self.lm_wire = layers, final_norm, embed, lm_wire

    @classmethod
    def synthetic(cls, cfg: Qwen3Config, seed: int = 0, group: int = 32, device="cuda",
                  int8_lm_head: bool = False, n_layers: int | None = None):
        """Seeded synthetic weights (no checkpoint needed): projection masters
        N(0, 0.02) -> int8 RTN per group; RMSNorm weights 1 + N(0, 0.1); tied bf16
        embedding N(0, 0.02)."""
        g = torch.Generator(device=device).manual_seed(seed)
        nl = cfg.n_layers if n_layers is None else n_layers

        def randn(*shape, std=1.0, mean=0.0):
            return (torch.randn(*shape, generator=g, device=device) * std + mean).to(torch.bfloat16)

        def qw(M, K):
            return quantize_to_wire(randn(M, K, std=0.02), group)

        layers = []
        for _ in range(nl):
            L = {"norm1": randn(cfg.D, std=0.1, mean=1.0)}
            L["wqkv"] = qw(cfg.QKV, cfg.D)
            L["qn"] = randn(cfg.HD, std=0.1, mean=1.0)
            L["kn"] = randn(cfg.HD, std=0.1, mean=1.0)
            L["wo"] = qw(cfg.D, cfg.QD)
            L["norm2"] = randn(cfg.D, std=0.1, mean=1.0)
            L["wg"] = qw(cfg.FF, cfg.D)
            L["wu"] = qw(cfg.FF, cfg.D)
            L["wd"] = qw(cfg.D, cfg.FF)
            layers.append(L)
        final_norm = randn(cfg.D, std=0.1, mean=1.0)
        embed = randn(cfg.V, cfg.D, std=0.02)
        lm = quantize_to_wire(embed, group) if int8_lm_head else None
        torch.cuda.synchronize()
        return cls(cfg, group, layers, final_norm, embed, lm)

    def weight_bytes(self) -> int:
        per = sum(t.numel() * t.element_size() for t in self.layers[0].values())
        return per * len(self.layers)

    def to_numpy(self, n_layers: int | None = None) -> dict:
        """Host copies in the layout of ``oracle.qwen3.OracleQwen3`` (test use)."""
        c, G = self.cfg, self.group

        def f(t):
            return t.float().cpu().numpy()

        out = {"layers": []}
        for L in self.layers[:n_layers]:
            d = {"norm1": f(L["norm1"]), "qn": f(L["qn"]), "kn": f(L["kn"]), "norm2": f(L["norm2"])}
            for name, (M, K) in (("wqkv", (c.QKV, c.D)), ("wo", (c.D, c.QD)), ("wg", (c.FF, c.D)),
                                 ("wu", (c.FF, c.D)), ("wd", (c.D, c.FF))):
                d[name + "_q"], d[name + "_s"] = wire_to_numpy(L[name], M, K, G)
            out["layers"].append(d)
        out["final_norm"] = f(self.final_norm)
        out["embed"] = f(self.embed)
        if self.lm_wire is not None:
            out["lm_q"], out["lm_s"] = wire_to_numpy(self.lm_wire, c.V, c.D, G)
        return out


class _StepLayer(C.Structure):
    """iron_qwen3_layer (include/iron_b200.h)."""
    _fields_ = [(n, C.c_void_p) for n in ("norm1", "wqkv", "qn", "kn", "wo", "norm2", "wg", "wu", "wd",
                                          "wqkv_t", "wo_t", "wgu_t", "wd_t")]


class _StepModel(C.Structure):
    """iron_qwen3_model (include/iron_b200.h)."""
    _fields_ = ([(n, C.c_int) for n in ("D", "FF", "Hq", "Hkv", "HD", "V", "n_layers", "group", "max_seq")]
                + [("eps", C.c_float)]
                + [(n, C.c_void_p) for n in ("layers", "final_norm", "embed", "lm_w8", "angles", "kv", "x", "raw",
                                             "attn", "x1", "gh", "attn_ws", "cand", "tok", "pos", "seq_len",
                                             "kv_off", "logits", "sync", "trace")])


def _one(v) -> int:
    """The single value of an int or a one-element sequence / array."""
    if isinstance(v, int):
        return v
    a = np.asarray(v).reshape(-1)
    if a.size != 1:
        raise ValueError(f"the batch-1 step takes one value (got {a.size})")
    return int(a[0])


class Qwen3B200:
    """Greedy Qwen3 decoder over ``batch`` independent streams on one GPU.

    ``__call__(x, seq_pos)`` keeps Qwen3NPU's interface (qwen3_npu_int8.py:594-621):
    hidden state of the new token in, greedy token id out.  ``step_tokens`` feeds
    token ids through the embedding; ``generate`` prefills a prompt token by token
    (as check_cosine_int8.py:51-52 does) and then decodes greedily."""

    def __init__(self, weights: Qwen3Weights, max_seq: int, batch: int = 1, lm_head: str = "bf16",
                 use_graph: bool = True, keep_logits: bool = False, device="cuda", impl: str | None = None):
        cfg = weights.cfg
        self.cfg, self.w, self.max_seq, self.B = cfg, weights, max_seq, batch
        if lm_head not in ("bf16", "int8"):
            raise ValueError("lm_head must be 'bf16' or 'int8'")
        if lm_head == "int8" and weights.lm_wire is None:
            raise ValueError("int8 lm_head requested but the weights carry no lm_head wire")
        if lm_head == "int8" or keep_logits:
            keep_logits = True
        self.lm_head, self.use_graph = lm_head, use_graph
        dev = torch.device(device)
        B, L = batch, len(weights.layers)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(B, cfg.D, **bf)
        self.xf = torch.zeros(B, cfg.D, **bf)
        self.q = torch.zeros(B, cfg.QD, **bf)
        self.raw = torch.zeros(B, cfg.QKV, **bf)
        self.attn = torch.zeros(B, cfg.QD, **bf)
        self.x1 = torch.zeros(B, cfg.D, **bf)
        self.gh = torch.zeros(B, cfg.FF, **bf)
        self.kv = torch.zeros(L, B, cfg.Hkv, 2 * max_seq * cfg.HD, **bf)
        self.angles = rope_angle_table(max_seq, cfg.HD, cfg.theta).to(dev)
        self.logits = torch.zeros(B, cfg.V, **bf) if keep_logits else None
        # device params: token ids, positions, valid lengths, KV element offsets (one
        # tensor so that a step's (token, position) input is a single 8-byte copy)
        self.params = torch.zeros(4, B, dtype=torch.int32, device=dev)
        self.params[2] = 1
        self.tok, self.pos, self.len, self.off = self.params[0], self.params[1], self.params[2], self.params[3]
        self.host_params = torch.zeros(2, B, dtype=torch.int32, pin_memory=True)
        self.attn_ws = torch.empty(_lib.lib().iron_decode_attn_workspace_bytes(B, cfg.Hq, cfg.HD, max_seq),
                                   dtype=torch.uint8, device=dev)
        # scratch of the batch 16+ tensor-core projections (run one at a time on the
        # decoder stream, so they share one) and of the lm_head + argmax; each starts
        # with a status word that _read_tokens brings back with the tokens
        self.tc_ws = _lib.tc_workspace([(cfg.QKV, cfg.D), (cfg.D, cfg.QD), (cfg.FF, cfg.D), (cfg.D, cfg.FF)],
                                       B, dev)
        self.head_ws = _lib.tc_workspace([(cfg.V, cfg.D)], B, dev, lm_head=True)
        self.stream = torch.cuda.Stream(device=dev)
        self._graphs: dict[bool, torch.cuda.CUDAGraph] = {}
        self._step_launches: dict = {}  # (from_tokens, advance) -> kernels one step launched
        # "step": the whole token in one persistent kernel (batch 1);
        # "ops": the chained per-operator kernels, replayed as a CUDA graph
        self.impl = impl or ("step" if batch == 1 else "ops")
        if self.impl not in ("step", "ops"):
            raise ValueError("impl must be 'step' or 'ops'")
        if self.impl == "step":
            if batch != 1:
                raise ValueError("the persistent step kernel decodes one stream (batch 1)")
            self._init_step(dev)
        else:  # below 16 streams no tensor-core projection runs: no status words to read
            status = [_lib.status_word(self.tc_ws), _lib.status_word(self.head_ws)] if B >= 16 else []
            self.io = _lib.StepIO(self.params, self.tok, status, cfg.HD, self.stream)

    def _pack_tiles(self, wire, M, K_full, col0, K, dev, st, out=None):
        """16-row tiles of rows [0, M), columns [col0, col0 + K) of a plain wire
        (iron_qwen3_pack_tiles); into ``out`` when given."""
        G = self.w.group
        n = _lib.lib().iron_qwen3_tiles_bytes(M, K, G)
        if out is None:
            out = torch.empty(n, dtype=torch.uint8, device=dev)
        abi("iron_qwen3_pack_tiles", ptr(wire), K_full + 2 * (K_full // G), M, K_full, col0, K, G, ptr(out), st)
        return out

    def _qkv_group_rows(self) -> torch.Tensor:
        """Row order of the step kernel's QKV tiles: per KV head h the q rows of its
        query heads, then its k rows, then its v rows."""
        c = self.cfg
        GQ, HD = c.Hq // c.Hkv, c.HD
        rows = []
        for h in range(c.Hkv):
            rows.append(torch.arange(h * GQ * HD, (h + 1) * GQ * HD))
            rows.append(torch.arange(c.QD + h * HD, c.QD + (h + 1) * HD))
            rows.append(torch.arange(c.QD + c.Hkv * HD + h * HD, c.QD + c.Hkv * HD + (h + 1) * HD))
        return torch.cat(rows)

    def _init_step(self, dev):
        c, w = self.cfg, self.w
        L = _lib.lib()
        G = w.group
        st = torch.cuda.current_stream(dev).cuda_stream
        # the step kernel's weight tiles (made once; the plain wires stay for the other paths)
        perm = self._qkv_group_rows().to(dev)
        self._step_packed = []
        layers = (_StepLayer * len(w.layers))()
        for i, Lw in enumerate(w.layers):
            for n in ("norm1", "wqkv", "qn", "kn", "wo", "norm2", "wg", "wu", "wd"):
                if ptr(Lw[n]) % 16:  # the kernel bulk-copies weights: 16-byte aligned bases
                    raise ValueError(f"layer {i} {n}: device pointer not 16-byte aligned")
                setattr(layers[i], n, ptr(Lw[n]))
            qkv_rows = Lw["wqkv"].view(c.QKV, -1).index_select(0, perm).contiguous()
            wqkv_t = self._pack_tiles(qkv_rows, c.QKV, c.D, 0, c.D, dev, st)
            wo_t = self._pack_tiles(Lw["wo"], c.D, c.QD, 0, c.QD, dev, st)
            # gate/up: tile t = gate rows 8t..8t+7 over up rows 8t..8t+7
            gu_rows = torch.stack([Lw["wg"].view(c.FF // 8, 8, -1), Lw["wu"].view(c.FF // 8, 8, -1)], 1)
            gu_rows = gu_rows.reshape(2 * c.FF, -1).contiguous()
            wgu_t = self._pack_tiles(gu_rows, 2 * c.FF, c.D, 0, c.D, dev, st)
            # down: the 4 column slices of every 16-row tile, tile-major
            ks = c.FF // 4
            sl = [self._pack_tiles(Lw["wd"], c.D, c.FF, j * ks, ks, dev, st).view(c.D // 16, -1) for j in range(4)]
            wd_t = torch.stack(sl, 1).reshape(-1).contiguous()
            torch.cuda.current_stream(dev).synchronize()  # the row copies are released below
            del qkv_rows, gu_rows, sl
            self._step_packed.append((wqkv_t, wo_t, wgu_t, wd_t))
            layers[i].wqkv_t, layers[i].wo_t = ptr(wqkv_t), ptr(wo_t)
            layers[i].wgu_t, layers[i].wd_t = ptr(wgu_t), ptr(wd_t)
        self._lm_tiles = None
        if self.lm_head == "int8":
            self._lm_tiles = self._pack_tiles(w.lm_wire, c.V, c.D, 0, c.D, dev, st)
        torch.cuda.current_stream(dev).synchronize()
        if ptr(w.embed) % 16:
            raise ValueError("embed: device pointer not 16-byte aligned")
        self._layer_table = torch.frombuffer(bytearray(bytes(layers)), dtype=torch.uint8).to(dev)
        m = _StepModel()
        m.D, m.FF, m.Hq, m.Hkv, m.HD, m.V = c.D, c.FF, c.Hq, c.Hkv, c.HD, c.V
        m.n_layers, m.group, m.max_seq, m.eps = len(w.layers), w.group, self.max_seq, c.eps
        m.layers = ptr(self._layer_table)
        m.final_norm, m.embed = ptr(w.final_norm), ptr(w.embed)
        m.lm_w8 = ptr(self._lm_tiles) if self._lm_tiles is not None else None
        m.angles, m.kv = ptr(self.angles), ptr(self.kv)
        m.x, m.raw, m.attn, m.x1, m.gh = ptr(self.x), ptr(self.raw), ptr(self.attn), ptr(self.x1), ptr(self.gh)
        mp = C.byref(m)
        self.step_ws = torch.zeros(L.iron_qwen3_attn_ws_bytes(mp), dtype=torch.uint8, device=dev)
        self.cand = torch.empty(L.iron_qwen3_cand_bytes(), dtype=torch.uint8, device=dev)
        self.sync = torch.zeros(L.iron_qwen3_sync_words(mp), dtype=torch.int32, device=dev)
        m.attn_ws, m.cand = ptr(self.step_ws), ptr(self.cand)
        m.tok, m.pos, m.seq_len, m.kv_off = ptr(self.tok), ptr(self.pos), ptr(self.len), ptr(self.off)
        m.logits = ptr(self.logits) if self.logits is not None else None
        m.sync = ptr(self.sync)
        m.trace = None
        self._model = m
        self._mref = C.byref(m)
        # host side of step_tokens: {token, position | next token, error word}, pinned
        self._host_io = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        self._host_np = self._host_io.numpy()
        self._host_in = self._host_io.data_ptr()
        self._host_out = self._host_in + 8
        self._step_host = L.iron_qwen3_step_host

    def enable_trace(self) -> torch.Tensor:
        """Step kernel only: record the hidden state entering every layer and the final
        one, (n_layers + 1, D) bf16, on every following step (parity checks)."""
        if self.impl != "step":
            raise ValueError("the layer trace is recorded by the persistent step kernel")
        self.trace = torch.zeros(len(self.w.layers) + 1, self.cfg.D, dtype=torch.bfloat16, device=self.x.device)
        self._model.trace = ptr(self.trace)
        return self.trace

    def check(self):
        """Raise if a persistent step timed out on one of its bounded waits."""
        if self.impl == "step":
            err = int(self.sync[1].item())
            if err:
                abi("iron_qwen3_sync_reset", C.byref(self._model), self.stream.cuda_stream)
                raise RuntimeError(f"decode step aborted on a bounded device wait (code {err})")

    # ---- the step, as a flat list of ABI launches ----
    def _launch_step(self, from_tokens: bool, advance: bool, st: int):
        c, w, B = self.cfg, self.w, self.B
        G = w.group
        if from_tokens:
            abi("iron_embedding", ptr(w.embed), c.V, ptr(self.tok), B, c.D, ptr(self.x), st)
        for i, Lw in enumerate(w.layers):
            kv = self.kv[i]
            abi("iron_qkv_head", ptr(self.x), ptr(Lw["norm1"]), ptr(Lw["wqkv"]), G, 1, 0, ptr(Lw["qn"]),
                ptr(Lw["kn"]), ptr(self.angles), 1, ptr(self.q), ptr(kv), c.D, c.HD, c.Hq, c.Hkv,
                self.max_seq, B, 0, ptr(self.off), c.eps, 1, ptr(self.raw), ptr(self.tc_ws),
                self.tc_ws.numel(), st)
            abi("iron_decode_attn", ptr(self.q), ptr(kv), ptr(self.attn), B, c.Hq, c.Hkv, c.HD,
                self.max_seq, 0, 0, 1, ptr(self.len), ptr(self.attn_ws), self.attn_ws.numel(), st)
            abi("iron_mlp_block", ptr(self.x), ptr(self.attn), 1, ptr(Lw["norm2"]), ptr(Lw["wo"]), 1, 0, 0,
                ptr(Lw["wg"]), ptr(Lw["wu"]), 1, ptr(Lw["wd"]), 1, G, 0, ptr(self.x1), ptr(self.gh),
                ptr(self.x), c.D, c.FF, c.QD, B, c.eps, ptr(self.tc_ws), self.tc_ws.numel(), st)
        abi("iron_rmsnorm", ptr(self.x), ptr(w.final_norm), ptr(self.xf), B, c.D, c.eps, 1, st)
        if self.lm_head == "bf16":
            abi("iron_lm_head_bf16_argmax", ptr(w.embed), c.V, c.D, ptr(self.xf), B, ptr(self.logits),
                ptr(self.tok), ptr(self.head_ws), self.head_ws.numel(), st)
        else:
            abi("iron_lm_head_w8_argmax", ptr(w.lm_wire), c.V, c.D, G, ptr(self.xf), B, ptr(self.logits),
                ptr(self.tok), ptr(self.head_ws), self.head_ws.numel(), st)
        if advance:
            abi("iron_decode_advance", ptr(self.pos), ptr(self.len), ptr(self.off), B, c.HD, st)

    def launches_per_step(self, from_tokens: bool = True, advance: bool = True) -> int:
        """Kernels one step launches, as the library counted them over the last eager or
        captured step of this kind; before any, the batch <= 8 count: embedding, 7 per
        layer (QKV GEMV + head epilogue, attention split + combine, O / gate-up / down
        GEMVs), final RMSNorm, lm_head (+ argmax passes) and the position advance."""
        if self.impl == "step":
            return 1
        counted = self._step_launches.get((from_tokens, advance))
        if counted is not None:  # counted by the library over an eager or captured step
            return counted
        head = 2 if self.lm_head == "bf16" else 3
        return int(from_tokens) + 7 * len(self.w.layers) + 1 + head + int(advance)

    def time_lm_head(self, reps: int = 20) -> float:
        """Mean duration (ms) of the lm_head GEMV + argmax on the decoder stream."""
        c, st = self.cfg, self.stream
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        args = (ptr(self.w.embed), c.V, c.D, ptr(self.xf), self.B, ptr(self.logits), ptr(self.tok),
                ptr(self.head_ws), self.head_ws.numel(), st.cuda_stream)
        for _ in range(3):
            abi("iron_lm_head_bf16_argmax", *args)
        ev[0].record(st)
        for _ in range(reps):
            abi("iron_lm_head_bf16_argmax", *args)
        ev[1].record(st)
        st.synchronize()
        return ev[0].elapsed_time(ev[1]) / reps

    def run_step(self, from_tokens: bool = True, advance: bool = True):
        """Enqueue one decode step on ``self.stream`` (graph replay when enabled)."""
        st = self.stream
        key = (from_tokens, advance)
        if self.impl == "step":
            abi("iron_qwen3_decode_step", C.byref(self._model), int(from_tokens), int(advance), st.cuda_stream)
            return
        with torch.cuda.stream(st):
            if not self.use_graph:
                self._launch_counted(key, st.cuda_stream)
                return
            g = self._graphs.get(key)
            if g is None:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    self._launch_counted(key, st.cuda_stream)
                self._graphs[key] = g
            g.replay()

    def _launch_counted(self, key, st: int):
        """_launch_step with the library's launch count taken around it."""
        c0 = _lib.launch_count()
        self._launch_step(key[0], key[1], st)
        self._step_launches[key] = _lib.launch_count() - c0

    def set_position(self, pos):
        """Host write of the per-stream positions (int or sequence of B ints)."""
        p = torch.as_tensor(pos, dtype=torch.int32).reshape(-1).expand(self.B).clone()
        with torch.cuda.stream(self.stream):
            self.pos.copy_(p.to(self.pos.device, non_blocking=False))
            self.len.copy_(self.pos + 1)
            self.off.copy_(self.pos * (2 * self.cfg.HD))

    def reset(self):
        self.kv.zero_()
        self.set_position(0)

    def _read_tokens(self) -> torch.Tensor:
        """Next tokens to the host; the persistent step's error word rides along."""
        if self.impl == "step":
            with torch.cuda.stream(self.stream):
                both = torch.cat([self.tok, self.sync[1:2]]).cpu()
            if int(both[-1]):
                self.check()
            return both[:-1]
        out = self.io.get()
        B = self.B
        code = int(out[B]) or int(out[B + 1]) if B >= 16 else 0
        if code:
            self.tc_ws[:4].zero_()
            self.head_ws[:4].zero_()
            _lib.raise_on_status(code, "decode step")
        return torch.from_numpy(out[:B].copy())

    def _put_inputs(self, tokens, pos):
        """(token, position) per stream -> device in one copy from pinned memory (the
        chained kernels' valid lengths and K/V offsets ride along)."""
        if self.impl == "ops":
            self.io.put(tokens, pos)
            return
        self.host_params[0] = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).expand(self.B)
        self.host_params[1] = torch.as_tensor(pos, dtype=torch.int32).reshape(-1).expand(self.B)
        with torch.cuda.stream(self.stream):
            self.params[0:2].copy_(self.host_params, non_blocking=True)

    def __call__(self, x, seq_pos: int) -> int:
        """Qwen3NPU.__call__: hidden state (D,) bf16 of the new token -> argmax token."""
        if self.B != 1:
            raise ValueError("__call__ is the batch-1 interface; use step_tokens for batches")
        self._put_inputs(0, seq_pos)
        with torch.cuda.stream(self.stream):
            self.x[0].copy_(torch.as_tensor(x).to(torch.bfloat16).reshape(-1), non_blocking=False)
        self.run_step(from_tokens=False, advance=False)
        return int(self._read_tokens()[0])

    def step_tokens(self, tokens, pos) -> torch.Tensor:
        """One step for B streams from token ids at positions ``pos`` -> next tokens (host)."""
        if self.impl == "step":  # one library call: copy in, the step, copy out, wait
            hn = self._host_np
            hn[0], hn[1] = _one(tokens), _one(pos)
            rc = self._step_host(self._mref, self._host_in, self._host_out, 1, self.stream.cuda_stream)
            if rc < 0:
                if int(hn[3]):
                    self.check()  # resets the hand-off words and raises
                raise _lib.IronError(f"iron_qwen3_step_host failed ({rc}): {_lib.last_error()}")
            return torch.from_numpy(hn[2:3].copy())
        self._put_inputs(tokens, pos)
        self.run_step(from_tokens=True, advance=False)
        return self._read_tokens()

    #: prompt rows per prefill block: each projection of a block is one tensor-core
    #: contraction launch (its rows in row blocks of up to 128, a second grid dimension)
    PREFILL_ROWS = 1024

    def prefill(self, prompt, stream: int = 0, start: int = 0, exact: bool = False) -> int:
        """Run the prompt ``prompt`` (token ids) of stream ``stream`` through every layer
        at once, its tokens at positions ``start`` .. ``start + len(prompt) - 1``.

        Does what the reference's prompt loop does one token at a time
        (check_cosine_int8.py:49-54: one ``Qwen3NPU.__call__`` per token): fills the K/V
        cache of those positions and returns the greedy token after the last one,
        which the stream's next step reads (its position is set to the one after the
        prompt).  Per layer, blocks of up to ``PREFILL_ROWS`` prompt rows run the
        decode step's operators as batched launches: the QKV projection with its
        RMSNorm (tcgen05 contraction from 16 rows on), the per-head q/k norms, RoPE and
        K/V writes at the rows' positions (``iron_qkv_rows``), causal attention over
        the cache (``iron_attn_mq``), and the O / gate-up / down block
        (``iron_mlp_block``).  The last row's final RMSNorm, lm_head and argmax
        follow; the logits are kept in ``self.prefill_logits``.  ``exact`` runs the
        projections with the decode step's exact kernel in launches of 8 rows instead of
        the tensor-core contraction (slower; no float32 summation in the projections)."""
        c, w, G = self.cfg, self.w, self.w.group
        ids = [int(t) for t in prompt]
        P = len(ids)
        if P < 1 or start < 0 or start + P > self.max_seq:
            raise ValueError(f"prompt of {P} tokens at {start} does not fit a {self.max_seq}-token cache")
        if not 0 <= stream < self.B:
            raise ValueError(f"stream {stream} outside the batch of {self.B}")
        dev, st = self.x.device, self.stream
        R = min(P, self.PREFILL_ROWS)
        bf = dict(dtype=torch.bfloat16, device=dev)
        x = torch.empty(P, c.D, **bf)
        raw, q, attn = torch.empty(R, c.QKV, **bf), torch.empty(R, c.QD, **bf), torch.empty(R, c.QD, **bf)
        x1, gh = torch.empty(R, c.D, **bf), torch.empty(R, c.FF, **bf)
        xf = torch.empty(1, c.D, **bf)
        L = _lib.lib()
        tw = _lib.tc_workspace([(c.QKV, c.D), (c.D, c.QD), (c.FF, c.D), (c.D, c.FF)], 1 if exact else R, dev)
        aw = _lib.workspace(L.iron_attn_mq_workspace_bytes(R, c.Hq, c.Hkv, c.HD, self.max_seq), dev)
        hw = _lib.workspace(L.iron_argmax_workspace_bytes(1), dev)
        self.prefill_logits = torch.empty(1, c.V, **bf)
        ids_dev = torch.tensor(ids, dtype=torch.int32).pin_memory()
        with torch.cuda.stream(st):
            ids_d = ids_dev.to(dev, non_blocking=True)
            s_ = st.cuda_stream
            abi("iron_embedding", ptr(w.embed), c.V, ptr(ids_d), P, c.D, ptr(x), s_)
            for li, Lw in enumerate(w.layers):
                kv = self.kv[li, stream]
                for r0 in range(0, P, R):
                    n = min(R, P - r0)
                    xr = x[r0:r0 + n]
                    abi("iron_gemv_w8a16_ex", ptr(Lw["wqkv"]), None, c.QKV, c.D, G, 0, ptr(xr), c.D, n,
                        ptr(Lw["norm1"]), c.eps, 1, None, 0, ptr(raw), c.QKV, ptr(tw), tw.numel(), s_)
                    abi("iron_qkv_rows", ptr(raw), n, ptr(Lw["qn"]), ptr(Lw["kn"]), ptr(self.angles), ptr(q),
                        ptr(kv), c.HD, c.Hq, c.Hkv, self.max_seq, start + r0, c.eps, 1, s_)
                    abi("iron_attn_mq", ptr(q), ptr(kv), ptr(attn), n, c.Hq, c.Hkv, c.HD, self.max_seq, 0, 0,
                        start + r0, None, self.max_seq, 1, ptr(aw), aw.numel(), s_)
                    abi("iron_mlp_block", ptr(xr), ptr(attn), 1, ptr(Lw["norm2"]), ptr(Lw["wo"]), 1, 0, 0,
                        ptr(Lw["wg"]), ptr(Lw["wu"]), 1, ptr(Lw["wd"]), 1, G, 0, ptr(x1), ptr(gh), ptr(xr),
                        c.D, c.FF, c.QD, n, c.eps, ptr(tw), tw.numel(), s_)
            abi("iron_rmsnorm", ptr(x[P - 1:]), ptr(w.final_norm), ptr(xf), 1, c.D, c.eps, 1, s_)
            tok = self.tok[stream:stream + 1]
            if self.lm_head == "bf16":
                abi("iron_lm_head_bf16_argmax", ptr(w.embed), c.V, c.D, ptr(xf), 1, ptr(self.prefill_logits),
                    ptr(tok), ptr(hw), hw.numel(), s_)
            else:
                abi("iron_lm_head_w8_argmax", ptr(w.lm_wire), c.V, c.D, G, ptr(xf), 1, ptr(self.prefill_logits),
                    ptr(tok), ptr(hw), hw.numel(), s_)
            status = torch.stack([_lib.status_word(tw)[0], tok[0]]).cpu()
            # the stream continues after the prompt
            nxt = start + P
            self.pos[stream].fill_(nxt)
            self.len[stream].fill_(nxt + 1)
            self.off[stream].fill_(nxt * 2 * c.HD)
        _lib.raise_on_status(int(status[0]), "prefill")
        return int(status[1])

    def generate(self, prompt, n_new: int, batched_prefill: bool = True) -> list:
        """Prefill ``prompt`` (ids, batch 1), then greedy-decode ``n_new`` tokens.

        ``batched_prefill`` runs the prompt through ``prefill`` (all rows of a layer at
        once); otherwise token by token through the decode step, as the reference's
        prompt loop.  The decode steps replay the captured step back to back: the device
        advances the position and feeds each argmax token to the next step's
        embedding; the tokens are gathered on the device and read back once."""
        if self.B != 1:
            raise ValueError("generate() is batch 1")
        if len(prompt) + n_new > self.max_seq:
            raise ValueError("prompt + new tokens exceed max_seq")
        if batched_prefill:
            self.prefill(prompt)
        else:
            for p, t in enumerate(prompt):
                self.step_tokens([t], p)
        hist = torch.empty(n_new, dtype=torch.int32, device=self.tok.device)
        self.set_position(len(prompt))
        with torch.cuda.stream(self.stream):
            hist[0].copy_(self.tok[0])
        for i in range(1, n_new):
            self.run_step(from_tokens=True, advance=True)
            with torch.cuda.stream(self.stream):
                hist[i].copy_(self.tok[0])
        self.stream.synchronize()
        self.check()
        return hist.cpu().tolist()
