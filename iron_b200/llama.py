"""Batched bf16 Llama decode on the B200 (Llama-3.2-1B shape, many ragged streams per GPU).

IRON runs Llama-3.2-1B on the NPU through bf16 operators (iron/applications/
llama_3.2_1b/llama_npu.py) and on the CPU through llama_cpu.py.  Here one GPU
decodes ``batch`` independent streams, each at its own position (ragged K/V
lengths), with the chained operator kernels replayed as one CUDA graph per step:

  embedding -> per layer: RMSNorm (the Llama form, iron_rmsnorm mode 2), QKV
  projection (bf16 weights), RoPE + K/V cache write, GQA decode attention over each
  stream's own length, O projection,
  residual add, RMSNorm, gate and up projections, SiLU, multiply, down projection,
  residual add -> final RMSNorm -> tied lm_head + greedy argmax -> positions += 1.

From 16 streams on every projection (and the lm_head) is one tcgen05 tensor-core
contraction that streams the weight once (``iron_gemv_bf16`` /
``iron_lm_head_bf16_argmax``).  Several GPUs run independent replicas (data
parallel, one process each): the streams do not share anything.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call as abi, ptr
from .qwen3 import rope_angle_table


@dataclass(frozen=True)
class LlamaConfig:
    D: int = 2048
    FF: int = 8192
    Hq: int = 32
    Hkv: int = 8
    HD: int = 64
    V: int = 128256
    n_layers: int = 16
    eps: float = 1e-5
    theta: float = 5e5

    @property
    def QD(self) -> int:
        return self.Hq * self.HD

    @property
    def QKV(self) -> int:
        return (self.Hq + 2 * self.Hkv) * self.HD

    @classmethod
    def llama_3_2_1b(cls):
        return cls()


class LlamaWeights:
    """Device-resident bf16 Llama weights: per layer norm1, wqkv (q, k, v stacked), wo,
    norm2, wg, wu, wd; final_norm; the tied embedding / lm_head."""

    def __init__(self, cfg: LlamaConfig, layers: list, final_norm, embed):
        self.cfg, self.layers, self.final_norm, self.embed = cfg, layers, final_norm, embed

    @classmethod
    def synthetic(cls, cfg: LlamaConfig, seed: int = 0, device="cuda", n_layers: int | None = None):
        """Seeded synthetic weights: projections and the embedding N(0, 0.02), RMSNorm
        weights 1 + N(0, 0.1), all bf16."""
        g = torch.Generator(device=device).manual_seed(seed)

        def randn(*shape, std=1.0, mean=0.0):
            return (torch.randn(*shape, generator=g, device=device) * std + mean).to(torch.bfloat16)

        layers = []
        for _ in range(cfg.n_layers if n_layers is None else n_layers):
            layers.append({"norm1": randn(cfg.D, std=0.1, mean=1.0), "wqkv": randn(cfg.QKV, cfg.D, std=0.02),
                           "wo": randn(cfg.D, cfg.QD, std=0.02), "norm2": randn(cfg.D, std=0.1, mean=1.0),
                           "wg": randn(cfg.FF, cfg.D, std=0.02), "wu": randn(cfg.FF, cfg.D, std=0.02),
                           "wd": randn(cfg.D, cfg.FF, std=0.02)})
        final_norm = randn(cfg.D, std=0.1, mean=1.0)
        embed = randn(cfg.V, cfg.D, std=0.02)
        torch.cuda.synchronize()
        return cls(cfg, layers, final_norm, embed)

    def to_numpy(self, n_layers: int | None = None) -> dict:
        """Host copies in the layout of ``oracle.llama.OracleLlama`` (test use)."""
        def f(t):
            return t.float().cpu().numpy()

        return {"layers": [{k: f(v) for k, v in L.items()} for L in self.layers[:n_layers]],
                "final_norm": f(self.final_norm), "embed": f(self.embed)}


class LlamaB200:
    """Greedy Llama decoder over ``batch`` independent streams on one GPU, each stream at
    its own position.  ``step_tokens(tokens, positions)`` runs one decode step and
    returns the next tokens; ``run_step`` replays the captured step with the tokens and
    positions already on the device (the argmax feeds the next step)."""

    def __init__(self, weights: LlamaWeights, max_seq: int, batch: int = 1, use_graph: bool = True,
                 keep_logits: bool = False, device="cuda"):
        c = weights.cfg
        self.cfg, self.w, self.max_seq, self.B, self.use_graph = c, weights, max_seq, batch, use_graph
        dev = torch.device(device)
        B, L = batch, len(weights.layers)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x, self.xn, self.x1 = (torch.zeros(B, c.D, **bf) for _ in range(3))
        self.raw = torch.zeros(B, c.QKV, **bf)
        self.q, self.attn = torch.zeros(B, c.QD, **bf), torch.zeros(B, c.QD, **bf)
        self.o = torch.zeros(B, c.D, **bf)
        self.g, self.u = torch.zeros(B, c.FF, **bf), torch.zeros(B, c.FF, **bf)
        self.kv = torch.zeros(L, B, c.Hkv, 2 * max_seq * c.HD, **bf)
        self.angles = rope_angle_table(max_seq, c.HD, c.theta).to(dev)
        self.logits = torch.zeros(B, c.V, **bf) if keep_logits else None
        self.params = torch.zeros(4, B, dtype=torch.int32, device=dev)
        self.params[2] = 1
        self.tok, self.pos, self.len, self.off = self.params[0], self.params[1], self.params[2], self.params[3]
        self.attn_ws = torch.empty(_lib.lib().iron_decode_attn_workspace_bytes(B, c.Hq, c.HD, max_seq),
                                   dtype=torch.uint8, device=dev)
        # scratch of the 16+ stream tensor-core projections (one at a time on the decoder
        # stream: one shared workspace) and of the lm_head + argmax
        self.tc_ws = _lib.tc_workspace([(c.QKV, c.D), (c.D, c.QD), (c.FF, c.D), (c.D, c.FF)], B, dev)
        self.head_ws = _lib.tc_workspace([(c.V, c.D)], B, dev, lm_head=True)
        self.stream = torch.cuda.Stream(device=dev)
        self._graphs: dict = {}
        self._step_launches: dict = {}  # advance -> kernels one step launched
        # below 16 streams no tensor-core projection runs: no status words to read
        status = [_lib.status_word(self.tc_ws), _lib.status_word(self.head_ws)] if B >= 16 else []
        self.io = _lib.StepIO(self.params, self.tok, status, c.HD, self.stream)

    def launches_per_step(self, advance: bool = True) -> int:
        """Our kernels per step, as the library counted them over the last eager or captured
        step; before any, the count at 16+ streams: embedding; per layer 2 RMSNorms, 5
        projections, RoPE, attention split + combine, 2 adds, SiLU, multiply; final
        RMSNorm, lm_head + 2 argmax passes; the position advance."""
        counted = self._step_launches.get(advance)
        if counted is not None:  # counted by the library over an eager or captured step
            return counted
        return 1 + 15 * len(self.w.layers) + 1 + 3 + int(advance)

    def _launch_counted(self, advance: bool, st: int):
        """_launch_step with the library's launch count taken around it."""
        c0 = _lib.launch_count()
        self._launch_step(advance, st)
        self._step_launches[advance] = _lib.launch_count() - c0

    def _launch_step(self, advance: bool, st: int):
        c, w, B = self.cfg, self.w, self.B
        tw = (ptr(self.tc_ws), self.tc_ws.numel())
        abi("iron_embedding", ptr(w.embed), c.V, ptr(self.tok), B, c.D, ptr(self.x), st)
        for i, Lw in enumerate(w.layers):
            kv = self.kv[i]
            abi("iron_rmsnorm", ptr(self.x), ptr(Lw["norm1"]), ptr(self.xn), B, c.D, c.eps, 2, st)
            abi("iron_gemv_bf16", ptr(Lw["wqkv"]), c.QKV, c.D, ptr(self.xn), B, 0, ptr(self.raw), *tw, st)
            abi("iron_rope_kv", ptr(self.raw), ptr(self.angles), ptr(self.q), ptr(kv), c.HD, c.Hq, c.Hkv,
                self.max_seq, B, ptr(self.off), st)
            abi("iron_decode_attn", ptr(self.q), ptr(kv), ptr(self.attn), B, c.Hq, c.Hkv, c.HD, self.max_seq,
                0, 0, 1, ptr(self.len), ptr(self.attn_ws), self.attn_ws.numel(), st)
            abi("iron_gemv_bf16", ptr(Lw["wo"]), c.D, c.QD, ptr(self.attn), B, 0, ptr(self.o), *tw, st)
            abi("iron_add", ptr(self.x), ptr(self.o), ptr(self.x1), B * c.D, st)
            abi("iron_rmsnorm", ptr(self.x1), ptr(Lw["norm2"]), ptr(self.xn), B, c.D, c.eps, 2, st)
            abi("iron_gemv_bf16", ptr(Lw["wg"]), c.FF, c.D, ptr(self.xn), B, 0, ptr(self.g), *tw, st)
            abi("iron_gemv_bf16", ptr(Lw["wu"]), c.FF, c.D, ptr(self.xn), B, 0, ptr(self.u), *tw, st)
            abi("iron_silu", ptr(self.g), ptr(self.g), B * c.FF, 0, st)
            abi("iron_mul", ptr(self.g), ptr(self.u), ptr(self.g), B * c.FF, st)
            abi("iron_gemv_bf16", ptr(Lw["wd"]), c.D, c.FF, ptr(self.g), B, 0, ptr(self.o), *tw, st)
            abi("iron_add", ptr(self.x1), ptr(self.o), ptr(self.x), B * c.D, st)
        abi("iron_rmsnorm", ptr(self.x), ptr(w.final_norm), ptr(self.xn), B, c.D, c.eps, 2, st)
        abi("iron_lm_head_bf16_argmax", ptr(w.embed), c.V, c.D, ptr(self.xn), B,
            None if self.logits is None else ptr(self.logits), ptr(self.tok), ptr(self.head_ws),
            self.head_ws.numel(), st)
        if advance:
            abi("iron_decode_advance", ptr(self.pos), ptr(self.len), ptr(self.off), B, c.HD, st)

    def run_step(self, advance: bool = True):
        """Enqueue one decode step on ``self.stream`` (graph replay when enabled)."""
        st = self.stream
        with torch.cuda.stream(st):
            if not self.use_graph:
                self._launch_counted(advance, st.cuda_stream)
                return
            g = self._graphs.get(advance)
            if g is None:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    self._launch_counted(advance, st.cuda_stream)
                self._graphs[advance] = g
            g.replay()

    def set_positions(self, pos):
        """Host write of the per-stream positions (int or B ints)."""
        p = torch.as_tensor(pos, dtype=torch.int32).reshape(-1).expand(self.B).clone()
        with torch.cuda.stream(self.stream):
            self.pos.copy_(p.to(self.pos.device))
            self.len.copy_(self.pos + 1)
            self.off.copy_(self.pos * (2 * self.cfg.HD))

    def step_tokens(self, tokens, pos) -> torch.Tensor:
        """One step for the B streams from token ids at positions ``pos`` -> next tokens (host)."""
        self.io.put(tokens, pos)  # tokens, positions, lengths, K/V offsets: one copy
        self.run_step(advance=False)
        out = self.io.get()
        B = self.B
        code = int(out[B]) or int(out[B + 1]) if B >= 16 else 0
        if code:
            self.tc_ws[:4].zero_()
            self.head_ws[:4].zero_()
            _lib.raise_on_status(code, "decode step")
        return torch.from_numpy(out[:B].copy())
