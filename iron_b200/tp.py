"""Tensor-parallel Qwen3 decode: one process per GPU, NCCL or peer memory between them.

IRON decodes on one NPU; its operators have no tensor parallelism.  Here a
Qwen3 model (Qwen3-8B: 32 query / 8 KV heads, FF 12288) is split over ``world``
ranks the Megatron way, on the reference's own operator boundaries:

- QKV is column-parallel by heads: rank r holds query heads
  [r Hq/n, (r+1) Hq/n) and KV heads [r Hkv/n, (r+1) Hkv/n) of Wqkv, computes their
  q/k RMSNorm + RoPE and keeps their KV cache;
- decode attention runs on the local heads only;
- O is row-parallel (its K = the local heads' columns): each rank's float32
  partial sums are all-reduced, then x1 = bf16(x + bf16(sum));
- gate/up are column-parallel (FF/n rows each, RMSNorm of x1 in the prologue) and
  down row-parallel (K = FF/n): all-reduce, then x = bf16(x1 + bf16(sum));
- the tied lm_head is vocabulary-parallel: each rank takes the greedy argmax of
  its V/n rows, the (value, index) pairs are all-gathered and the largest wins
  (ties -> lowest index, numpy.argmax semantics).

Two all-reduces of batch x D float32 per layer and one all-gather of 8 bytes
per stream per step.  With world = 1 the same step reproduces the chained
single-GPU path (``Qwen3B200(impl="ops")``) exactly: the float32 partial is the
rounding that the fused residual epilogue applies.

``Qwen3TP._stages`` is a generator of launches that yields at every cross-rank
step; ``NcclCollective`` performs them with ``torch.distributed`` on the decode
stream, ``PeerCollective`` with the library's peer-memory exchange (plain stores
over NVLink into symmetric buffers, bounded flag waits); both are captured, with the
kernels, in the step's CUDA graph after one eager step.  Tests drive several ranks
on one GPU in lock step (``step_lockstep``) to check the split arithmetic with the
real kernels.
"""

from __future__ import annotations

import torch

from ._lib import call as abi, ptr
from .qwen3 import Qwen3B200, Qwen3Config, Qwen3Weights

EPI_STORE, EPI_RESID, EPI_F32 = 0, 1, 2


# ---------------------------------------------------------------------------
# wire slicing (plain wires: row r = [K int8 | K/G bf16 scales])
# ---------------------------------------------------------------------------
def wire_rows(wire: torch.Tensor, M: int, K: int, group: int, r0: int, r1: int) -> torch.Tensor:
    """Rows [r0, r1) of a plain wire, as a new contiguous wire."""
    rb = K + 2 * (K // group)
    return wire.view(M, rb)[r0:r1].contiguous().view(-1)


def wire_cols(wire: torch.Tensor, M: int, K: int, group: int, k0: int, k1: int) -> torch.Tensor:
    """Columns [k0, k1) (whole quantisation groups) of a plain wire, as a new wire of
    K' = k1 - k0: the int8 columns and the scales of their groups."""
    if k0 % group or k1 % group:
        raise ValueError(f"column split [{k0}, {k1}) does not fall on group-{group} boundaries")
    rb = K + 2 * (K // group)
    v = wire.view(M, rb)
    q = v[:, k0:k1]
    s = v[:, K + 2 * (k0 // group):K + 2 * (k1 // group)]
    return torch.cat([q, s], dim=1).contiguous().view(-1)


def shard_config(cfg: Qwen3Config, world: int) -> Qwen3Config:
    """The per-rank shape: Hq/n query heads, Hkv/n KV heads, FF/n, V/n vocabulary rows."""
    for name, n in (("Hq", cfg.Hq), ("Hkv", cfg.Hkv), ("FF", cfg.FF), ("V", cfg.V)):
        if n % world:
            raise ValueError(f"{name}={n} does not split over {world} ranks")
    return Qwen3Config(D=cfg.D, FF=cfg.FF // world, Hq=cfg.Hq // world, Hkv=cfg.Hkv // world, HD=cfg.HD,
                       V=cfg.V // world, n_layers=cfg.n_layers, eps=cfg.eps, theta=cfg.theta)


def shard_ranges(cfg: Qwen3Config, rank: int, world: int) -> dict:
    """Rank ``rank``'s slices of the full model: row ranges of Wqkv (its query, key and
    value heads, in that order), Wg / Wu and the lm_head; column ranges of Wo and Wd."""
    lc = shard_config(cfg, world)
    HD = cfg.HD
    qa, ka = rank * lc.Hq * HD, rank * lc.Hkv * HD
    return {"qkv_rows": [(qa, qa + lc.Hq * HD),
                         (cfg.Hq * HD + ka, cfg.Hq * HD + ka + lc.Hkv * HD),
                         ((cfg.Hq + cfg.Hkv) * HD + ka, (cfg.Hq + cfg.Hkv) * HD + ka + lc.Hkv * HD)],
            "o_cols": (rank * lc.QD, (rank + 1) * lc.QD),
            "ff_rows": (rank * lc.FF, (rank + 1) * lc.FF),
            "d_cols": (rank * lc.FF, (rank + 1) * lc.FF),
            "vocab_rows": (rank * lc.V, (rank + 1) * lc.V)}


def shard_weights(w: Qwen3Weights, rank: int, world: int) -> Qwen3Weights:
    """Rank ``rank``'s weights; ``embed`` of the result is its lm_head vocabulary rows
    (the embedding lookup keeps the full table)."""
    c, G = w.cfg, w.group
    lc = shard_config(c, world)
    sr = shard_ranges(c, rank, world)
    layers = []
    for L in w.layers:
        d = {"norm1": L["norm1"], "qn": L["qn"], "kn": L["kn"], "norm2": L["norm2"],
             "wqkv": torch.cat([wire_rows(L["wqkv"], c.QKV, c.D, G, a, b) for a, b in sr["qkv_rows"]]),
             "wo": wire_cols(L["wo"], c.D, c.QD, G, *sr["o_cols"]),
             "wg": wire_rows(L["wg"], c.FF, c.D, G, *sr["ff_rows"]),
             "wu": wire_rows(L["wu"], c.FF, c.D, G, *sr["ff_rows"]),
             "wd": wire_cols(L["wd"], c.D, c.FF, G, *sr["d_cols"])}
        layers.append(d)
    v0, v1 = sr["vocab_rows"]
    return Qwen3Weights(lc, G, layers, w.final_norm, w.embed[v0:v1].contiguous())


# ---------------------------------------------------------------------------
# collectives
# ---------------------------------------------------------------------------
class LocalCollective:
    """world = 1: the sum is the partial itself; the gather is a copy."""

    def __call__(self, op):
        if op[0] == "gather":
            op[1][0].copy_(op[2])

    def error(self):
        return None


class NcclCollective:
    """The cross-rank steps over ``torch.distributed`` (NCCL), on the current stream."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group

    def __call__(self, op):
        if op[0] == "sum":
            self.dist.all_reduce(op[1], group=self.group)
        else:
            self.dist.all_gather_into_tensor(op[1], op[2], group=self.group)

    def error(self):
        return None


class PeerCollective:
    """The cross-rank steps over peer memory (``iron_peer_exchange``): each rank pushes
    its float32 partials (or argmax pairs) into every rank's symmetric buffer with plain
    stores over NVLink and a release flag, waits (bounded) for the others' flags in its
    own buffer and sums the rows in rank order -- deterministic, no NCCL on the data
    path.  The symmetric buffer comes from ``torch.distributed._symmetric_memory``
    (peer-mapped device memory, no multicast).  Every rank must own its GPU: the
    kernel of one rank waits for the kernels of the others."""

    def __init__(self, world: int, rank: int, cap_words: int, device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        group = group or dist.group.WORLD
        where = [None] * world
        dist.all_gather_object(where, (__import__("socket").gethostname(), torch.cuda.current_device()), group=group)
        if len(set(where)) != world:
            raise RuntimeError(f"peer exchange needs one GPU per rank, got {where}")
        L = _lib.lib()
        self.world, self.rank, self.cap = world, rank, cap_words
        self.buf = symm.empty(int(L.iron_peer_buffer_bytes(world, cap_words)), dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.hdl = symm.rendezvous(self.buf, group)
        self.peers = torch.tensor(list(self.hdl.buffer_ptrs), dtype=torch.int64, device=device)
        self.epochs = torch.zeros(int(L.iron_peer_epoch_words(cap_words)), dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize()
        dist.barrier(group=group)  # every buffer is zero before any rank pushes

    def __call__(self, op):
        st = torch.cuda.current_stream().cuda_stream
        if op[0] == "sum":
            t = op[1]
            abi("iron_peer_exchange", ptr(self.peers), self.world, self.rank, self.cap, ptr(t), ptr(t), t.numel(), 0,
                ptr(self.epochs), ptr(self.err), st)
        else:
            out, src = op[1], op[2]
            abi("iron_peer_exchange", ptr(self.peers), self.world, self.rank, self.cap, ptr(src), ptr(out),
                src.numel(), 1, ptr(self.epochs), ptr(self.err), st)

    def error(self):
        """The device error word (a timed-out wait), read with the step's tokens."""
        return self.err


class Qwen3TP(Qwen3B200):
    """Rank ``rank`` of a ``world``-way tensor-parallel Qwen3 decoder (batch streams).

    ``weights`` are the full model; the rank keeps its shard.  The step, inputs and
    outputs are those of ``Qwen3B200`` (``step_tokens``, ``run_step``,
    ``set_position``); every rank is given the same tokens and returns the same
    greedy tokens."""

    def __init__(self, weights: Qwen3Weights, rank: int = 0, world: int = 1, max_seq: int = 4096,
                 batch: int = 1, use_graph: bool | None = None, device="cuda", collective=None):
        local = shard_weights(weights, rank, world)
        if use_graph is None:
            use_graph = True
        super().__init__(local, max_seq, batch=batch, keep_logits=True, use_graph=use_graph, device=device,
                         impl="ops")
        self.rank, self.world = rank, world
        self.full_cfg = weights.cfg
        self.embed_full = weights.embed
        self.v0 = rank * local.cfg.V
        dev = self.x.device
        self.part = torch.zeros(batch, local.cfg.D, dtype=torch.float32, device=dev)
        self.pairs = torch.zeros(batch, 2, dtype=torch.int32, device=dev)
        self.gathered = torch.zeros(world, batch, 2, dtype=torch.int32, device=dev)
        if collective is None or collective == "nccl":
            collective = LocalCollective() if world == 1 else NcclCollective()
        elif collective == "peer":
            collective = LocalCollective() if world == 1 else PeerCollective(world, rank, batch * local.cfg.D, dev)
        self.collective = collective
        self._eager_done: set = set()

    def run_step(self, from_tokens: bool = True, advance: bool = True):
        """As Qwen3B200.run_step; with world > 1 the first step of each kind runs eagerly
        (it sets up the NCCL communicators), later ones replay a captured graph that
        holds the collectives too."""
        key = (from_tokens, advance)
        if self.use_graph and self.world > 1 and key not in self._eager_done:
            self._eager_done.add(key)
            with torch.cuda.stream(self.stream):
                self._launch_counted(key, self.stream.cuda_stream)
            return
        super().run_step(from_tokens, advance)

    def launches_per_step(self, from_tokens: bool = True, advance: bool = True) -> int:
        """Our kernels per step, as the library counted them over the last eager or captured
        step of this kind; before any, the batch <= 8 count: embedding; per layer QKV GEMV + head
        epilogue, attention split + combine, O GEMV, residual add, gate/up GEMV, down
        GEMV, residual add; final RMSNorm; lm_head GEMV + argmax pass; argmax pair and
        merge; the position advance."""
        counted = self._step_launches.get((from_tokens, advance))
        if counted is not None:  # counted by the library over an eager or captured step
            return counted
        return int(from_tokens) + 9 * len(self.w.layers) + 1 + 2 + 2 + int(advance)

    def _stages(self, from_tokens: bool, advance: bool, st: int):
        c, w, B, G = self.cfg, self.w, self.B, self.w.group
        if from_tokens:
            abi("iron_embedding", ptr(self.embed_full), self.full_cfg.V, ptr(self.tok), B, c.D, ptr(self.x), st)
        for i, Lw in enumerate(w.layers):
            kv = self.kv[i]
            abi("iron_qkv_head", ptr(self.x), ptr(Lw["norm1"]), ptr(Lw["wqkv"]), G, 1, 0, ptr(Lw["qn"]),
                ptr(Lw["kn"]), ptr(self.angles), 1, ptr(self.q), ptr(kv), c.D, c.HD, c.Hq, c.Hkv,
                self.max_seq, B, 0, ptr(self.off), c.eps, 1, ptr(self.raw), ptr(self.tc_ws),
                self.tc_ws.numel(), st)
            abi("iron_decode_attn", ptr(self.q), ptr(kv), ptr(self.attn), B, c.Hq, c.Hkv, c.HD,
                self.max_seq, 0, 0, 1, ptr(self.len), ptr(self.attn_ws), self.attn_ws.numel(), st)
            # O, row-parallel: float32 partials -> sum over ranks -> x1 = bf16(x + bf16(sum))
            abi("iron_gemv_w8a16_ex", ptr(Lw["wo"]), None, c.D, c.QD, G, 0, ptr(self.attn), c.QD, B, None,
                0.0, 0, None, EPI_F32, ptr(self.part), c.D, ptr(self.tc_ws), self.tc_ws.numel(), st)
            yield ("sum", self.part)
            abi("iron_resid_add_f32", ptr(self.x), ptr(self.part), ptr(self.x1), B * c.D, st)
            # gate/up, column-parallel, RMSNorm(x1) in the prologue
            abi("iron_gemv_w8a16_ex", ptr(Lw["wg"]), ptr(Lw["wu"]), c.FF, c.D, G, 0, ptr(self.x1), c.D, B,
                ptr(Lw["norm2"]), c.eps, 0, None, EPI_STORE, ptr(self.gh), c.FF, ptr(self.tc_ws),
                self.tc_ws.numel(), st)
            # down, row-parallel: x = bf16(x1 + bf16(sum))
            abi("iron_gemv_w8a16_ex", ptr(Lw["wd"]), None, c.D, c.FF, G, 0, ptr(self.gh), c.FF, B, None,
                0.0, 0, None, EPI_F32, ptr(self.part), c.D, ptr(self.tc_ws), self.tc_ws.numel(), st)
            yield ("sum", self.part)
            abi("iron_resid_add_f32", ptr(self.x1), ptr(self.part), ptr(self.x), B * c.D, st)
        abi("iron_rmsnorm", ptr(self.x), ptr(w.final_norm), ptr(self.xf), B, c.D, c.eps, 1, st)
        # vocabulary-parallel greedy argmax
        abi("iron_lm_head_bf16_argmax", ptr(w.embed), c.V, c.D, ptr(self.xf), B, ptr(self.logits),
            ptr(self.tok), ptr(self.head_ws), self.head_ws.numel(), st)
        abi("iron_argmax_pair", ptr(self.logits), c.V, B, ptr(self.tok), self.v0, ptr(self.pairs), st)
        yield ("gather", self.gathered, self.pairs)
        abi("iron_argmax_merge", ptr(self.gathered), self.world, B, ptr(self.tok), st)
        if advance:
            abi("iron_decode_advance", ptr(self.pos), ptr(self.len), ptr(self.off), B, c.HD, st)

    def _launch_step(self, from_tokens: bool, advance: bool, st: int):
        for op in self._stages(from_tokens, advance, st):
            self.collective(op)

    def _read_tokens(self) -> torch.Tensor:
        """Next tokens to the host, with the tensor-core status words (16+ streams) and the
        peer exchange's error word riding along; raises on a nonzero one."""
        from . import _lib
        err = self.collective.error() if hasattr(self.collective, "error") else None
        words = [self.tok]
        if self.B >= 16:
            words += [_lib.status_word(self.tc_ws), _lib.status_word(self.head_ws)]
        if err is not None:
            words.append(err)
        with torch.cuda.stream(self.stream):
            got = torch.cat(words).cpu()
        if err is not None and int(got[-1]):
            raise RuntimeError("tensor-parallel step: a peer exchange gave up on a bounded wait")
        if self.B >= 16:
            code = int(got[self.B]) or int(got[self.B + 1])
            if code:
                self.tc_ws[:4].zero_()
                self.head_ws[:4].zero_()
                _lib.raise_on_status(code, "decode step")
        return got[:self.B]

    def close(self):
        """Release the captured step graphs (before the process group is destroyed)."""
        self._graphs.clear()


def step_lockstep(ranks: list, tokens, pos) -> torch.Tensor:
    """One step of ``len(ranks)`` Qwen3TP ranks living on one GPU, driven in lock step:
    every cross-rank step is done on the device by summing / stacking the ranks'
    buffers in rank order.  Returns rank 0's next tokens (host).  Test use."""
    for r in ranks:
        r._put_inputs(tokens, pos)
    gens = [r._stages(True, False, r.stream.cuda_stream) for r in ranks]
    while True:
        ops = [next(g, None) for g in gens]
        if all(o is None for o in ops):
            break
        if any(o is None for o in ops):
            raise RuntimeError("ranks disagree on their cross-rank steps")
        torch.cuda.synchronize()
        if ops[0][0] == "sum":
            total = ops[0][1].clone()
            for o in ops[1:]:
                total += o[1]
            for o in ops:
                o[1].copy_(total)
        else:
            stacked = torch.stack([o[2] for o in ops])
            for o in ops:
                o[1].copy_(stacked)
        torch.cuda.synchronize()
    return ranks[0]._read_tokens()
