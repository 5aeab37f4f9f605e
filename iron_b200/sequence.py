"""OperatorSequence on the B200: a runlist of operators replayed as one CUDA graph.

Mirrors IRON's ``OperatorSequence`` (iron/common/sequence.py:270-566) and its
runtime callable (:578-862): named buffers laid out from the operators' arg
specs (with ``name[start:end]`` byte slices and explicit ``buffer_sizes``),
``get_buffer(name).torch_view()``, a ``params`` scratchpad written by name and
``sync()``-ed before a call, and ``__call__()`` that runs the whole runlist and
waits for it.  On the first call the runlist is run once eagerly (workspaces
are allocated then) and captured into a CUDA graph (recorded, not run again); later
calls replay the graph, reading runtime parameters from device memory.  All buffers live in
one device arena with 256-byte aligned members.
"""

from __future__ import annotations

import time

import torch

from .base import AIERuntimeArgSpec, Operator, ParamScratchpad

ALIGN = 256


class DeviceBuffer:
    """A named byte range of the sequence arena (IRON's XRTSubBuffer role)."""

    def __init__(self, raw: torch.Tensor, name: str):
        self.raw = raw  # uint8 CUDA tensor
        self.name = name

    def torch_view(self, dtype=torch.bfloat16) -> torch.Tensor:
        """Flat device view; writes go straight to device memory."""
        n = self.raw.numel() // torch.empty((), dtype=dtype).element_size()
        return self.raw[:n * torch.empty((), dtype=dtype).element_size()].view(dtype)

    def to_torch(self, dtype=torch.bfloat16) -> torch.Tensor:
        """Host copy of the buffer contents."""
        return self.torch_view(dtype).cpu()

    def to(self, device) -> "DeviceBuffer":
        """IRON's host/device sync of a buffer (``to("npu")`` / ``to("cpu")``,
        iron/common/sequence.py XRT buffers).  The buffer is device memory and
        ``torch_view`` reads and writes it directly, so there is nothing to move; device
        work of earlier calls has finished when a call returns."""
        if device not in ("npu", "cpu", "cuda"):
            raise ValueError(f"unknown device {device!r}")
        return self

    def fill_(self, value, dtype=torch.bfloat16) -> "DeviceBuffer":
        """Fill every element (read as ``dtype``) with ``value`` (the XRT tensor's
        ``fill_``, which also syncs it to the device)."""
        self.torch_view(dtype).fill_(value)
        return self

    @property
    def nbytes(self) -> int:
        return self.raw.numel()


class OperatorSequence(Operator):
    """Concatenate a runlist of operators into one dispatch (a CUDA graph)."""

    def __init__(self, name, runlist, input_args, output_args, buffer_sizes=None, dispatch="auto",
                 extra_flags=None, share_designs=False, independent_buffer_args=None,
                 independent_buffer_groups=None, context=None, use_cuda_graph=True, *args, **kwargs):
        if not all(isinstance(op, Operator) and all(isinstance(b, str) for b in bufs)
                   for op, *bufs in runlist):
            raise TypeError("runlist entries must be (Operator, *str) tuples; each operator must be "
                            "an Operator and each buffer name must be a str")
        if dispatch not in ("auto", "fused", "separate"):
            raise ValueError(f"dispatch {dispatch!r}: the B200 sequence runs 'auto'/'fused' (one CUDA "
                             f"graph) or 'separate' (eager launches); CPU goldens live outside the product")
        self._name = name + "_shared" if share_designs else name
        self.runlist = runlist
        self.input_args = list(input_args)
        self.output_args = list(output_args)
        self.explicit_buffer_sizes = dict(buffer_sizes or {})
        self.independent_buffer_args = list(independent_buffer_args or [])
        self.independent_buffer_groups = dict(independent_buffer_groups or {})
        self.extra_flags = list(extra_flags or [])
        self.context = context
        self.use_cuda_graph = use_cuda_graph and dispatch != "separate"
        self.subbuffer_layout = None

    @property
    def name(self) -> str:
        return self._name

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (n,)) for n in self.input_args]

    def calculate_buffer_layout(self):
        """Byte layout of every named buffer (iron/common/sequence.py:384-516)."""
        sizes: dict[str, int] = {}
        slices: dict[str, tuple[str, int, int]] = {}
        for op, *bufs in self.runlist:
            specs = op.get_arg_spec()
            if len(specs) != len(bufs):
                raise ValueError(f"Number of buffers ({len(bufs)}) must match operator argument "
                                 f"specification ({len(specs)}) for operator {op!r}")
            for b, spec in zip(bufs, specs):
                if "[" in b and b.endswith("]"):
                    base = b[:b.index("[")]
                    start, end = map(int, b[b.index("[") + 1:-1].split(":"))
                    if base not in sizes and base not in self.explicit_buffer_sizes:
                        raise ValueError(f"Sliced buffer '{b}' requires explicit size for base buffer "
                                         f"'{base}' in buffer_sizes parameter")
                    if end - start < spec.nbytes:
                        raise ValueError(f"slice '{b}' ({end - start} B) is smaller than its arg spec {spec}")
                    slices[b] = (base, start, end)
                elif b not in sizes:
                    sizes[b] = spec.nbytes
                elif sizes[b] != spec.nbytes:
                    raise ValueError(f"Buffer '{b}' has conflicting sizes between operators: "
                                     f"{sizes[b]} vs {spec.nbytes} bytes")
        known = set(sizes) | set(slices) | set(self.explicit_buffer_sizes)
        for a in self.input_args + self.output_args:
            if a not in known:
                raise ValueError(f"argument {a} not found in runlist buffers")
        for k, v in self.explicit_buffer_sizes.items():
            sizes[k] = max(int(v), sizes.get(k, 0))
        layout, off = {}, 0
        for name, n in sizes.items():
            layout[name] = (off, n)
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        for name, (base, s, e) in slices.items():
            boff, blen = layout[base]
            if e > blen:
                raise ValueError(f"slice '{name}' ends past its base buffer ({blen} B)")
            layout[name] = (boff + s, e - s)
        return layout, off

    def compile(self, dry_run: bool = False):
        for op, *_ in self.runlist:
            op.compile(dry_run)
        self.subbuffer_layout, self.arena_bytes = self.calculate_buffer_layout()
        return self

    def get_layout_for_buffer(self, name):
        return self.subbuffer_layout[name]

    def get_callable(self, device="cuda"):
        if self.subbuffer_layout is None:
            self.compile()
        return SequenceCallable(self, device)


class SequenceCallable:
    """Runtime of a compiled OperatorSequence (IRON's SequenceFullELFCallable surface)."""

    def __init__(self, seq: OperatorSequence, device="cuda"):
        self.op = seq
        self.device = torch.device(device)
        self.arena = torch.zeros(max(seq.arena_bytes, ALIGN), dtype=torch.uint8, device=self.device)
        names = []
        for op, *_ in seq.runlist:
            names += list(op.get_params_used())
        self.params = ParamScratchpad(names, device=self.device)
        self._buffers: dict[str, DeviceBuffer] = {}
        self._graph = None
        self.stream = torch.cuda.Stream(device=self.device)
        self.last_elapsed = 0.0
        self._plan = [(op, [self.get_buffer(b) for b in bufs]) for op, *bufs in seq.runlist]

    def get_buffer(self, name: str) -> DeviceBuffer:
        if name not in self._buffers:
            if name not in self.op.subbuffer_layout:
                raise ValueError(f"Unknown buffer '{name}'")
            off, n = self.op.subbuffer_layout[name]
            self._buffers[name] = DeviceBuffer(self.arena[off:off + n], name)
        return self._buffers[name]

    def sync_independent_buffers(self):
        """Buffers are device-resident; nothing to push."""

    @property
    def input_buffer(self) -> DeviceBuffer:
        """IRON's input / scratch / output XRT buffers are one device arena here: each
        name is the whole arena, whose ``to()`` has nothing to move."""
        return DeviceBuffer(self.arena, "arena")

    scratch_buffer = input_buffer
    output_buffer = input_buffer

    def _run_eager(self):
        for op, bufs in self._plan:
            views = []
            for b, spec in zip(bufs, op.get_arg_spec()):
                t = b.torch_view(spec.dtype)
                n = 1
                for s in spec.shape:
                    n *= int(s)
                views.append(t[:n].view(spec.shape) if spec.shape else t[:1])
            op.launch(views, self.params, self.stream.cuda_stream)

    def __call__(self):
        t0 = time.perf_counter()
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            if not self.op.use_cuda_graph:
                self._run_eager()
            elif self._graph is None:
                # this call's work, run eagerly (operator workspaces are allocated here,
                # outside the capture); the capture then records the same launches without
                # running them, so a runlist that updates buffers in place (the residual
                # adds of a decoder) runs exactly once per call
                self._run_eager()
                self.stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream):
                    self._run_eager()
                self._graph = g
            else:
                self._graph.replay()
        self.stream.synchronize()
        self.last_elapsed = time.perf_counter() - t0


class SwiGLUDecode(OperatorSequence):
    """SwiGLU decode FFN as a sequence of GEMV, GEMV, SiLU, Mul, GEMV
    (iron/operators/swiglu_decode/op.py:13-70).  Buffers: ``in``, ``w_gate``,
    ``w_up``, ``w_down``, ``out``."""

    def __init__(self, embedding_dim, hidden_dim, prio_accuracy=False, context=None):
        from .operators import GEMV, ElementwiseMul, SiLU
        self.hidden_dim = hidden_dim
        self.embedding_dim = embedding_dim
        self.prio_accuracy = prio_accuracy
        n_cols = 8
        gemv_1 = GEMV(M=hidden_dim, K=embedding_dim, num_aie_columns=n_cols, tile_size_input=4,
                      tile_size_output=hidden_dim // n_cols)
        silu = SiLU(size=hidden_dim, num_aie_columns=n_cols, tile_size=hidden_dim // (n_cols * 2))
        mul = ElementwiseMul(size=hidden_dim, num_aie_columns=n_cols, tile_size=hidden_dim // n_cols)
        gemv_2 = GEMV(M=embedding_dim, K=hidden_dim, num_aie_columns=n_cols, tile_size_input=1,
                      tile_size_output=embedding_dim // n_cols)
        runlist = [
            (gemv_1, "w_gate", "in", "left"),
            (gemv_1, "w_up", "in", "right"),
            (silu, "left", "left_swished"),
            (mul, "left_swished", "right", "intermediate"),
            (gemv_2, "w_down", "intermediate", "out"),
        ]
        super().__init__(name=f"swiglu_decode_e{embedding_dim}_h{hidden_dim}", runlist=runlist,
                         input_args=["in"], output_args=["out"], context=context)
