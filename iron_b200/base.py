"""Operator plumbing that mirrors IRON's operator API on the B200.

IRON's operators (iron/common/base.py:31-215) are dataclasses with
``get_arg_spec() -> [AIERuntimeArgSpec]``, ``compile()`` and ``get_callable()``
returning ``call(*buffers)`` with buffers in arg-spec order.  The same surface
is kept here; ``compile()`` only checks that the CUDA library is loaded (the
kernels are prebuilt for sm_100a), and buffers are CUDA torch tensors.
Runtime scalars that IRON keeps in a parameter scratchpad
(``params.write(name, value)``, iron/common/sequence.py:684-711) live in a
device int32 buffer so that a captured CUDA graph reads the current value.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field
from typing import Any, Callable, ClassVar

import torch

from . import _lib


@dataclass(frozen=True)
class AIERuntimeArgSpec:
    """One runtime argument: direction in {in, out, inout}, shape, element dtype.

    Mirrors iron/common/base.py:203-215.  Buffers are bf16-typed even when they
    carry int8 wire bytes (gemv_int8/op.py:158-169), exactly as in IRON."""

    direction: str
    shape: tuple[int, ...]
    dtype: Any = torch.bfloat16

    def __post_init__(self) -> None:
        if self.direction not in {"in", "out", "inout"}:
            raise ValueError(f"Invalid direction {self.direction!r}: must be one of 'in', 'out', 'inout'")

    @property
    def nbytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n * torch.empty((), dtype=self.dtype).element_size()


class ParamScratchpad:
    """Named int32 runtime parameters resident on the device.

    ``write(name, value)`` stages a value on the host; ``sync()`` copies every
    staged value to the device buffer on the current stream.  Kernels read the
    device slots, so graph replays see fresh values without re-capture."""

    def __init__(self, names, device="cuda"):
        self.names = list(dict.fromkeys(names))
        self.index = {n: i for i, n in enumerate(self.names)}
        n = max(1, len(self.names))
        self.host = torch.zeros(n, dtype=torch.int32, pin_memory=torch.cuda.is_available())
        self.dev = torch.zeros(n, dtype=torch.int32, device=device)

    def write(self, name, value) -> None:
        if name not in self.index:
            raise KeyError(f"unknown runtime parameter {name!r} (known: {self.names})")
        self.host[self.index[name]] = int(value)

    def sync(self, stream=None) -> None:
        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self.dev.copy_(self.host, non_blocking=True)

    def slot(self, name) -> torch.Tensor:
        i = self.index[name]
        return self.dev[i:i + 1]

    def value(self, name) -> int:
        return int(self.host[self.index[name]])


def _serialize(v) -> str:
    if isinstance(v, bool):
        return str(int(v))
    if isinstance(v, float):
        return f"{v:g}".replace(".", "p").replace("-", "m")
    if isinstance(v, (list, tuple)):
        return "x".join(str(x) for x in v)
    return str(v)


class Operator:
    """Base class of the B200 operators (IRON's AIEOperatorBase / MLIROperator surface)."""

    _name_aliases: ClassVar[dict[str, str]] = {
        "num_aie_columns": "c",
        "num_channels": "ch",
        "tile_size": "t",
        "size": "sz",
    }
    #: names of runtime parameters the operator reads (sequence params scratchpad)
    runtime_params: ClassVar[tuple[str, ...]] = ()

    @property
    def name(self) -> str:
        """Unique name from the dataclass fields (iron/common/base.py:127-148)."""
        aliases = type(self)._name_aliases
        parts = (f"{aliases.get(f.name, f.name)}{_serialize(getattr(self, f.name))}"
                 for f in dataclasses.fields(self)
                 if f.repr and getattr(self, f.name) is not None)
        return type(self).__name__ + "_" + "_".join(parts) + "_b200"

    def get_arg_spec(self) -> list[AIERuntimeArgSpec]:
        raise NotImplementedError

    def compile(self, dry_run: bool = False) -> "Operator":
        """Kernels are prebuilt; load the library so a missing build fails here."""
        if not dry_run:
            _lib.lib()
        return self

    def get_params_used(self) -> tuple[str, ...]:
        return tuple(p for p in self.runtime_params if p)

    def get_callable(self, params: ParamScratchpad | None = None) -> Callable[..., Any]:
        """Return ``call(*buffers)``; buffers are CUDA tensors in arg-spec order."""
        self.compile()
        own = params if params is not None else (
            ParamScratchpad(self.get_params_used()) if self.get_params_used() else None)
        op = self

        def call(*buffers, stream=None):
            specs = op.get_arg_spec()
            if len(buffers) != len(specs):
                raise ValueError(f"{op.name}: expected {len(specs)} buffers, got {len(buffers)}")
            for b, s in zip(buffers, specs):
                if b.numel() * b.element_size() < s.nbytes:
                    raise ValueError(f"{op.name}: buffer of {b.numel() * b.element_size()} bytes "
                                     f"is smaller than its arg spec {s}")
            op.launch(list(buffers), own, _lib.stream_ptr(stream))

        call.params = own
        call.op = self
        return call

    def launch(self, buffers: list[torch.Tensor], params: ParamScratchpad | None, stream: int) -> None:
        raise NotImplementedError


def field_norepr(default):
    return field(default=default, repr=False)
