"""IRON operators on the Qwen3 decode path, re-implemented over the B200 C ABI.

Each class keeps the constructor fields, validation errors and arg spec of the
IRON operator it replaces (file:line in the class docstring), so a runlist or
test written against IRON runs unchanged.  NPU-placement fields
(``num_aie_columns``, tile sizes, fifo depths, ...) are accepted; they affect
only the wire layouts whose geometry they define (the int8 tile wires), never
the GPU launch.  Every ``call`` launches sm_100a kernels from
``libiron_b200.so`` on the current CUDA stream; there is no CPU path.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import ClassVar

import torch

from . import _lib
from ._lib import call as abi, ptr
from .base import AIERuntimeArgSpec, Operator, ParamScratchpad


def _domain(kernel_source: str | None) -> int:
    """Payload domain of an int8 wire from IRON's kernel-source selector:
    ``mv_int8.cc`` (default) reads the biased q+128 bytes, ``*_signed.cc`` two's
    complement (gemv_int8/op.py:92-101, swiglu_mlp_dp/op_ours.py:31-44)."""
    return 0 if (kernel_source and "signed" in kernel_source) else 1


def wrow_bytes(K: int, group: int) -> int:
    """Bytes of one int8 wire row: K payload bytes + K/group bf16 scales."""
    return K + 2 * (K // group)


# ---------------------------------------------------------------------------
# GEMV
# ---------------------------------------------------------------------------

@dataclass
class GEMVInt8(Operator):
    """int8-weight GEMV with in-kernel group dequantisation (W8A16).

    Replaces iron/operators/gemv_int8/op.py:20-178.  Arg spec: the packed tile
    wire viewed as bf16 elements, the bf16 vector, the bf16 output.
    ``batch_rows`` (B200 extension) is the number of activation rows sharing one
    weight (decode batch); ``num_batches`` keeps IRON's meaning of independent
    GEMVs each with its own wire.  ``group_size`` defaults to IRON's 128."""

    M: int
    K: int
    num_aie_columns: int = 1
    tile_size_input: int = 2
    tile_size_output: int | None = None
    num_batches: int = 1
    kernel_vector_size: int = field(default=128, repr=False)
    weight_depth: int = field(default=2, repr=False)
    kernel_source: str | None = field(default=None, repr=False)
    context: object = field(default=None, repr=False)
    group_size: int = field(default=128, repr=False)
    batch_rows: int = field(default=1, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **Operator._name_aliases, "num_aie_columns": "col", "tile_size_input": "tsi",
        "tile_size_output": "tso", "num_batches": "batch"}

    def __post_init__(self):
        if self.tile_size_output is None:
            self.tile_size_output = self.tile_size_input
        if not (self.tile_size_output % self.tile_size_input == 0
                and self.tile_size_output >= self.tile_size_input):
            raise ValueError("tile_size_output must be a multiple of tile_size_input")
        if not (self.K >= self.kernel_vector_size and self.K % self.kernel_vector_size == 0):
            raise ValueError("K must be multiple of kernel_vector_size")
        if self.K % self.group_size != 0:
            raise ValueError(f"K must be a multiple of GROUP_SIZE={self.group_size}")
        if self.M % self.tile_size_input != 0:
            raise ValueError("M must be a multiple of tile_size_input")
        if self.batch_rows < 1:
            raise ValueError("batch_rows must be at least 1")
        self._tc_ws = None  # tensor-core scratch, from 16 batch rows on

    @property
    def tile_bytes(self) -> int:
        return self.tile_size_input * wrow_bytes(self.K, self.group_size)

    def wire_bytes(self) -> int:
        return (self.M // self.tile_size_input) * self.tile_bytes

    def get_arg_spec(self):
        bd = (self.num_batches,) if self.num_batches > 1 else ()
        rd = (self.batch_rows,) if self.batch_rows > 1 else ()
        return [
            AIERuntimeArgSpec("in", (self.num_batches * self.wire_bytes() // 2,)),
            AIERuntimeArgSpec("in", bd + rd + (self.K,)),
            AIERuntimeArgSpec("out", bd + rd + (self.M,)),
        ]

    def launch(self, bufs, params, stream):
        wire, x, y = bufs
        wb = self.wire_bytes()
        ws = self._workspace(x.device)
        for i in range(self.num_batches):
            abi("iron_gemv_w8a16", wire.data_ptr() + i * wb, self.M, self.K, self.group_size,
                self.tile_size_input, 0, 0, _domain(self.kernel_source),
                x.data_ptr() + i * self.batch_rows * self.K * 2, self.batch_rows, None,
                y.data_ptr() + i * self.batch_rows * self.M * 2, ptr(ws),
                0 if ws is None else ws.numel(), stream)

    def _workspace(self, device):
        """The tensor-core contraction's scratch (16+ batch rows on plain wires); the
        GEMVs of one call run in order on one stream and share it."""
        if self.batch_rows < 16 or self.tile_size_input != 1:
            return None
        if self._tc_ws is None or self._tc_ws.device != device:
            self._tc_ws = _lib.tc_workspace([(self.M, self.K)], self.batch_rows, device)
        return self._tc_ws

    def tc_status(self, clear: bool = True) -> int:
        """Status word of the tensor-core contraction (0, or the code of a bounded device
        wait that timed out); synchronous."""
        if self._tc_ws is None:
            return 0
        return int(_lib.lib().iron_tc_status(ptr(self._tc_ws), int(clear)))


@dataclass
class GEMV(Operator):
    """bf16 GEMV ``C = A @ B`` (iron/operators/gemv/op.py:20-163), float32 accumulation.

    ``num_batches > 1`` runs independent GEMVs, each with its own matrix."""

    M: int
    K: int
    num_aie_columns: int = 1
    tile_size_input: int = 2
    tile_size_output: int | None = None
    num_batches: int = 1
    kernel_vector_size: int = field(default=64, repr=False)
    epilogue: str = field(default="none", repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **Operator._name_aliases, "num_aie_columns": "col", "tile_size_input": "tsi",
        "tile_size_output": "tso", "num_batches": "batch"}

    def __post_init__(self):
        if self.tile_size_output is None:
            self.tile_size_output = self.tile_size_input
        if not (self.tile_size_output % self.tile_size_input == 0
                and self.tile_size_output >= self.tile_size_input):
            raise ValueError("tile_size_output must be a multiple of tile_size_input")
        while self.kernel_vector_size > 16 and self.K < 2 * self.kernel_vector_size:
            self.kernel_vector_size //= 2
        if self.K % self.kernel_vector_size or self.K < 2 * self.kernel_vector_size:
            raise ValueError(f"K ({self.K}) must be a multiple of kernel_vector_size "
                             f"({self.kernel_vector_size}) and at least twice as large")
        if self.epilogue != "none":
            raise ValueError(f"unsupported epilogue {self.epilogue!r} (only 'none' is on the decode path)")
        if self.K % 8:
            raise ValueError("K must be a multiple of 8 (16-byte rows)")

    def get_arg_spec(self):
        bd = (self.num_batches,) if self.num_batches > 1 else ()
        return [AIERuntimeArgSpec("in", bd + (self.M, self.K)),
                AIERuntimeArgSpec("in", bd + (self.K,)),
                AIERuntimeArgSpec("out", bd + (self.M,))]

    def launch(self, bufs, params, stream):
        A, x, y = bufs
        abi("iron_gemv_bf16", ptr(A), self.M, self.K, ptr(x), self.num_batches,
            1 if self.num_batches > 1 else 0, ptr(y), None, 0, stream)


# ---------------------------------------------------------------------------
# RMSNorm / elementwise
# ---------------------------------------------------------------------------

@dataclass
class RMSNorm(Operator):
    """(Weighted) RMSNorm over rows of ``tile_size`` (iron/operators/rms_norm/op.py:20-130).

    ``golden_rounding`` (B200 extension, default on) rounds every intermediate to bf16
    as the op's golden does on bf16 tensors (rms_norm/reference.py:8-17); off gives the
    float32 single-rounding arithmetic of aie_kernels/aie2p/rms_norm.cc."""

    size: int
    num_aie_columns: int
    num_channels: int
    tile_size: int
    weighted: bool = False
    epsilon: float = 1e-5
    context: object = field(default=None, repr=False)
    golden_rounding: bool = field(default=True, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {**Operator._name_aliases, "weighted": "w", "epsilon": "eps"}

    def __post_init__(self):
        m = self.num_aie_columns * self.num_channels * self.tile_size
        if self.size % m != 0:
            raise ValueError(f"size ({self.size}) must be a multiple of "
                             f"num_aie_columns * num_channels * tile_size ({m})")

    def get_arg_spec(self):
        specs = [AIERuntimeArgSpec("in", (self.size // self.tile_size, self.tile_size))]
        if self.weighted:
            specs.append(AIERuntimeArgSpec("in", (self.tile_size,)))
        specs.append(AIERuntimeArgSpec("out", (self.size // self.tile_size, self.tile_size)))
        return specs

    def launch(self, bufs, params, stream):
        x, w, y = (bufs[0], bufs[1], bufs[2]) if self.weighted else (bufs[0], None, bufs[1])
        abi("iron_rmsnorm", ptr(x), ptr(w), ptr(y), self.size // self.tile_size, self.tile_size,
            float(self.epsilon), 1 if self.golden_rounding else 0, stream)


@dataclass
class _BinaryElementwise(Operator):
    """Binary elementwise base (iron/common/operator_bases.py BinaryElementwiseOperator)."""

    size: int
    tile_size: int
    num_aie_columns: int = 8
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {**Operator._name_aliases, "num_aie_columns": "col"}
    _abi: ClassVar[str] = ""

    def __post_init__(self):
        if self.size % (self.num_aie_columns * self.tile_size) != 0:
            raise ValueError(f"size ({self.size}) must be a multiple of "
                             f"num_aie_columns * tile_size ({self.num_aie_columns * self.tile_size})")

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.size,)), AIERuntimeArgSpec("in", (self.size,)),
                AIERuntimeArgSpec("out", (self.size,))]

    def launch(self, bufs, params, stream):
        a, b, c = bufs
        abi(self._abi, ptr(a), ptr(b), ptr(c), self.size, stream)


@dataclass
class ElementwiseAdd(_BinaryElementwise):
    """``c = a + b`` in bf16 (iron/operators/elementwise_add/op.py:10-23)."""
    _abi: ClassVar[str] = "iron_add"


@dataclass
class ElementwiseMul(_BinaryElementwise):
    """``c = a * b`` in bf16 (iron/operators/elementwise_mul/op.py:10-23)."""
    _abi: ClassVar[str] = "iron_mul"


@dataclass
class SiLU(Operator):
    """SiLU (iron/operators/silu/op.py:10-24).  ``tanh_form`` (B200 extension) selects
    the bf16 tanh-sigmoid arithmetic of aie_kernels/aie2p/silu.cc instead of the exact
    logistic of silu/reference.py."""

    size: int
    num_aie_columns: int
    tile_size: int
    num_channels: int = field(default=1, init=False, repr=False)
    context: object = field(default=None, repr=False)
    tanh_form: bool = field(default=False, repr=False)

    def __post_init__(self):
        if self.size % (self.num_aie_columns * self.tile_size) != 0:
            raise ValueError(f"size ({self.size}) must be a multiple of "
                             f"num_aie_columns * tile_size ({self.num_aie_columns * self.tile_size})")

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.size,)), AIERuntimeArgSpec("out", (self.size,))]

    def launch(self, bufs, params, stream):
        abi("iron_silu", ptr(bufs[0]), ptr(bufs[1]), self.size, 1 if self.tanh_form else 0, stream)


# ---------------------------------------------------------------------------
# data movement and softmax of the Llama decode runlist (llama_npu.py:279-557)
# ---------------------------------------------------------------------------

@dataclass
class RoPE(Operator):
    """Rotary position embedding over (rows, cols) (iron/operators/rope/op.py:18-102;
    golden rope/reference.py:88-154): method 0 two halves, 1 interleaved; ``angles``
    holds interleaved [cos, sin] pairs, and each of its ``angle_rows`` rows serves
    ``rows / angle_rows`` consecutive rows of x.  The output may be the input buffer."""

    rows: int
    cols: int
    angle_rows: int | None = None
    num_aie_columns: int = 1
    method_type: int = 0
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **Operator._name_aliases, "num_aie_columns": "col", "angle_rows": "arows", "method_type": "m"}

    def __post_init__(self):
        if self.angle_rows is None:
            self.angle_rows = self.rows
        if not (self.cols % 32 == 0 and self.cols >= 32):
            raise ValueError("cols must be multiple of 32 and >= 32")
        if self.rows % self.num_aie_columns != 0:
            raise ValueError("rows must be divisible by num_aie_columns")
        if not (self.angle_rows <= self.rows and self.rows % self.angle_rows == 0):
            raise ValueError("angle_rows must divide rows")
        if not (self.angle_rows >= self.num_aie_columns and self.angle_rows % self.num_aie_columns == 0):
            raise ValueError("angle_rows must be divisible by num_aie_columns")
        if self.method_type not in {0, 1}:
            raise ValueError(f"method_type must be 0 or 1, got {self.method_type}")

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.rows, self.cols)),
                AIERuntimeArgSpec("in", (self.angle_rows, self.cols)),
                AIERuntimeArgSpec("out", (self.rows, self.cols))]

    def launch(self, bufs, params, stream):
        x, ang, y = bufs
        abi("iron_rope_rows", ptr(x), ptr(ang), ptr(y), self.rows, self.cols, self.angle_rows,
            self.method_type, stream)


def _i64_array(vals):
    import ctypes
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


@dataclass
class StridedCopy(Operator):
    """Strided copy between two flat buffers (iron/operators/strided_copy/op.py:18-100;
    golden strided_copy/reference.py): elements gathered by the input access pattern
    (sizes, strides, offset; up to 4 dimensions) are scattered by the output one.
    ``input_offset_parameter`` / ``output_offset_parameter`` name runtime parameters
    (element counts) added to the offsets on every call, as the reference's DMA reads
    them from the scratchpad.  Output elements the pattern does not visit keep their
    values (the KV cache of the Llama runlist).  An element that would land outside
    its buffer is skipped and sets the device word ``err`` (``status()``)."""

    input_sizes: list
    input_strides: list
    input_offset: int
    output_sizes: list
    output_strides: list
    output_offset: int
    input_buffer_size: int = field(repr=False)
    output_buffer_size: int = field(repr=False)
    dtype: object = field(default=torch.bfloat16, repr=False)
    transfer_size: int | None = None
    num_aie_channels: int = 1
    input_offset_parameter: str | None = None
    output_offset_parameter: str | None = None
    kwargs: dict = field(default_factory=dict, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **Operator._name_aliases, "input_sizes": "isz", "input_strides": "ist", "input_offset": "ioff",
        "output_sizes": "osz", "output_strides": "ost", "output_offset": "ooff", "transfer_size": "tr",
        "num_aie_channels": "ch", "input_offset_parameter": "ipar", "output_offset_parameter": "opar"}

    def __post_init__(self):
        if len(self.input_sizes) != len(self.input_strides):
            raise ValueError(f"input_sizes and input_strides must have the same length "
                             f"({len(self.input_sizes)} vs {len(self.input_strides)})")
        if len(self.output_sizes) != len(self.output_strides):
            raise ValueError(f"output_sizes and output_strides must have the same length "
                             f"({len(self.output_sizes)} vs {len(self.output_strides)})")
        if not (1 <= len(self.input_sizes) <= 4 and 1 <= len(self.output_sizes) <= 4):
            raise ValueError("access patterns have 1 to 4 dimensions")
        self._err = None

    @property
    def runtime_params(self):
        return tuple(p for p in (self.input_offset_parameter, self.output_offset_parameter) if p)

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (int(self.input_buffer_size),), dtype=self.dtype),
                AIERuntimeArgSpec("out", (int(self.output_buffer_size),), dtype=self.dtype)]

    def status(self) -> int:
        """1 if a call skipped an element outside its buffer (then cleared), else 0."""
        if self._err is None:
            return 0
        v = int(self._err.item())
        self._err.zero_()
        return v

    def launch(self, bufs, params, stream):
        src, dst = bufs
        if self._err is None or self._err.device != src.device:
            self._err = torch.zeros(1, dtype=torch.int32, device=src.device)
        ia = params.slot(self.input_offset_parameter) if self.input_offset_parameter else None
        oa = params.slot(self.output_offset_parameter) if self.output_offset_parameter else None
        abi("iron_strided_copy", ptr(src), int(self.input_buffer_size), ptr(dst), int(self.output_buffer_size),
            src.element_size(), len(self.input_sizes), _i64_array(self.input_sizes),
            _i64_array(self.input_strides), int(self.input_offset), len(self.output_sizes),
            _i64_array(self.output_sizes), _i64_array(self.output_strides), int(self.output_offset),
            int(self.num_aie_channels), ptr(ia), ptr(oa), ptr(self._err), stream)


@dataclass
class Repeat(Operator):
    """Repeat-interleave along the leading dimension (iron/operators/repeat/op.py:18-69;
    golden repeat/reference.py): (rows, cols) -> (rows * repeat, cols)."""

    rows: int
    cols: int
    repeat: int
    transfer_size: int | None = None
    dtype: object = field(default=torch.bfloat16, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {**Operator._name_aliases, "repeat": "by", "transfer_size": "ts"}

    def __post_init__(self):
        if self.rows < 1 or self.cols < 1 or self.repeat < 1:
            raise ValueError("rows, cols and repeat must be positive")

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.rows, self.cols), dtype=self.dtype),
                AIERuntimeArgSpec("out", (self.rows * self.repeat, self.cols), dtype=self.dtype)]

    def launch(self, bufs, params, stream):
        x, y = bufs
        abi("iron_repeat_rows", ptr(x), ptr(y), self.rows, self.cols * x.element_size(), self.repeat, stream)


@dataclass
class Softmax(Operator):
    """Row softmax over ``cols`` (iron/operators/softmax/op.py:18-109; golden
    softmax/reference.py), float32 inside, bf16 out.  With ``vector_size_parameter`` the
    runtime parameter of that name gives the row length that counts (the mask kernel of
    softmax/design.py:86-103): entries past it are masked and come out zero.  Without
    it, ``rtp_vector_size`` (default ``cols``) does."""

    rows: int
    cols: int
    num_aie_columns: int = 1
    num_channels: int = 1
    rtp_vector_size: int | None = None
    vector_size_parameter: str | None = None
    context: object = field(default=None, repr=False)

    @property
    def size(self):
        return self.rows * self.cols

    def __post_init__(self):
        if self.rows % 16 != 0:
            raise ValueError(f"rows ({self.rows}) must be a multiple of 16")
        if self.cols % 16 != 0:
            raise ValueError(f"cols ({self.cols}) must be a multiple of 16")
        if self.rows % self.num_aie_columns != 0:
            raise ValueError(f"rows ({self.rows}) must be a multiple of num_aie_columns ({self.num_aie_columns})")

    @property
    def runtime_params(self):
        return (self.vector_size_parameter,) if self.vector_size_parameter else ()

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.size,)), AIERuntimeArgSpec("out", (self.size,))]

    def launch(self, bufs, params, stream):
        x, y = bufs
        n = self.cols if self.rtp_vector_size is None else int(self.rtp_vector_size)
        dev = params.slot(self.vector_size_parameter) if self.vector_size_parameter else None
        abi("iron_softmax_rows", ptr(x), ptr(y), self.rows, self.cols, n, ptr(dev), stream)


@dataclass
class Transpose(Operator):
    """Transpose of (M, N) bf16 matrices (iron/operators/transpose/op.py:18-129; golden
    transpose/reference.py); ``num_batches`` > 1 transposes that many matrices laid
    back to back."""

    M: int
    N: int
    num_aie_columns: int
    num_channels: int
    m: int
    n: int
    s: int
    num_batches: int = 1
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {**Operator._name_aliases, "num_batches": "batch"}

    def __post_init__(self):
        if self.M % self.m != 0:
            raise ValueError(f"Matrix rows ({self.M}) must be a multiple of {self.m}")
        if self.N % self.n != 0:
            raise ValueError(f"Matrix columns ({self.N}) must be a multiple of {self.n}")
        if self.m % self.s != 0:
            raise ValueError(f"AIE tile rows ({self.m}) must be a multiple of {self.s}")
        if self.n % self.s != 0:
            raise ValueError(f"AIE tile columns ({self.n}) must be a multiple of {self.s}")
        if self.M * self.N % (self.m * self.n * self.num_aie_columns * self.num_channels) != 0:
            raise ValueError("Transfer size must be divisible by m*n*num_columns*num_channels")
        if self.N // self.num_aie_columns // self.n < 1:
            raise ValueError(f"num_aie_columns ({self.num_aie_columns}) exceeds N/n ({self.N // self.n})")
        if self.M // self.num_channels // self.m < 1:
            raise ValueError(f"num_channels ({self.num_channels}) exceeds M/m ({self.M // self.m})")

    def get_arg_spec(self):
        bd = (self.num_batches,) if self.num_batches > 1 else ()
        return [AIERuntimeArgSpec("in", bd + (self.M * self.N,)),
                AIERuntimeArgSpec("out", bd + (self.N * self.M,))]

    def launch(self, bufs, params, stream):
        x, y = bufs
        abi("iron_transpose", ptr(x), ptr(y), self.M, self.N, self.num_batches, stream)


# ---------------------------------------------------------------------------
# decode attention
# ---------------------------------------------------------------------------

@dataclass
class DecodeAttention(Operator):
    """Fused single-query GQA decode attention (iron/operators/decode_attn/op.py:20-181).

    Split-KV flash decoding.  ``batch_queries`` > 0 is the multi-query verify mode
    (op.py:40-56): ``num_new_tokens`` queries at positions ``S_kv_base`` .. (runtime
    parameter), causal or over the whole cache (``iron_attn_mq``).
    ``use_runtime_seq_len`` reads the valid length
    from the ``S_kv_eff`` runtime parameter (qwen3_npu_int8.py:609); otherwise
    every cached position is valid.  KV layouts: per-token ``[K_t|V_t]``
    (``kv_token_interleaved``, the default), IRON's legacy ``[K_block|V_block]``
    per ``block_kv`` tokens, or ``kv_halves`` (B200 extension) for the
    ``[K half | V half]`` buffer of decode_attn/reference.py:74-93."""

    num_heads: int
    num_kv_heads: int
    head_dim: int
    seq_len_kv: int
    num_aie_columns: int = 8
    block_kv: int = 64
    use_runtime_seq_len: bool = field(default=False, repr=False)
    batch_queries: int = 0
    num_new_tokens: int = 0
    causal: bool = True
    kv_token_interleaved: bool = True
    out_buffer_tokens: int = 0
    kv_layout: str = "combined"
    context: object = field(default=None, repr=False)
    kv_halves: bool = field(default=False, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        "num_heads": "h", "num_kv_heads": "kv", "head_dim": "d", "seq_len_kv": "skv",
        "num_aie_columns": "col", "block_kv": "bkv", "batch_queries": "m", "num_new_tokens": "new",
        "kv_layout": "kvl"}

    def __post_init__(self):
        if self.seq_len_kv % 64 != 0:
            raise ValueError("seq_len_kv must be a multiple of 64")
        if self.block_kv % 16 != 0:
            raise ValueError("block_kv must be a multiple of 16")
        if self.batch_queries > 0:
            if self.num_new_tokens % self.batch_queries != 0:
                raise ValueError(f"num_new_tokens ({self.num_new_tokens}) must be a multiple "
                                 f"of batch_queries ({self.batch_queries})")
            if not self.use_runtime_seq_len:
                raise ValueError("batch mode requires use_runtime_seq_len")
        if self.kv_layout != "combined":
            raise NotImplementedError("only the combined KV argument is implemented on B200")
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if self.head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        self._ws = None

    @property
    def runtime_params(self):
        if self.batch_queries:  # verify mode: the cached-token count before the new block
            return ("S_kv_base",)
        return ("S_kv_eff",) if self.use_runtime_seq_len else ()

    @property
    def layout_code(self) -> int:
        if self.kv_halves:
            return 1
        return 0 if self.kv_token_interleaved else 2

    def get_arg_spec(self):
        """Verify mode (op.py:156-181): Q is (num_new_tokens*H, D) token-major and O has
        max(out_buffer_tokens, num_new_tokens) tokens, of which num_new_tokens are written."""
        H, KV, D, S = self.num_heads, self.num_kv_heads, self.head_dim, self.seq_len_kv
        q_rows = self.num_new_tokens * H if self.batch_queries else H
        o_tokens = max(self.out_buffer_tokens, self.num_new_tokens) if self.batch_queries else 1
        return [AIERuntimeArgSpec("in", (q_rows, D)),
                AIERuntimeArgSpec("in", (KV, 2 * S * D)),
                AIERuntimeArgSpec("out", (o_tokens * H, D))]

    def workspace(self, device) -> torch.Tensor:
        L = _lib.lib()
        if self.batch_queries:
            n = L.iron_attn_mq_workspace_bytes(self.num_new_tokens, self.num_heads, self.num_kv_heads,
                                               self.head_dim, self.seq_len_kv)
        else:
            n = L.iron_decode_attn_workspace_bytes(1, self.num_heads, self.head_dim, self.seq_len_kv)
        if self._ws is None or self._ws.numel() < n or self._ws.device != device:
            self._ws = torch.empty(n, dtype=torch.uint8, device=device)
        return self._ws

    def launch(self, bufs, params, stream):
        q, kv, o = bufs
        ws = self.workspace(q.device)
        if self.batch_queries:
            # the query groups of the reference (batch_queries per KV pass) are one
            # kernel here: every CTA streams its positions once for 64 (token, head) rows
            abi("iron_attn_mq", ptr(q), ptr(kv), ptr(o), self.num_new_tokens, self.num_heads,
                self.num_kv_heads, self.head_dim, self.seq_len_kv, self.layout_code, self.block_kv, 0,
                ptr(params.slot("S_kv_base")), self.seq_len_kv, int(self.causal), ptr(ws), ws.numel(), stream)
            return
        dev_len = params.slot("S_kv_eff") if self.use_runtime_seq_len else None
        abi("iron_decode_attn", ptr(q), ptr(kv), ptr(o), 1, self.num_heads, self.num_kv_heads,
            self.head_dim, self.seq_len_kv, self.layout_code, self.block_kv, self.seq_len_kv,
            ptr(dev_len), ptr(ws), ws.numel(), stream)


# ---------------------------------------------------------------------------
# fused QKV head
# ---------------------------------------------------------------------------

@dataclass
class QKVHeadDataParallel(Operator):
    """Fused decode QKV head (iron/operators/qkv_head_dp/op.py:20-231).

    RMSNorm(cur, n_in) -> int8 [Q|K|V] GEMV -> per-head q/k RMSNorm -> RoPE; q to the
    q output, K_t and V_t into the per-token interleaved KV cache at the element
    offset held by the runtime parameter ``kv_offset_parameter``."""

    D: int
    HD: int
    Hq: int
    Hkv: int
    max_seq: int
    num_aie_columns: int = 8
    epsilon: float = 1e-6
    tile_size_input: int = 4
    stack_size: int = 0xD00
    kv_offset_parameter: str | None = "kv_off"
    weight_depth: int = field(default=2, repr=False)
    misc_chunked: bool = field(default=True, repr=False)
    misc_obj_elems: int | None = field(default=None, repr=False)
    runtime_tile_loop: bool = field(default=False, repr=False)
    kernel_source: str | None = field(default=None, repr=False)
    attn_colmajor: bool = field(default=False)
    with_attn: bool = field(default=False)
    attn_row3: bool = field(default=False)
    mlp_row4: bool = field(default=False)
    inplace_norm: bool = field(default=False, repr=False)
    misc_memtile: bool = field(default=False, repr=False)
    merge_drains: bool = field(default=False)
    context: object = field(default=None, repr=False)
    group_size: int = field(default=128, repr=False)
    kv_offset: int = field(default=0, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {"kv_offset_parameter": "kvpar"}

    def __post_init__(self):
        if self.with_attn or self.attn_row3 or self.mlp_row4 or self.misc_memtile:
            raise ValueError("the merged-layer NPU arms (with_attn/attn_row3/mlp_row4/misc_memtile) "
                             "have no B200 counterpart: run QKV head, DecodeAttention and the MLP as "
                             "separate operators")
        if self.D % self.group_size:
            raise ValueError(f"D must be a multiple of the group size {self.group_size}")
        if self.HD not in (64, 128):
            raise ValueError("HD must be 64 or 128")
        self._raw = None

    @property
    def runtime_params(self):
        return (self.kv_offset_parameter,) if self.kv_offset_parameter else ()

    def wire_elems(self) -> int:
        rows = (self.Hq + 2 * self.Hkv) * self.HD
        return rows * wrow_bytes(self.D, self.group_size) // 2

    def get_arg_spec(self):
        QD = self.Hq * self.HD
        misc = self.misc_obj_elems or self.HD
        return [AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (self.D,)),
                AIERuntimeArgSpec("in", (self.wire_elems(),)),
                AIERuntimeArgSpec("in", (misc,)), AIERuntimeArgSpec("in", (misc,)),
                AIERuntimeArgSpec("in", (misc,)),
                AIERuntimeArgSpec("out", (QD,)),
                AIERuntimeArgSpec("inout", (self.Hkv * self.max_seq * self.HD * 2,))]

    def launch(self, bufs, params, stream):
        cur, n_in, wire, n_qn, n_kn, ang, q, kv = bufs
        n = (self.Hq + 2 * self.Hkv) * self.HD
        if self._raw is None or self._raw.device != cur.device:
            self._raw = torch.empty(n, dtype=torch.bfloat16, device=cur.device)
        off_dev = params.slot(self.kv_offset_parameter) if self.kv_offset_parameter else None
        abi("iron_qkv_head", ptr(cur), ptr(n_in), ptr(wire), self.group_size, self.tile_size_input,
            _domain(self.kernel_source), ptr(n_qn), ptr(n_kn), ptr(ang), 0, ptr(q), ptr(kv),
            self.D, self.HD, self.Hq, self.Hkv, self.max_seq, 1, self.kv_offset, ptr(off_dev),
            float(self.epsilon), 1, ptr(self._raw), None, 0, stream)


@dataclass
class QKVHeadDataParallelOurs(QKVHeadDataParallel):
    """QKV head writing IRON's interleaved K|V cache (qkv_head_dp/op_ours.py:31-262)."""


# ---------------------------------------------------------------------------
# SwiGLU MLP block
# ---------------------------------------------------------------------------

@dataclass
class SwiGLUMLPDataParallel(Operator):
    """Decode SwiGLU MLP block with bf16 weights (iron/operators/swiglu_mlp_dp/op.py:23-227).

    ``x1 = cur + a; hf = RMSNorm_w(x1); nxt = x1 + Wd @ (silu(Wg@hf) * (Wu@hf))`` with the
    bf16 stores of swiglu_mlp_dp/test.py:79-91.  ``gh_scratch`` is a caller buffer."""

    D: int
    FF: int
    num_aie_columns: int = 8
    num_aie_rows: int = 1
    epsilon: float = 1e-5
    QD: int = None
    fuse_o: bool = False
    weight_dtype: str = field(default="bf16", repr=False)
    group_size: int = field(default=0, repr=False)
    weight_depth: int = field(default=2, repr=False)
    tile_rows_gu: int = field(default=0, repr=False)
    context: object = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        "epsilon": "eps", "num_aie_columns": "cols", "num_aie_rows": "rows", "fuse_o": "fo",
        "weight_dtype": "wdt", "group_size": "g", "weight_depth": "wd", "tile_rows_gu": "tr"}

    def __post_init__(self):
        if self.D <= 0 or self.FF <= 0:
            raise ValueError(f"D ({self.D}) and FF ({self.FF}) must be positive")
        if self.fuse_o:
            if not self.QD or self.QD <= 0:
                raise ValueError("fuse_o requires QD (the attention context width)")
            if self.num_aie_rows != 1:
                raise ValueError("fuse_o is only derived for num_aie_rows=1 (see design.py)")
            if type(self) is SwiGLUMLPDataParallel:
                raise NotImplementedError("fuse_o is implemented for the int8 arm (SwiGLUMLPDataParallelOurs)")
        self._tmp = None

    def get_arg_spec(self):
        return [AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (self.D,)),
                AIERuntimeArgSpec("in", (self.D,)),
                AIERuntimeArgSpec("in", (self.FF * self.D,)), AIERuntimeArgSpec("in", (self.FF * self.D,)),
                AIERuntimeArgSpec("in", (self.D * self.FF,)),
                AIERuntimeArgSpec("inout", (self.FF,)),
                AIERuntimeArgSpec("out", (self.D,))]

    def launch(self, bufs, params, stream):
        cur, a, n_pf, wg, wu, wd, gh, nxt = bufs
        D, FF = self.D, self.FF
        if self._tmp is None or self._tmp.device != cur.device:
            self._tmp = torch.empty(3 * D + 2 * FF, dtype=torch.bfloat16, device=cur.device)
        x1, hf, d = self._tmp[:D], self._tmp[D:2 * D], self._tmp[2 * D:3 * D]
        g, u = self._tmp[3 * D:3 * D + FF], self._tmp[3 * D + FF:]
        abi("iron_add", ptr(cur), ptr(a), ptr(x1), D, stream)
        abi("iron_rmsnorm", ptr(x1), ptr(n_pf), ptr(hf), 1, D, float(self.epsilon), 0, stream)
        abi("iron_gemv_bf16", ptr(wg), FF, D, ptr(hf), 1, 0, ptr(g), None, 0, stream)
        abi("iron_gemv_bf16", ptr(wu), FF, D, ptr(hf), 1, 0, ptr(u), None, 0, stream)
        abi("iron_silu", ptr(g), ptr(g), FF, 1, stream)
        abi("iron_mul", ptr(g), ptr(u), ptr(gh), FF, stream)
        abi("iron_gemv_bf16", ptr(wd), D, FF, ptr(gh), 1, 0, ptr(d), None, 0, stream)
        abi("iron_add", ptr(x1), ptr(d), ptr(nxt), D, stream)


@dataclass
class SwiGLUMLPDataParallelOurs(SwiGLUMLPDataParallel):
    """Fused SwiGLU MLP block over int8 tile wires (iron/operators/swiglu_mlp_dp/op_ours.py:47-582).

    Wires: Wg/Wu with ``tile_rows_gu``-row tiles, Wd with ``tile_rows_gu/(FF/D)``-row tiles,
    and under ``fuse_o`` the per-core tile-major Wo wire with its pad rows
    (op_ours.py:357-421, qwen3_npu_int8.py:407-436).  ``group_size`` defaults to IRON's 128."""

    tile_rows_gu: int = field(default=12, repr=False)
    weight_depth: int = field(default=1, repr=False)
    weight_memtile: bool = field(default=False)
    weight_stage_depth: int = field(default=16)
    kernel_source: str | None = field(default=None, repr=False)
    acc_kernel_source: str | None = field(default=None, repr=False)

    _name_aliases: ClassVar[dict[str, str]] = {
        **SwiGLUMLPDataParallel._name_aliases, "weight_memtile": "wmm", "weight_stage_depth": "wsd"}

    def __post_init__(self):
        super().__post_init__()
        if self.group_size == 0:
            self.group_size = 128
        if self.FF % self.D != 0:
            raise NotImplementedError("the chunked (FF % D != 0) 4B wire is not on the Qwen3-0.6B path")
        self.ff_pad = self.FF
        R = self.FF // self.D
        if self.tile_rows_gu % R:
            raise ValueError(f"tile_rows_gu={self.tile_rows_gu} must be a multiple of FF/D={R}")

    @property
    def n_cores(self) -> int:
        return self.num_aie_columns * self.num_aie_rows

    def _wrow(self, K: int) -> int:
        """Wire row in bf16 element units (op_ours.py `_wrow`)."""
        return wrow_bytes(K, self.group_size) // 2

    def _wo_tiling(self):
        """(n, N_O_TILES, TSI_O, WTILE bytes), swiglu_mlp_dp/op_ours.py:357-369."""
        n = self.n_cores
        wtile = self.tile_rows_gu * self._wrow(self.D) * 2
        wrow_qd = self._wrow(self.QD) * 2
        if wtile % wrow_qd:
            raise ValueError(f"fuse_o needs the shared weight tile ({wtile} B) to be a whole "
                             f"number of Wo rows ({wrow_qd} B each)")
        tsi_o = wtile // wrow_qd
        return n, -(-(self.D // n) // tsi_o), tsi_o, wtile

    def get_arg_spec(self):
        wg = self.ff_pad * self._wrow(self.D)
        wd = self.D * self._wrow(self.FF)
        if self.fuse_o:
            n, n_o, _, wtile = self._wo_tiling()
            wo = n * n_o * wtile // 2
            return [AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (self.QD,)),
                    AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (wo,)),
                    AIERuntimeArgSpec("in", (wg,)), AIERuntimeArgSpec("in", (wg,)),
                    AIERuntimeArgSpec("in", (wd,)),
                    AIERuntimeArgSpec("inout", (self.ff_pad,)), AIERuntimeArgSpec("inout", (self.D,)),
                    AIERuntimeArgSpec("out", (self.D,))]
        return [AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (self.D,)),
                AIERuntimeArgSpec("in", (self.D,)), AIERuntimeArgSpec("in", (wg,)),
                AIERuntimeArgSpec("in", (wg,)), AIERuntimeArgSpec("in", (wd,)),
                AIERuntimeArgSpec("inout", (self.ff_pad,)), AIERuntimeArgSpec("out", (self.D,))]

    def launch(self, bufs, params, stream):
        dom = _domain(self.kernel_source)
        R = self.FF // self.D
        tsi_gu, tsi_d = self.tile_rows_gu, self.tile_rows_gu // R
        if self.fuse_o:
            cur, cx, n_pf, wo, wg, wu, wd, gh, a_s, nxt = bufs
            n, n_o, tsi_o, _ = self._wo_tiling()
            abi("iron_mlp_block", ptr(cur), ptr(cx), 1, ptr(n_pf), ptr(wo), tsi_o, self.D // n, n_o,
                ptr(wg), ptr(wu), tsi_gu, ptr(wd), tsi_d, self.group_size, dom, ptr(a_s), ptr(gh),
                ptr(nxt), self.D, self.FF, self.QD, 1, float(self.epsilon), None, 0, stream)
        else:
            cur, a, n_pf, wg, wu, wd, gh, nxt = bufs
            if self._tmp is None or self._tmp.device != cur.device:
                self._tmp = torch.empty(self.D, dtype=torch.bfloat16, device=cur.device)
            abi("iron_mlp_block", ptr(cur), ptr(a), 0, ptr(n_pf), None, 1, 0, 0,
                ptr(wg), ptr(wu), tsi_gu, ptr(wd), tsi_d, self.group_size, dom, ptr(self._tmp), ptr(gh),
                ptr(nxt), self.D, self.FF, 0, 1, float(self.epsilon), None, 0, stream)


__all__ = [
    "GEMVInt8", "GEMV", "RMSNorm", "ElementwiseAdd", "ElementwiseMul", "SiLU", "DecodeAttention",
    "QKVHeadDataParallel", "QKVHeadDataParallelOurs", "SwiGLUMLPDataParallel",
    "SwiGLUMLPDataParallelOurs", "ParamScratchpad", "AIERuntimeArgSpec",
]
