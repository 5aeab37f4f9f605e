"""ctypes binding of ``libiron_b200.so`` (the C ABI declared in ``include/iron_b200.h``).

There is no fallback: if the library is missing or a call fails, an exception
is raised.  ``lib()`` loads the in-tree library once per process.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libiron_b200.so"

P = C.c_void_p
I = C.c_int
I64 = C.c_int64
F = C.c_float

# name -> (restype, argtypes); mirrors include/iron_b200.h
SIGNATURES: dict[str, tuple] = {
    "iron_version": (C.c_char_p, []),
    "iron_last_error": (I, [C.c_char_p, I]),
    "iron_gemv_w8a16": (I, [P, I, I, I, I, I, I, I, P, I, P, P, P, I64, P]),
    "iron_dequant_w8": (I, [P, I, I, I, I, I, I, I, P, P]),
    "iron_quantize_rtn": (I, [P, I, I, I, I, I, P, P]),
    "iron_gemv_bf16": (I, [P, I, I, P, I, I, P, P, I64, P]),
    "iron_lm_head_bf16_argmax": (I, [P, I, I, P, I, P, P, P, I64, P]),
    "iron_lm_head_w8_argmax": (I, [P, I, I, I, P, I, P, P, P, I64, P]),
    "iron_lm_head_workspace_bytes": (I64, [I, I, I]),
    "iron_argmax_workspace_bytes": (I64, [I]),
    "iron_argmax_bf16": (I, [P, I, I, P, P, P]),
    "iron_rmsnorm": (I, [P, P, P, I, I, F, I, P]),
    "iron_add": (I, [P, P, P, I64, P]),
    "iron_tc_status": (I, [P, I]),
    "iron_tc_workspace_bytes": (I64, [I, I, I]),
    "iron_launch_count": (I64, []),
    "iron_rope_kv": (I, [P, P, P, P, I, I, I, I, I, P, P]),
    "iron_qkv_rows": (I, [P, I, P, P, P, P, P, I, I, I, I, I, F, I, P]),
    "iron_gemv_w8a16_ex": (I, [P, P, I, I, I, I, P, I, I, P, C.c_float, I, P, I, P, I, P, I64, P]),
    "iron_resid_add_f32": (I, [P, P, P, I64, P]),
    "iron_argmax_pair": (I, [P, I, I, P, I, P, P]),
    "iron_argmax_merge": (I, [P, I, I, P, P]),
    "iron_peer_buffer_bytes": (I64, [I, I]),
    "iron_peer_epoch_words": (I, [I]),
    "iron_peer_exchange": (I, [P, I, I, I, P, P, I, I, P, P, P]),
    "iron_mul": (I, [P, P, P, I64, P]),
    "iron_silu": (I, [P, P, I64, I, P]),
    "iron_embedding": (I, [P, I, P, I, I, P, P]),
    "iron_decode_advance": (I, [P, P, P, I, I, P]),
    "iron_rope_rows": (I, [P, P, P, I, I, I, I, P]),
    "iron_strided_copy": (I, [P, I64, P, I64, I, I, P, P, I64, I, P, P, I64, I, P, P, P, P]),
    "iron_repeat_rows": (I, [P, P, I64, I64, I, P]),
    "iron_softmax_rows": (I, [P, P, I, I, I, P, P]),
    "iron_transpose": (I, [P, P, I, I, I, P]),
    "iron_qkv_head": (I, [P, P, P, I, I, I, P, P, P, I, P, P, I, I, I, I, I, I, I, P, F, I, P, P, I64, P]),
    "iron_decode_attn_workspace_bytes": (I64, [I, I, I, I]),
    "iron_decode_attn": (I, [P, P, P, I, I, I, I, I, I, I, I, P, P, I64, P]),
    "iron_decode_attn_static_capacity_bytes": (I64, []),
    "iron_decode_attn_static": (I, [P, P, P, I, I, I, I, I, I, I, I, P, P]),
    "iron_attn_mq_workspace_bytes": (I64, [I, I, I, I, I]),
    "iron_attn_mq": (I, [P, P, P, I, I, I, I, I, I, I, I, P, I, I, P, I64, P]),
    "iron_qwen3_sync_words": (I, [P]),
    "iron_qwen3_attn_ws_bytes": (I64, [P]),
    "iron_qwen3_cand_bytes": (I64, []),
    "iron_qwen3_grid": (I, [P]),
    "iron_qwen3_decode_step": (I, [P, I, I, P]),
    "iron_qwen3_step_host": (I, [P, P, P, I, P]),
    "iron_qwen3_sync_reset": (I, [P, P]),
    "iron_qwen3_tiles_bytes": (I64, [I, I, I]),
    "iron_qwen3_pack_tiles": (I, [P, I64, I, I, I, I, I, P, P]),
    "iron_mlp_block": (I, [P, P, I, P, P, I, I, I, P, P, I, P, I, I, I, P, P, P, I, I, I, I, F, P, I64, P]),
}

_LIB = None


class IronError(RuntimeError):
    """A non-zero status from the iron_b200 C ABI."""


def lib():
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m iron_b200.build` (needs nvcc)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def launch_count() -> int:
    """Kernels the library has launched in this process (``iron_launch_count``)."""
    return int(lib().iron_launch_count())


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().iron_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name: str, *args) -> int:
    """Call an ABI function; raise IronError on a negative status."""
    rc = getattr(lib(), name)(*args)
    if rc < 0:
        raise IronError(f"{name} failed ({rc}): {last_error()}")
    return rc


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("iron_b200 kernels take CUDA tensors (got a CPU tensor)")
    return t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def workspace(nbytes: int, device):
    """Zero-filled device scratch of ``nbytes`` (at least 256) bytes.  torch's caching
    allocator hands out 512-byte aligned blocks, above the 256 bytes the entry points
    ask for."""
    import torch
    return torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def tc_workspace(shapes, batch: int, device, lm_head: bool = False):
    """Scratch for the batch 16..256 tensor-core projections of ``shapes`` ((M, K) pairs)
    that run one after another on one stream (``iron_tc_workspace_bytes``, the largest),
    or of a batched lm_head + argmax (``iron_lm_head_workspace_bytes``)."""
    L = lib()
    fn = L.iron_lm_head_workspace_bytes if lm_head else L.iron_tc_workspace_bytes
    return workspace(max(fn(M, K, batch) for M, K in shapes), device)


def status_word(ws):
    """The int32 status word at the head of a tensor-core workspace, as a device view
    (read it with the step's results; ``iron_tc_status`` is the synchronous form)."""
    import torch
    return ws[:4].view(torch.int32)


def raise_on_status(code: int, what: str):
    if code:
        raise IronError(f"{what}: a tensor-core projection stopped on a bounded device wait "
                        f"(code {code}); its outputs are not valid")


class StepIO:
    """Host side of one decode step of B streams on ``stream``.

    ``put`` writes the step's token ids, positions, valid lengths (position + 1) and
    K/V element offsets (position * 2 * HD) into a pinned (4, B) int32 buffer and copies
    it to the device params in one copy; ``get`` copies the B next tokens and the given
    status words into a pinned buffer, waits for the stream and returns that buffer as
    a numpy array (tokens, then the status words)."""

    def __init__(self, params, tok, status_words, HD: int, stream):
        import torch
        self.B, self.HD, self.stream = int(params.shape[1]), int(HD), stream
        self.params, self.tok, self.status = params, tok, list(status_words)
        self.hin = torch.zeros(4, self.B, dtype=torch.int32, pin_memory=True)
        self.hout = torch.zeros(self.B + len(self.status), dtype=torch.int32, pin_memory=True)
        self.nin, self.nout = self.hin.numpy(), self.hout.numpy()

    @staticmethod
    def _host(v):
        import torch
        return v.detach().cpu().numpy() if torch.is_tensor(v) else v

    def put(self, tokens, pos):
        import numpy as np
        import torch
        n = self.nin
        n[0] = self._host(tokens)
        n[1] = self._host(pos)
        np.add(n[1], 1, out=n[2])
        np.multiply(n[1], 2 * self.HD, out=n[3])
        with torch.cuda.stream(self.stream):
            self.params.copy_(self.hin, non_blocking=True)

    def get(self):
        import torch
        B = self.B
        with torch.cuda.stream(self.stream):
            self.hout[:B].copy_(self.tok, non_blocking=True)
            for i, s in enumerate(self.status):
                self.hout[B + i:B + i + 1].copy_(s, non_blocking=True)
        self.stream.synchronize()
        return self.nout
