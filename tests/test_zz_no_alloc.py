"""The allocation-free decode attention entry point (iron_decode_attn_static).

It exists for callers that cannot allocate device memory themselves -- a host
plugin with no allocator of its own, or a runtime that forbids allocation while
it decodes -- and keeps its split-KV partials in a fixed array inside the
library instead of a caller workspace.  These tests call it through the C ABI
and check it against the workspace entry point (iron_decode_attn) on the same
inputs, twice in a row so that the second call runs over whatever the first
left in the shared array.  This file is collected last on purpose.
"""

import numpy as np
import pytest
import torch

from iron_b200 import _lib
from oracle import ops
from oracle.bf16 import rnd

from helpers import assert_close, dev_bf16, host

pytestmark = pytest.mark.gpu


def _case(seed, batch, H, KV, HD, S):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, H, HD, generator=g, device="cuda").to(torch.bfloat16)
    kv = torch.randn(batch, KV, 2 * S * HD, generator=g, device="cuda").to(torch.bfloat16)
    return q, kv


def _with_workspace(q, kv, batch, H, KV, HD, S, L, lens):
    out = torch.empty(batch, H, HD, dtype=torch.bfloat16, device="cuda")
    n = _lib.lib().iron_decode_attn_workspace_bytes(batch, H, HD, S)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    _lib.call("iron_decode_attn", q.data_ptr(), kv.data_ptr(), out.data_ptr(), batch, H, KV, HD, S, 0, 0, L,
              None if lens is None else lens.data_ptr(), ws.data_ptr(), n, _lib.stream_ptr())
    return out


def _static(q, kv, batch, H, KV, HD, S, L, lens):
    out = torch.empty(batch, H, HD, dtype=torch.bfloat16, device="cuda")
    _lib.call("iron_decode_attn_static", q.data_ptr(), kv.data_ptr(), out.data_ptr(), batch, H, KV, HD, S, 0, 0,
              L, None if lens is None else lens.data_ptr(), _lib.stream_ptr())
    return out


def test_static_scratch_matches_workspace_entry_point_twice():
    """Two consecutive calls of different shapes and lengths, each against the
    workspace entry point on the same inputs."""
    cases = [
        dict(seed=1, batch=1, H=16, KV=8, HD=128, S=1152, L=1089, ragged=False),
        dict(seed=2, batch=4, H=32, KV=8, HD=128, S=512, L=0, ragged=True),
    ]
    for c in cases:
        q, kv = _case(c["seed"], c["batch"], c["H"], c["KV"], c["HD"], c["S"])
        lens = None
        if c["ragged"]:
            lens = torch.tensor([1, 77, 300, 512][:c["batch"]], dtype=torch.int32, device="cuda")
        args = (q, kv, c["batch"], c["H"], c["KV"], c["HD"], c["S"], c["L"], lens)
        got = _static(*args)
        want = _with_workspace(*args)
        torch.cuda.synchronize()
        assert not np.isnan(host(got)).any()
        assert_close(host(got), host(want), what=f"static scratch vs workspace ({c})")


def test_static_scratch_rejects_oversized_shapes():
    cap = _lib.lib().iron_decode_attn_static_capacity_bytes()
    assert cap == 8 << 20
    batch, H, HD, S = 64, 32, 128, 32768
    assert _lib.lib().iron_decode_attn_workspace_bytes(batch, H, HD, S) > cap
    q = torch.zeros(1, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.IronError, match="needs .* bytes of scratch"):
        _lib.call("iron_decode_attn_static", q.data_ptr(), q.data_ptr(), q.data_ptr(), batch, H, 8, HD, S,
                  0, 0, 1, None, _lib.stream_ptr())


def test_static_scratch_block_layout_against_oracle():
    """IRON's block layout ([K_block | V_block] per block_kv positions, kv_layout 2,
    decode_attn.cc:95-97) with block_kv 64 at a length that ends inside a block, twice:
    against the oracle's decode attention (decode_attn/reference.py:26-38) and
    bit-for-bit against the workspace entry point."""
    rng = np.random.default_rng(5)
    H, KV, HD, S, B = 16, 8, 128, 512, 64
    Q = rnd(rng.standard_normal((H, HD)).astype(np.float32))
    K = rnd(rng.standard_normal((KV, S, HD)).astype(np.float32))
    V = rnd(rng.standard_normal((KV, S, HD)).astype(np.float32))
    kv = dev_bf16(np.concatenate([K.reshape(KV, S // B, B, HD), V.reshape(KV, S // B, B, HD)],
                                 axis=2).reshape(KV, -1))
    q = dev_bf16(Q)
    n = _lib.lib().iron_decode_attn_workspace_bytes(1, H, HD, S)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    for L in (300, 449):
        got = torch.empty(H, HD, dtype=torch.bfloat16, device="cuda")
        want_ws = torch.empty(H, HD, dtype=torch.bfloat16, device="cuda")
        _lib.call("iron_decode_attn_static", q.data_ptr(), kv.data_ptr(), got.data_ptr(), 1, H, KV, HD, S, 2, B,
                  L, None, _lib.stream_ptr())
        _lib.call("iron_decode_attn", q.data_ptr(), kv.data_ptr(), want_ws.data_ptr(), 1, H, KV, HD, S, 2, B, L,
                  None, ws.data_ptr(), n, _lib.stream_ptr())
        torch.cuda.synchronize()
        assert_close(host(got), ops.decode_attention(Q, K, V, L - 1, HD, H, KV), what=f"static, block layout, L={L}")
        assert torch.equal(got, want_ws)
