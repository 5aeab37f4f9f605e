"""CPU tests: the C-ABI library loads and exports every declared symbol; host-side
layout logic (arg specs, wire geometry, sequence buffer layout) matches IRON's."""

import re
from pathlib import Path

import pytest

from iron_b200 import _lib
from iron_b200.operators import (DecodeAttention, GEMVInt8, QKVHeadDataParallelOurs, RMSNorm,
                                 SwiGLUMLPDataParallelOurs)
from iron_b200.sequence import OperatorSequence

HEADER = Path(__file__).resolve().parents[1] / "include" / "iron_b200.h"


def declared():
    txt = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(iron_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert L.iron_version().startswith(b"iron_b200")


def test_error_reporting_without_gpu():
    """Argument validation runs on the host and reports through iron_last_error; a
    rejected call launches nothing (iron_launch_count stays put)."""
    c0 = _lib.launch_count()
    with pytest.raises(_lib.IronError, match="group must be"):
        _lib.call("iron_gemv_w8a16", 16, 64, 1024, 48, 1, 0, 0, 0, 16, 1, None, 16, None, 0, None)
    with pytest.raises(_lib.IronError, match="batch 0 below 1"):
        _lib.call("iron_lm_head_bf16_argmax", 16, 8, 8, 16, 0, None, 16, 16, 0, None)
    assert _lib.launch_count() == c0 >= 0


def test_gemvint8_arg_spec_matches_reference_formula():
    # gemv_int8/op.py:156-171: num_batches * (M / tile_m) * (tile_m*K + tile_m*(K/128)*2) // 2
    for M, K, tsi in [(512, 1024, 2), (2048, 4096, 2), (8192, 2048, 4), (151936, 1024, 4)]:
        op = GEMVInt8(M=M, K=K, tile_size_input=tsi)
        assert op.get_arg_spec()[0].shape == ((M // tsi) * (tsi * K + tsi * (K // 128) * 2) // 2,)
    with pytest.raises(ValueError):
        GEMVInt8(M=512, K=1000)
    with pytest.raises(ValueError):
        GEMVInt8(M=512, K=1024, tile_size_input=4, tile_size_output=6)


def test_mlp_ours_wire_geometry_matches_qwen3_chain():
    """0.6B numbers of swiglu_mlp_dp/op_ours.py:_wo_tiling/_wo_units/_wg_units/_wd_units."""
    op = SwiGLUMLPDataParallelOurs(D=1024, FF=3072, num_aie_columns=8, fuse_o=True, QD=2048, epsilon=1e-6)
    n, n_o, tsi_o, wtile = op._wo_tiling()
    assert (n, n_o, tsi_o, wtile) == (8, 22, 6, 12480)
    spec = op.get_arg_spec()
    assert spec[3].shape == (8 * 22 * 12480 // 2,)
    assert spec[4].shape == (3072 * 520,) and spec[6].shape == (1024 * 1560,)
    assert [s.direction for s in spec] == ["in"] * 7 + ["inout", "inout", "out"]


def test_qkv_and_attention_arg_specs():
    q = QKVHeadDataParallelOurs(D=1024, HD=128, Hq=16, Hkv=8, max_seq=512, kv_offset_parameter="k_cache_offset")
    spec = q.get_arg_spec()
    assert spec[2].shape == (4096 * 1040 // 2,) and spec[-1].shape == (8 * 512 * 128 * 2,)
    assert q.get_params_used() == ("k_cache_offset",)
    a = DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=512, use_runtime_seq_len=True)
    assert [s.shape for s in a.get_arg_spec()] == [(16, 128), (8, 2 * 512 * 128), (16, 128)]
    assert a.get_params_used() == ("S_kv_eff",)
    with pytest.raises(ValueError):
        DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=500)
    # verify mode (decode_attn/op.py:156-181): token-major Q of num_new_tokens*H rows, a
    # taller O when out_buffer_tokens asks, and the S_kv_base runtime parameter
    v = DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=256, block_kv=32,
                        use_runtime_seq_len=True, batch_queries=8, num_new_tokens=16, out_buffer_tokens=32)
    assert [s.shape for s in v.get_arg_spec()] == [(16 * 16, 128), (8, 2 * 256 * 128), (32 * 16, 128)]
    assert v.get_params_used() == ("S_kv_base",)
    assert "m8" in v.name and "new16" in v.name
    with pytest.raises(ValueError, match="multiple"):
        DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=256, use_runtime_seq_len=True,
                        batch_queries=8, num_new_tokens=12)
    with pytest.raises(ValueError, match="use_runtime_seq_len"):
        DecodeAttention(num_heads=16, num_kv_heads=8, head_dim=128, seq_len_kv=256, batch_queries=8,
                        num_new_tokens=16)


def test_sequence_layout_slices_and_conflicts():
    r1 = RMSNorm(size=1024, num_aie_columns=1, num_channels=1, tile_size=1024, weighted=True, epsilon=1e-6)
    seq = OperatorSequence("t", [(r1, "x", "w", "y"), (r1, "y", "w", "big[0:2048]")], ["x"], ["big"],
                           buffer_sizes={"big": 4096})
    layout, total = seq.calculate_buffer_layout()
    assert layout["x"][1] == 2048 and layout["big"][1] == 4096
    assert layout["big[0:2048]"] == (layout["big"][0], 2048)
    assert all(off % 256 == 0 for name, (off, n) in layout.items() if "[" not in name)
    r2 = RMSNorm(size=2048, num_aie_columns=1, num_channels=1, tile_size=1024)
    with pytest.raises(ValueError, match="conflicting"):
        OperatorSequence("t", [(r1, "x", "w", "y"), (r2, "y", "x")], ["x"], ["x"]).calculate_buffer_layout()


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    """The product has no CPU path: without the built library every call raises."""
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libiron_b200.so")
    monkeypatch.setattr(_lib, "_LIB", None)
    with pytest.raises(ImportError, match="not built"):
        _lib.call("iron_gemv_w8a16", 16, 64, 1024, 32, 1, 0, 0, 0, 16, 1, None, 16, None, 0, None)
    with pytest.raises(ImportError, match="not built"):
        _lib.launch_count()
