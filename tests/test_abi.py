"""The C ABI library loads and exports every symbol include/twilight_b200.h
declares; argument validation runs on the host (no kernel is launched)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "include" / "twilight_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tw_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(tw):
    lib = tw.load_library()
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
        assert name in tw._lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(tw._lib.SIGNATURES) == set(names)


def test_status_strings(tw):
    lib = tw.load_library()
    assert lib.tw_abi_version() == 3
    for code in range(8):
        assert lib.tw_status_string(code)
    assert tw._lib.status_string(1) == "row index out of bounds"
    with pytest.raises(ValueError, match="out of bounds"):
        tw._lib.check(1)
    with pytest.raises(RuntimeError):
        tw._lib.check(3)


def test_host_side_argument_checks(tw):
    lib = tw.load_library()
    L = tw._lib
    # unsupported head_dim / R, bad k, bad row size: rejected before any launch
    assert lib.tw_quest_score(None, None, None, 1, 1, 1, 128, 64, 0, None, None) == L.TW_ERR_UNSUPPORTED
    assert lib.tw_topk_pages(None, 1, 4, 5, None, None) == L.TW_ERR_BAD_ARG
    assert lib.tw_gather_kv(None, None, None, None, None, 0, 10, 256, None, None) == L.TW_OK
    assert lib.tw_gather_kv(None, None, None, None, None, 5, 10, 250, None, None) == L.TW_ERR_BAD_ARG
    assert lib.tw_int4_pack(None, 0, 1, 1, 128, 16, 0, None, None, None, 0, 0, None) == L.TW_ERR_UNSUPPORTED
    assert lib.tw_top_p_union(None, None, 1, 9, 1, 16, 0, 0.9, 10, 0, 0, None, 10, None, None, None,
                              None, None) == L.TW_ERR_BAD_ARG
    assert lib.tw_decode_attention(None, None, None, None, 1, 4, 10, 64, 0, ctypes.c_float(1.0),
                                   None, 0, None, None, 0, None) == L.TW_ERR_UNSUPPORTED
    assert lib.tw_decode_attention_workspace_size(8, 4, 4096, 128) > 0
    assert lib.tw_select_layer_workspace_size(8, 4, 2028, 256, 16) >= 8 * 4 * (2028 + 4096) * 4


def test_decode_layer_args_layout(tw):
    """The ctypes mirror of tw_decode_layer_args has the C struct's size and a
    plausible field layout (pointers 8-byte aligned)."""
    lib = tw.load_library()
    S = tw._lib.DecodeLayerArgs
    assert ctypes.sizeof(S) == lib.tw_decode_layer_args_size()
    for name, ctype in S._fields_:
        if ctype in (ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_size_t):
            assert getattr(S, name).offset % 8 == 0, name
    assert lib.tw_twilight_decode_layer(None, None) == tw._lib.TW_ERR_BAD_ARG
    assert S.stage_rows.offset == ctypes.sizeof(S) - 8
    assert S.stage_k.offset == S.reuse.offset + 8
    assert ctypes.sizeof(tw._lib.RowReuse) == lib.tw_row_reuse_size()
