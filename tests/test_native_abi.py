"""CPU checks of the C-ABI boundary: the shared library loads, exports every
entry point include/tpp_b200.h declares, and the ctypes signature table covers
exactly those entry points.  No kernel is launched."""
import re
from pathlib import Path

import pytest

from torchplusplus_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "tpp_b200.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|int64_t|uint64_t|const char\*)\s+(tpp_\w+)\s*\(", text,
                          flags=re.M))


def test_header_declares_entry_points():
    names = declared()
    assert {"tpp_rmsnorm", "tpp_linear", "tpp_attention_prefill", "tpp_attention_decode"} <= names


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in sorted(declared()):
        assert hasattr(lib, name), f"{name} declared in tpp_b200.h but not exported"


def test_signature_table_matches_header():
    assert set(N.SIGNATURES) == declared()


def test_version_and_error_strings_without_gpu():
    lib = N.lib()
    assert b"sm_100a" in lib.tpp_version()
    assert isinstance(lib.tpp_last_error(), bytes)


def test_argument_validation_needs_no_gpu():
    # shape errors are caught on the host before any launch
    with pytest.raises(N.TppError) as e:
        N.call("tpp_rmsnorm", None, 0, None, None, 0, 1, 0, 1e-6, 0, None)
    assert e.value.status == 1
    with pytest.raises(N.TppError) as e:
        N.call("tpp_attention_prefill", 16, 0, 0, 0, 16, 0, 0, 0, 16, 0, 0, 0, 16, 0, 0, 0,
               1, 1, 1, 2, 1, 96, 1, -1, 1.0, 0, None)
    assert e.value.status == 6  # head dim 96 unsupported
    # decode workspace query is pure host arithmetic
    assert N.lib().tpp_attention_decode_workspace(1, 16, 8, 128) >= 0


def test_persistent_row_pad_matches_header():
    """The Python side pads the persistent step's weight copies by the pitch
    the kernel expects (TPP_PERSISTENT_ROW_PAD)."""
    from torchplusplus_b200 import ops
    m = re.search(r"#define\s+TPP_PERSISTENT_ROW_PAD\s+(\d+)", HEADER.read_text())
    assert m and int(m.group(1)) == ops.PERSISTENT_ROW_PAD
