"""The C-ABI library loads and exports every symbol the header declares (no GPU)."""

import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "loraforge_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int64_t|int|const char\*)\s+(lf_\w+)\(", text, re.M)))


def test_header_and_binding_agree():
    from loraforge_b200 import _native

    assert declared_symbols() == sorted(_native.exported_symbols())


def test_library_exports_every_declared_symbol():
    from loraforge_b200 import _native

    lib = _native.library()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.lf_version() >= 100
    assert lib.lf_last_error_string() == b""


def test_invalid_arguments_fail_before_any_device_work():
    # Argument validation runs on the host and reports through lf_last_error_string.
    from loraforge_b200 import _native

    with pytest.raises(RuntimeError, match="row_tile must"):
        _native.call(
            "lf_row_expand", *([None] * 5), 8, *([None] * 7), 4, 8, 1, 16, 1, 1, 1, 256, 3, None
        )
    with pytest.raises(RuntimeError, match="num_slots"):
        _native.call("lf_group_tokens", None, 4, 0, 16, None, None, None, None, None)
    with pytest.raises(RuntimeError, match="num_slots"):
        _native.call("lf_group_token_runs", None, 4, 0, 16, None, None, None, None, None)
    with pytest.raises(RuntimeError, match="must not alias"):
        _native.call("lf_split_runs", 8, 16, 24, 32, 4, 16, 8, 40, 48, None)
    with pytest.raises(RuntimeError, match="aligned"):
        _native.call(
            "lf_row_shrink", 2, 8, 16, 16, None, None, 4, 8, 1, 1, 16, 16, None
        )


def test_slice_descriptor_layout_matches_header():
    from loraforge_b200 import _native

    assert ctypes.sizeof(_native.SliceDesc) == 32


def test_library_built_for_sm100a():
    # cuobjdump/ SASS inspection is not used; the build flags are the contract.
    from loraforge_b200 import _build

    assert "arch=compute_100a,code=sm_100a" in _build.ARCH


def test_import_is_lazy():
    code = (
        "import sys; import loraforge_b200.ops, loraforge_b200.ops.vllm_gemv;"
        "assert 'torch' not in sys.modules, 'torch imported eagerly'"
    )
    subprocess.run([sys.executable, "-c", code], check=True, cwd=ROOT)
