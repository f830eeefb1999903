"""C-ABI library loads and exports every entry point the header declares (no GPU needed)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "dflash_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dfl_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n


def test_ctypes_signatures_cover_header(lib):
    from dflash_b200 import _lib
    assert set(_declared()) == set(_lib.SIGNATURES)


def test_abi_version_and_error_string(lib):
    assert lib.dfl_abi_version() == 1
    assert isinstance(lib.dfl_last_error(), bytes)


def test_host_side_argument_errors_are_reported(lib):
    """Invalid arguments are rejected before any launch (works without a GPU)."""
    from dflash_b200 import _lib
    import pytest
    with pytest.raises(_lib.DFlashKernelError) as e:
        _lib.call("dfl_gemm_bf16", None, 0, None, 16, 64, 64, 0, None, 0, None, 0, None, 0, None, None, None, 0,
                  1e-6, None, None, 0, None)
    assert e.value.status == 1
    with pytest.raises(_lib.DFlashKernelError) as e:
        _lib.call("dfl_attention", 1, 1, 1, 0, 0, 1, None, None, 0, 16, 32, 8, 96, 1, 1.0, 16, 0, 1, 0, None, 0, 0, 1, 1 << 30,
                  None)
    assert e.value.status == 2  # head_dim 96 unsupported
