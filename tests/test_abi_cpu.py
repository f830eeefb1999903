"""C-ABI library loads and exports every entry point the header declares (no GPU needed)."""
import os
import re

import pytest

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


def test_argument_errors_are_reported_without_a_device(lib):
    """Entry points validate their arguments before any CUDA call: the status codes and the
    thread-local message of dfl_last_error (no GPU needed)."""
    import ctypes

    from dflash_b200 import _lib
    from dflash_b200._lib import DFlashKernelError
    cases = [
        # (entry point, args, expected status, message fragment)
        ("dfl_sample_keys", (None, 2, 16, ctypes.c_uint64(1), 2, 1, None, None), 1, "dfl_sample_keys"),
        ("dfl_sample_partials", (None, 10, 2, 10, None, 0.0, None, None), 1, "dfl_sample_partials"),
        ("dfl_attention_qkv", (None, 0, None, None, None, 1e-6, None, None, 0, 0, None, None, 0, 16, 32, 8, 1.0,
                               64, 0, None, 0, None, 0, None), 1, "dfl_attention_qkv"),
        ("dfl_tp_reduce_residual", (None, None, None, None, 0, 1, 1, 0, None, 0, None, 0, None, 16, 256, None), 1,
         "dfl_tp_reduce_residual"),
    ]
    for name, args, status, frag in cases:
        with pytest.raises(DFlashKernelError) as e:
            _lib.call(name, *args)
        assert e.value.status == status, name
        assert frag in str(e.value), name
    # zero-sized calls are no-ops that succeed
    _lib.call("dfl_sample_keys", None, 0, 16, ctypes.c_uint64(1), 2, 1, None, None)
    _lib.call("dfl_attention_qkv", None, 0, None, None, None, 1e-6, None, None, 0, 0, None, None, 0, 0, 32, 8, 1.0,
              64, 0, None, 0, None, 0, None)


def test_fused_attention_rejects_sequences_that_span_tiles(lib):
    """dfl_attention_qkv refuses layouts whose sequences cross 16-row tiles (status 2)."""
    import ctypes

    from dflash_b200 import _lib
    from dflash_b200._lib import DFlashKernelError
    dummy = ctypes.c_void_p(16)  # never dereferenced: the layout check comes first
    with pytest.raises(DFlashKernelError) as e:
        _lib.call("dfl_attention_qkv", dummy, (32 + 16) * 128, dummy, dummy, dummy, 1e-6, dummy, dummy, 0, 0,
                  dummy, dummy, 3, 48, 32, 8, 1.0, 64, 0, dummy, 4096, None, 0, None)
    assert e.value.status == 2 and "16-row tile" in str(e.value)


def test_step_abi_rejects_bad_arguments_without_a_device():
    """The step-level driver's argument checks run before any CUDA call."""
    import ctypes
    from dflash_b200 import _lib
    lib = _lib.load()
    h = ctypes.c_void_p()
    assert lib.dfl_ctx_create(None, None, 1, 64, 1, None, 0, 0, 0, ctypes.byref(h)) == 1
    assert b"invalid" in lib.dfl_last_error()
    for fn in ("dfl_draft_step", "dfl_verify_step", "dfl_rollback"):
        assert getattr(lib, fn)(None, None) == 1
    assert lib.dfl_ctx_destroy(None) == 0


def test_fused_projection_appends_reject_bad_arguments_without_a_device():
    """dfl_gemm_qkv_rope and dfl_gemm_kv_append_layers check their pointers, head geometry and
    layer count (at most 16) before any CUDA call; the launch-count query answers on the
    host for both (Hq = 0 with the layers' kv heads for the multi-layer form)."""
    import ctypes
    from dflash_b200 import _lib
    from dflash_b200._lib import DFlashKernelError
    d = ctypes.c_void_p(16)  # never dereferenced
    with pytest.raises(DFlashKernelError) as e:  # null positions
        _lib.call("dfl_gemm_qkv_rope", d, 2560, d, 16, 2560, None, None, 0, 1e-6, d, 6144, None, None, d, d, d, d, d,
                  d, 0, 0, None, 0, 0, 32, 8, 128, d, 1 << 20, None)
    assert e.value.status == 1
    norms = (ctypes.c_void_p * 17)(*([16] * 17))
    with pytest.raises(DFlashKernelError) as e:  # 17 layers
        _lib.call("dfl_gemm_kv_append_layers", d, 2560, d, 16, 2560, None, None, 0, 1e-6, d, 17 * 2048, d, None,
                  norms, d, d, d, 0, 0, 0, None, 0, 0, 17, 8, 128, d, 1 << 20, None)
    assert e.value.status == 1 and "16 layers" in str(e.value)
    lib = _lib.load()
    assert lib.dfl_gemm_qkv_rope_launches(16, 2560, 32, 8, 128) == 1  # cluster form, one row tile
    assert lib.dfl_gemm_qkv_rope_launches(20, 2560, 32, 8, 128) == 2  # two row tiles
    assert lib.dfl_gemm_qkv_rope_launches(16, 256, 4, 2, 64) == 2  # head_dim 64
    assert lib.dfl_gemm_qkv_rope_launches(16, 2560, 0, 40, 128) == 1  # five layers' context K/V
    assert lib.dfl_gemm_qkv_rope_launches(16, 100, 32, 8, 128) == -1


def test_tp_all_sum_norm_rejects_bad_arguments_without_a_device():
    """dfl_tp_reduce_residual_norm needs the norm weight, an output for the normed rows and a
    row width its shared memory holds (H <= 8192); it says so before any CUDA call."""
    import ctypes
    from dflash_b200 import _lib
    from dflash_b200._lib import DFlashKernelError
    d = ctypes.c_void_p(16)  # never dereferenced
    for norm_w, xn, H in ((None, d, 512), (d, None, 512), (d, d, 16384)):
        with pytest.raises(DFlashKernelError) as e:
            _lib.call("dfl_tp_reduce_residual_norm", d, d, d, d, 0, 1, 1, 0, d, H, None, 0, None, 4, H, norm_w, 1e-6,
                      xn, H, None)
        assert e.value.status == 1 and "8192" in str(e.value)
