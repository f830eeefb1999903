"""ctypes binding of the C ABI declared in include/dflash_b200.h.

The shared library is built in-tree by ``_build.build()``. There is no CPU
fallback: if the library is missing or a CUDA device is absent, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

from ._build import LIB_PATH

c_int32_p = POINTER(ctypes.c_int32)


class DFlashKernelError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, name: str, status: int, message: str):
        super().__init__(f"{name} failed with status {status}: {message}")
        self.status = status


# name -> (restype, argtypes); mirrors include/dflash_b200.h
SIGNATURES: dict[str, tuple] = {
    "dfl_abi_version": (c_int, []),
    "dfl_last_error": (c_char_p, []),
    "dfl_gemm_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "dfl_gemm_argmax_tiles": (c_int, [c_int]),
    "dfl_gemm_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p,
                              c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_float, c_void_p,
                              c_void_p, c_size_t, c_void_p]),
    "dfl_gemm_chain_workspace_bytes": (c_size_t, [c_void_p, c_int]),
    "dfl_gemm_chain": (c_int, [c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "dfl_gemm_bf16_wide": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64,
                                   c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_float,
                                   c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "dfl_gemm_wide_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "dfl_device_error": (c_int, [POINTER(c_int), c_int, c_void_p]),
    "dfl_sample_keys": (c_int, [c_void_p, c_int, c_int, ctypes.c_uint64, c_int, c_int, c_void_p, c_void_p]),
    "dfl_sample_partials": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_float, c_void_p, c_void_p]),
    "dfl_tp_alloc": (c_int, [c_size_t, POINTER(c_void_p), POINTER(ctypes.c_ubyte)]),
    "dfl_tp_open": (c_int, [POINTER(ctypes.c_ubyte), POINTER(c_void_p)]),
    "dfl_tp_close": (c_int, [c_void_p]),
    "dfl_tp_free": (c_int, [c_void_p]),
    "dfl_tp_reduce_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                                       c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p]),
    "dfl_tp_reduce_residual_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                                            c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p,
                                            c_float, c_void_p, c_int64, c_void_p]),
    "dfl_packed_weight_bytes": (c_size_t, [c_int, c_int]),
    "dfl_gemm_noalloc_scratch_bytes": (c_size_t, []),
    "dfl_gemm_bf16_noalloc": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int64,
                                      c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                                      c_float, c_void_p, c_void_p]),
    "dfl_pack_weight_bf16": (c_int, [c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "dfl_rmsnorm_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_float, c_void_p]),
    "dfl_embed_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p]),
    "dfl_gemm_qkv_rope": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_float,
                                  c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int,
                                  c_void_p, c_size_t, c_void_p]),
    "dfl_gemm_kv_append_layers": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
                                          c_float, c_void_p, c_int64, c_void_p, c_void_p, POINTER(c_void_p),
                                          c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                                          c_int64, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "dfl_gemm_qkv_rope_launches": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "dfl_qkv_rope_append": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int,
                                    c_float, c_int, c_void_p]),
    "dfl_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "dfl_attention_qkv": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                  c_int64, c_int64, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_int,
                                  c_int, c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "dfl_qkv_rope_append_paged": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int,
                                          c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_void_p]),
    "dfl_attention_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int,
                                    c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                    c_int, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_size_t,
                                    c_void_p]),
    "dfl_attention_launches": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "dfl_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                              c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_int64, c_void_p,
                              c_int64,
                              c_int, c_void_p, c_size_t, c_void_p]),
    "dfl_gdn_prep": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                             c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_float, c_void_p]),
    "dfl_gdn_rollback": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int,
                                 c_int, c_int, c_int, c_void_p]),
    "dfl_gated_rmsnorm": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int,
                                  c_int, c_float, c_void_p]),
    "dfl_argmax_reduce": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "dfl_step_prepare": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_int, c_void_p]),
    "dfl_draft_commit": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64,
                                 c_void_p, c_int64, c_int, c_void_p]),
    "dfl_verify_accept": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p,
                                  c_int, c_void_p, c_int64, c_int, c_void_p]),
    "dfl_ctx_create": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int,
                               POINTER(c_void_p)]),
    "dfl_ctx_destroy": (c_int, [c_void_p]),
    "dfl_ctx_prefill": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p]),
    "dfl_ctx_set_injection": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64]),
    "dfl_draft_step": (c_int, [c_void_p, c_void_p]),
    "dfl_verify_step": (c_int, [c_void_p, c_void_p]),
    "dfl_rollback": (c_int, [c_void_p, c_void_p]),
    "dfl_ctx_buffers": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int64), POINTER(c_void_p),
                                POINTER(c_int64)]),
    "dfl_ctx_read": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "dfl_gdr_recurrence": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                   c_int, c_void_p]),
}

_LIB: ctypes.CDLL | None = None


def library_path() -> Path:
    return LIB_PATH


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Loads (once) the C-ABI library; raises if it has not been built."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else Path(os.environ.get("DFLASH_B200_LIB", LIB_PATH))
    if not p.exists():
        raise RuntimeError(
            f"dflash-b200 native library not found at {p}; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a). There is no CPU fallback."
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.dfl_last_error().decode(errors="replace")
        raise DFlashKernelError(name, status, msg)


def query(name: str, *args):
    return getattr(load(), name)(*args)
