"""ctypes mirror of the step-level C ABI (``dfl_ctx_*``, ``dfl_draft_step``,
``dfl_verify_step``, ``dfl_rollback`` in include/dflash_b200.h).

``StepContext`` builds the C descriptions from a GPU ``TargetModel`` / ``DraftModel``
(the context borrows their packed weights, which must outlive it) and drives the decode
loop body from C: this is the binding a non-Python host reproduces with its own FFI
(reference loop: dflash_mlx/runtime.py:406-518).
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_void_p

import torch

from . import _lib
from .runtime import STATE_INTS


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("in_norm", "post_norm", "w_qkv", "w_o", "w_gu", "w_down", "q_norm",
                                        "k_norm")]


class Qwen3Desc(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                                     "rope_dim")] + \
               [("eps", c_float), ("rope_theta", c_float), ("embed", c_void_p), ("lm_head", c_void_p),
                ("final_norm", c_void_p), ("layers", POINTER(LayerWeights))]


class DraftDesc(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "block_size",
                                     "mask_token_id", "n_taps", "causal")] + \
               [("eps", c_float), ("rope_theta", c_float), ("target_layer_ids", POINTER(ctypes.c_int32)),
                ("fc", c_void_p), ("hidden_norm", c_void_p), ("final_norm", c_void_p), ("w_ctx_kv", c_void_p),
                ("layers", POINTER(LayerWeights))]


CTX_NO_GRAPH = 1


def _layers(layers) -> ctypes.Array:
    arr = (LayerWeights * max(1, len(layers)))()
    for i, lw in enumerate(layers):
        arr[i] = LayerWeights(*(lw[k].data_ptr() for k in ("in_norm", "post_norm", "w_qkv", "w_o", "w_gu", "w_down",
                                                           "q_norm", "k_norm")))
    return arr


def target_desc(target) -> tuple[Qwen3Desc, list]:
    c = target.cfg
    arr = _layers(target.layers)
    d = Qwen3Desc(c.hidden_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, c.head_dim,
                  c.intermediate_size, c.vocab_size, c.rope_dim, c.rms_norm_eps, c.rope_theta,
                  target.embed_w.data_ptr(), target.lm_head_w.data_ptr(), target.norm_w.data_ptr(), arr)
    return d, [arr]


def draft_desc(draft) -> tuple[DraftDesc, list]:
    c = draft.cfg
    arr = _layers(draft.layers)
    ids = (ctypes.c_int32 * len(c.target_layer_ids))(*sorted(c.target_layer_ids))
    d = DraftDesc(c.hidden_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, c.head_dim,
                  c.intermediate_size, c.block_size, c.mask_token_id, len(c.target_layer_ids),
                  int(draft.mask_mode == "causal"), c.rms_norm_eps, c.rope_theta, ids, draft.fc.data_ptr(),
                  draft.hidden_norm.data_ptr(), draft.norm_w.data_ptr(), draft.w_ctx_kv.data_ptr(), arr)
    return d, [arr, ids]


class StepContext:
    """One ``dfl_ctx``: B sequences decoded together by C-level step calls."""

    def __init__(self, target, draft, batch: int, max_total: int, block_size: int,
                 stop_token_ids=(), max_steps: int | None = None, use_graph: bool = True):
        self.lib = _lib.load()
        self.B, self.bs = batch, block_size
        td, keep = target_desc(target)
        dd, keep2 = draft_desc(draft) if draft is not None else (None, [])
        self._keep = keep + keep2 + [td, dd, target, draft]
        stops = sorted(stop_token_ids)
        sarr = (ctypes.c_int32 * max(1, len(stops)))(*stops)
        h = c_void_p()
        _lib.call("dfl_ctx_create", ctypes.byref(td), ctypes.byref(dd) if dd is not None else None, batch, max_total,
                  block_size, sarr, len(stops), int(max_steps or 0), 0 if use_graph else CTX_NO_GRAPH,
                  ctypes.byref(h))
        self.h = h
        st, tok, lg = c_void_p(), c_void_p(), c_void_p()
        ostride, lstride = c_int64(), c_int64()
        _lib.call("dfl_ctx_buffers", h, ctypes.byref(st), ctypes.byref(tok), ctypes.byref(ostride), ctypes.byref(lg),
                  ctypes.byref(lstride))
        self.out_stride, self.log_stride = ostride.value, lstride.value
        self.log_ptr = lg.value

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream

    def prefill(self, seq: int, prompt: list[int], max_new_tokens: int) -> None:
        arr = (ctypes.c_int32 * len(prompt))(*prompt)
        _lib.call("dfl_ctx_prefill", self.h, seq, arr, len(prompt), max_new_tokens, self._stream())

    def set_injection(self, trace: torch.Tensor, lengths: torch.Tensor, noise: torch.Tensor) -> None:
        self._inj = (trace, lengths, noise)
        _lib.call("dfl_ctx_set_injection", self.h, trace.data_ptr(), trace.stride(0), lengths.data_ptr(),
                  lengths.stride(0), noise.data_ptr(), noise.stride(0))

    def step(self) -> None:
        s = self._stream()
        _lib.call("dfl_draft_step", self.h, s)
        _lib.call("dfl_verify_step", self.h, s)
        _lib.call("dfl_rollback", self.h, s)

    def read(self) -> tuple[torch.Tensor, torch.Tensor]:
        st = torch.zeros((self.B, STATE_INTS), dtype=torch.int32)
        tok = torch.zeros((self.B, self.out_stride), dtype=torch.int32)
        _lib.call("dfl_ctx_read", self.h, st.data_ptr(), tok.data_ptr(), self._stream())
        return st, tok

    def outputs(self) -> list[list[int]]:
        """Committed tokens of every sequence, truncated like runtime.py:499-507, 518."""
        st, tok = self.read()
        outs = []
        for b in range(self.B):
            start, stop, total = int(st[b, 0]), int(st[b, 6]), int(st[b, 8])
            n = start + 1
            if stop >= 0:
                n = min(n, stop + 1)
            outs.append(tok[b, :min(n, total)].tolist())
        return outs

    def close(self) -> None:
        if self.h:
            _lib.call("dfl_ctx_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
