"""Tensor parallelism for the Qwen3.5 hybrid target (benchmark config 5: Qwen3.5-27B, batch 8, context 32768).

Sharding follows the reference's ``Model.shard`` (custom_qwen35_model.py:1286-1402):

* gated-delta layers: ``in_proj_qkv`` and the depthwise conv split by key / value
  head inside each of the q, k, v segments; ``in_proj_z``, ``in_proj_b``,
  ``in_proj_a``, ``dt_bias``, ``A_log`` split by value head; ``out_proj`` split
  along its input (row-parallel, followed by an all-sum);
* gated full attention: ``q_proj`` (per head [q | gate]) split by query head,
  ``k_proj`` / ``v_proj`` split by kv head, each kv head repeated first when there
  are more ranks than kv heads (custom_qwen35_model.py:1295-1308); ``o_proj``
  row-parallel;
* MLP: ``gate_proj`` / ``up_proj`` split by output row, ``down_proj`` row-parallel;
* embedding, final norm, lm_head and the draft are replicated.

The all-sum after each row-parallel projection is ``dfl_tp_reduce_residual``: each
rank's GEMM writes its fp32 partial into a peer-mapped slot; one kernel per call sums
the N partials in rank order from peer memory and applies the residual add, the tap
copy and the next RMSNorm's row sums of squares (the same bits on every rank, for
any number of rows).
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch

from . import _lib
from .config import TargetConfig


# ---------------------------------------------------------------------------
# weight sharding (host, device-agnostic)
# ---------------------------------------------------------------------------
def shard_config(cfg: TargetConfig, size: int) -> TargetConfig:
    """The per-rank geometry: heads and FFN rows divided by the rank count."""
    if size == 1:
        return cfg
    for name, v in (("num_attention_heads", cfg.num_attention_heads), ("intermediate_size", cfg.intermediate_size),
                    ("linear_num_key_heads", cfg.linear_num_key_heads),
                    ("linear_num_value_heads", cfg.linear_num_value_heads)):
        if v % size:
            raise ValueError(f"{name}={v} is not divisible by {size} ranks")
    if cfg.num_key_value_heads % size and size % cfg.num_key_value_heads:
        raise ValueError(f"{cfg.num_key_value_heads} kv heads cannot be spread over {size} ranks")
    return dataclasses.replace(
        cfg, num_attention_heads=cfg.num_attention_heads // size,
        num_key_value_heads=max(1, cfg.num_key_value_heads // size),
        intermediate_size=cfg.intermediate_size // size,
        linear_num_key_heads=cfg.linear_num_key_heads // size,
        linear_num_value_heads=cfg.linear_num_value_heads // size)


def _rows(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[0] // size
    return t[rank * n:(rank + 1) * n]


def _cols(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[1] // size
    return t[:, rank * n:(rank + 1) * n]


def _kv_rows(t: torch.Tensor, n_kv: int, hd: int, rank: int, size: int) -> torch.Tensor:
    """kv head slice for this rank; with more ranks than kv heads each head is
    repeated size / n_kv times first."""
    if size <= n_kv:
        return _rows(t, rank, size)
    h = rank // (size // n_kv)
    return t[h * hd:(h + 1) * hd]


def shard_weights(cfg: TargetConfig, weights: dict, rank: int, size: int) -> dict:
    """This rank's share of a qwen3_5 target's weights (same keys as the full set)."""
    if size == 1:
        return weights
    out = {k: v for k, v in weights.items() if k != "layers"}
    out["layers"] = [shard_layer(cfg, i, lw, rank, size) for i, lw in enumerate(weights["layers"])]
    return out


def shard_layer(cfg: TargetConfig, i: int, lw: dict, rank: int, size: int) -> dict:
    """This rank's share of layer i's weights."""
    if size == 1:
        return lw
    kd = cfg.linear_key_head_dim * cfg.linear_num_key_heads
    hd, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    s = {"input_layernorm": lw["input_layernorm"], "post_attention_layernorm": lw["post_attention_layernorm"],
         "gate_proj": _rows(lw["gate_proj"], rank, size), "up_proj": _rows(lw["up_proj"], rank, size),
         "down_proj": _cols(lw["down_proj"], rank, size)}
    if cfg.is_linear_layer(i):
        qkv, conv = lw["in_proj_qkv"], lw["conv1d"]
        seg = lambda t: torch.cat([_rows(t[:kd], rank, size), _rows(t[kd:2 * kd], rank, size),  # noqa: E731
                                   _rows(t[2 * kd:], rank, size)], 0)
        s.update({"in_proj_qkv": seg(qkv), "conv1d": seg(conv), "in_proj_z": _rows(lw["in_proj_z"], rank, size),
                  "in_proj_b": _rows(lw["in_proj_b"], rank, size), "in_proj_a": _rows(lw["in_proj_a"], rank, size),
                  "dt_bias": _rows(lw["dt_bias"], rank, size), "A_log": _rows(lw["A_log"], rank, size),
                  "norm": lw["norm"], "out_proj": _cols(lw["out_proj"], rank, size)})
    else:
        qh = Hq // size
        s.update({"q_proj": lw["q_proj"][rank * qh * 2 * hd:(rank + 1) * qh * 2 * hd],
                  "k_proj": _kv_rows(lw["k_proj"], Hkv, hd, rank, size),
                  "v_proj": _kv_rows(lw["v_proj"], Hkv, hd, rank, size),
                  "o_proj": lw["o_proj"][:, rank * qh * hd:(rank + 1) * qh * hd],
                  "q_norm": lw["q_norm"], "k_norm": lw["k_norm"]})
    return {k: v.contiguous() for k, v in s.items()}


# ---------------------------------------------------------------------------
# peer-mapped partial buffers
# ---------------------------------------------------------------------------
class _CudaArray:
    """__cuda_array_interface__ over raw device memory (fp32 elements)."""

    def __init__(self, ptr: int, shape: tuple[int, ...]):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


class TPComm:
    """One rank's peer-mapped all-sum state: two partial slots [max_rows, hidden] fp32
    (call parity), a flag array per rank, the call counter. Built collectively."""

    FLAG_BYTES = 256
    MAX_SLABS = 4  # K-range partial slabs a wide GEMM may leave per call (ops.wide_split limit)

    def __init__(self, rank: int, size: int, device: torch.device, max_rows: int, hidden: int, group=None):
        import torch.distributed as dist
        if size > 8:
            raise ValueError("at most 8 ranks")
        self.rank, self.size, self.device = rank, size, torch.device(device)
        self.max_rows, self.hidden = max_rows, hidden
        self.slot_bytes = self.MAX_SLABS * max_rows * hidden * 4
        nbytes = 2 * self.slot_bytes + self.FLAG_BYTES
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.call("dfl_tp_alloc", ctypes.c_size_t(nbytes), ctypes.byref(ptr), handle)
        self.local = ptr.value
        handles = [None] * size
        if size > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        else:
            handles = [bytes(handle)]
        self.peers = []
        for j in range(size):
            if j == rank:
                self.peers.append(self.local)
            else:
                p = ctypes.c_void_p()
                h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[j])
                _lib.call("dfl_tp_open", h, ctypes.byref(p))
                self.peers.append(p.value)
        self._lib = lib
        dev = self.device
        arr = ctypes.c_void_p * size
        self.parts_arr = [arr(*[p + par * self.slot_bytes for p in self.peers]) for par in (0, 1)]
        self.flags_arr = arr(*[p + 2 * self.slot_bytes for p in self.peers])
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)  # [epoch, done]
        self.slots = [torch.as_tensor(_CudaArray(self.local + par * self.slot_bytes,
                                                 (self.MAX_SLABS * max_rows * hidden,)), device=dev)
                      for par in (0, 1)]
        if size > 1:
            torch.cuda.synchronize(dev)
            dist.barrier(group=group)

    def partial(self, parity: int, M: int, slabs: int = 1) -> torch.Tensor:
        """This rank's partial slot for a call of the given parity: [M, hidden], or
        [slabs, M, hidden] K-range slabs."""
        if M > self.max_rows or slabs > self.MAX_SLABS:
            raise ValueError(f"{slabs} x {M} rows exceed the all-sum buffer ({self.MAX_SLABS} x {self.max_rows})")
        v = self.slots[parity][:slabs * M * self.hidden]
        return v.view(M, self.hidden) if slabs == 1 else v.view(slabs, M, self.hidden)

    def reduce_residual(self, parity: int, h: torch.Tensor, tap: torch.Tensor | None, sumsq_out: torch.Tensor | None,
                        M: int, slabs: int = 1, norm_w: torch.Tensor | None = None, eps: float = 0.0,
                        xn: torch.Tensor | None = None) -> None:
        """h[:M] <- h + sum over ranks (and K-range slabs) of the parity slot; tap copy;
        row sums of squares; with norm_w, also xn = RMSNorm(h) * norm_w (the next
        projection's input, the same bits as that projection's own norm)."""
        from .ops import _ptr, _row_stride, _stream
        args = (self.parts_arr[parity], self.flags_arr, self.counters.data_ptr(), self.counters.data_ptr() + 4,
                self.rank, self.size, slabs, M * self.hidden, _ptr(h), _row_stride(h), _ptr(tap),
                _row_stride(tap) if tap is not None else 0, _ptr(sumsq_out), M, self.hidden)
        if norm_w is None:
            _lib.call("dfl_tp_reduce_residual", *args, _stream())
        else:
            _lib.call("dfl_tp_reduce_residual_norm", *args, _ptr(norm_w), float(eps), _ptr(xn), _row_stride(xn),
                      _stream())

    def close(self) -> None:
        for j, p in enumerate(self.peers):
            if j != self.rank and p:
                _lib.call("dfl_tp_close", ctypes.c_void_p(p))
        self.slots = []
        if self.local:
            torch.cuda.synchronize(self.device)
            _lib.call("dfl_tp_free", ctypes.c_void_p(self.local))
            self.local = 0
