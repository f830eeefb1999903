"""Torch-facing wrappers of the C-ABI kernels.

Each wrapper checks dtype / device / layout, passes raw device pointers and the
current CUDA stream to the C ABI and raises ``DFlashKernelError`` on a non-zero
status. Tensors must live on a CUDA device: there is no CPU path.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL, EPI_ARGMAX, EPI_STORE_F32, EPI_PARTIALS = 0, 1, 2, 3, 4, 5
ATTN_CHUNK = 128
KV_LAYERS_MAX = 16  # layers one dfl_gemm_kv_append_layers call appends


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("dflash-b200 ops take CUDA tensors only (no CPU fallback)")


def _row_stride(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"expected a 2-D row-major view, got shape {tuple(t.shape)} stride {t.stride()}")
    return t.stride(0)


class Workspace:
    """Per-device scratch for split-K GEMM partials and attention chunk partials.

    The GEMM region starts zeroed and the kernels leave their arrival counters at
    zero, so it is reusable across launches and CUDA-graph replays on one stream.
    ``wide`` selects the wide GEMM (whole-K tiles, for many rows) for every gemm()
    issued with this workspace; its RMSNorm prologue output lives in ``wide_x``.
    """

    CHAIN_BYTES = 6 << 20  # dfl_gemm_chain scratch: counters + one partial tile pair per CTA

    def __init__(self, device: torch.device, gemm_bytes: int = 64 << 20, attn_bytes: int = 64 << 20,
                 wide: bool = False, wide_split: int = 1):
        self.device = torch.device(device)
        self.chain = torch.zeros(self.CHAIN_BYTES, dtype=torch.uint8, device=self.device)
        self.gemm = torch.zeros(gemm_bytes, dtype=torch.uint8, device=self.device)
        self.attn = torch.empty(attn_bytes, dtype=torch.uint8, device=self.device)
        self.wide = wide
        self.wide_split = wide_split  # most K ranges a wide GEMM may split into
        self.wide_x = torch.empty(0, dtype=torch.uint8, device=self.device)

    def ensure_wide(self, nbytes: int) -> None:
        if nbytes > self.wide_x.numel():
            self.wide_x = torch.empty(nbytes, dtype=torch.uint8, device=self.device)

    def ensure_attn(self, nbytes: int) -> None:
        if nbytes > self.attn.numel():
            self.attn = torch.empty(nbytes, dtype=torch.uint8, device=self.device)

    def ensure_gemm(self, nbytes: int) -> None:
        if nbytes > self.gemm.numel():
            self.gemm = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)


_WS: dict[int, Workspace] = {}


def workspace(device: torch.device | None = None) -> Workspace:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None:
        ws = Workspace(torch.device("cuda", idx))
        _WS[idx] = ws
    return ws


class PackedWeight:
    """A [N, K] bf16 weight in the GEMM's pre-tiled HBM layout (dfl_pack_weight_bf16):
    128-row x 64-column units, each one contiguous 16 KB block in the tensor cores'
    128-byte-swizzled K-major image."""

    def __init__(self, w: torch.Tensor):
        _need_cuda(w)
        if w.dtype != torch.bfloat16 or w.dim() != 2:
            raise ValueError("pack_weight takes a 2-D bf16 matrix")
        w = w.contiguous()
        self.N, self.K = w.shape
        nbytes = int(_lib.query("dfl_packed_weight_bytes", self.N, self.K))
        if nbytes == 0:
            raise ValueError(f"cannot pack a [{self.N}, {self.K}] weight (K must be a multiple of 64)")
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
        _lib.call("dfl_pack_weight_bf16", _ptr(w), self.N, self.K, _ptr(self.data), nbytes, _stream())

    @property
    def shape(self) -> tuple[int, int]:
        return (self.N, self.K)

    @property
    def device(self) -> torch.device:
        return self.data.device

    def data_ptr(self) -> int:
        return self.data.data_ptr()


def pack_weight(w: torch.Tensor) -> PackedWeight:
    return PackedWeight(w)


def gemm(x: torch.Tensor, w: PackedWeight | torch.Tensor, epilogue: int = EPI_STORE, residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None, out2: torch.Tensor | None = None,
         argmax_partials: torch.Tensor | None = None, ws: Workspace | None = None,
         norm_w: torch.Tensor | None = None, sumsq_in: torch.Tensor | None = None, eps: float = 1e-6,
         sumsq_out: torch.Tensor | None = None) -> torch.Tensor:
    """y = xn @ w.T (bf16 in, fp32 accumulate) with a fused epilogue; xn = RMSNorm(x) * norm_w
    when norm_w is given (sumsq_in: [M, K/32] fp32 row sum-of-squares partials of x)."""
    if isinstance(w, torch.Tensor):  # convenience for tests: pack on the fly
        w = PackedWeight(w)
    _need_cuda(x, residual, out, out2, argmax_partials, norm_w, sumsq_in, sumsq_out)
    if x.dtype != torch.bfloat16:
        raise ValueError("gemm takes bf16 x")
    M, K = x.shape
    N, K2 = w.shape
    if K != K2:
        raise ValueError(f"gemm shape mismatch x{tuple(x.shape)} w{tuple(w.shape)}")
    ldx = _row_stride(x)
    ws = ws or workspace(x.device)
    if ws.wide:
        fn = "dfl_gemm_bf16_wide"
        ks = wide_split(N, K, ws)
        ws.ensure_wide(int(_lib.query("dfl_gemm_wide_workspace_bytes", M, N, K, int(norm_w is not None), ks)))
        scratch, tail = ws.wide_x, (ks,)
    else:
        fn = "dfl_gemm_bf16"
        ws.ensure_gemm(int(_lib.query("dfl_gemm_workspace_bytes", M, N, K, epilogue)))
        scratch, tail = ws.gemm, ()
    n_parts = 0
    if norm_w is not None:
        if sumsq_in is None or sumsq_in.shape[0] < M or sumsq_in.dtype != torch.float32:
            raise ValueError("the fused RMSNorm needs fp32 sumsq_in partials [M, K/32]")
        n_parts = sumsq_in.shape[1]
        if n_parts != K // 32 or not sumsq_in.is_contiguous():
            raise ValueError("sumsq_in must be contiguous [M, K/32]")
    if sumsq_out is not None and (sumsq_out.shape[1] != N // 32 or not sumsq_out.is_contiguous()):
        raise ValueError("sumsq_out must be contiguous [M, N/32]")
    if epilogue == EPI_ARGMAX:
        ntiles = int(_lib.query("dfl_gemm_argmax_tiles", N))
        if argmax_partials is None:
            argmax_partials = torch.empty((M, ntiles, 2), dtype=torch.float32, device=x.device)
        _lib.call(fn, _ptr(x), ldx, _ptr(w), M, N, K, epilogue, None, 0, None, 0, None, 0,
                  _ptr(argmax_partials), _ptr(norm_w), _ptr(sumsq_in), n_parts, float(eps), None, *tail,
                  _ptr(scratch), scratch.numel(), _stream())
        return argmax_partials
    n_out = N // 2 if epilogue == EPI_SILU_MUL else N
    out_dtype = torch.float32 if epilogue in (EPI_STORE_F32, EPI_PARTIALS) else torch.bfloat16
    if epilogue == EPI_PARTIALS:
        if not ws.wide:
            raise ValueError("the partials epilogue is a wide-GEMM form")
        if out is None:
            out = torch.empty((tail[0], M, N), dtype=out_dtype, device=x.device)
        if out.dim() != 3 or out.shape[0] < tail[0] or out.stride(1) != N:
            raise ValueError(f"the partials epilogue writes [{tail[0]}, M, {N}] slabs")
    if out is None:
        out = torch.empty((M, n_out), dtype=out_dtype, device=x.device)
    if out.dtype != out_dtype:
        raise ValueError(f"epilogue {epilogue} writes {out_dtype}")
    if residual is not None and epilogue != EPI_RESIDUAL:
        raise ValueError("residual given without the residual epilogue")
    ldr = _row_stride(residual) if residual is not None else 0
    ldy2 = _row_stride(out2) if out2 is not None else 0
    ldy = N if epilogue == EPI_PARTIALS else _row_stride(out)
    _lib.call(fn, _ptr(x), ldx, _ptr(w), M, N, K, epilogue, _ptr(residual), ldr, _ptr(out),
              ldy, _ptr(out2), ldy2, None, _ptr(norm_w), _ptr(sumsq_in), n_parts, float(eps),
              _ptr(sumsq_out), *tail, _ptr(scratch), scratch.numel(), _stream())
    return out


class GemmOp(ctypes.Structure):
    """dfl_gemm_op: the arguments of one dfl_gemm_bf16 call inside a dfl_gemm_chain."""
    _fields_ = [("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("w_packed", ctypes.c_void_p),
                ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int), ("epilogue", ctypes.c_int),
                ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("ldy", ctypes.c_int64), ("y2", ctypes.c_void_p), ("ldy2", ctypes.c_int64),
                ("argmax_partials", ctypes.c_void_p), ("norm_w", ctypes.c_void_p), ("sumsq_in", ctypes.c_void_p),
                ("n_parts", ctypes.c_int), ("eps", ctypes.c_float), ("sumsq_out", ctypes.c_void_p)]


CHAIN_MAX_ROWS = 16
CHAIN_MAX_OPS = 6


def chain_op(x: torch.Tensor, w: PackedWeight, epilogue: int = EPI_STORE, residual: torch.Tensor | None = None,
             out: torch.Tensor | None = None, out2: torch.Tensor | None = None,
             argmax_partials: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
             sumsq_in: torch.Tensor | None = None, eps: float = 1e-6,
             sumsq_out: torch.Tensor | None = None) -> GemmOp:
    """One op of a GEMM chain (the arguments of ``gemm`` without running it)."""
    _need_cuda(x, residual, out, out2, argmax_partials, norm_w, sumsq_in, sumsq_out)
    M, K = x.shape
    if M > CHAIN_MAX_ROWS:
        raise ValueError("a GEMM chain takes at most 16 rows")
    n_parts = sumsq_in.shape[1] if (norm_w is not None and sumsq_in is not None) else 0
    return GemmOp(_ptr(x), _row_stride(x), w.data_ptr(), M, w.N, K, epilogue, _ptr(residual),
                  _row_stride(residual) if residual is not None else 0, _ptr(out),
                  _row_stride(out) if out is not None else 0, _ptr(out2), _row_stride(out2) if out2 is not None else 0,
                  _ptr(argmax_partials), _ptr(norm_w), _ptr(sumsq_in), n_parts, float(eps), _ptr(sumsq_out))


def gemm_chain(op_list: list[GemmOp], ws: Workspace | None = None) -> None:
    """Runs up to six decode-block GEMMs (M <= 16), each reading the previous one's output,
    as one persistent launch (dfl_gemm_chain)."""
    if not op_list:
        return
    if len(op_list) > CHAIN_MAX_OPS:
        raise ValueError(f"a GEMM chain holds at most {CHAIN_MAX_OPS} ops")
    ws = ws or workspace()
    arr = (GemmOp * len(op_list))(*op_list)
    need = int(_lib.query("dfl_gemm_chain_workspace_bytes", arr, len(op_list)))
    if need > ws.chain.numel():
        raise ValueError(f"GEMM chain scratch too small ({ws.chain.numel()} < {need})")
    _lib.call("dfl_gemm_chain", arr, len(op_list), _ptr(ws.chain), ws.chain.numel(), _stream())


_SMS: dict[int, int] = {}


def wide_split(N: int, K: int, ws: Workspace) -> int:
    """K ranges of a wide GEMM: enough (128-row tile x range) items for every SM when the
    weight has few 128-row tiles, at most ws.wide_split. Depends on N, K and the
    workspace's limit only, so every call of a session splits a weight the same way."""
    if ws.wide_split <= 1:
        return 1
    dev = ws.device.index if ws.device.index is not None else torch.cuda.current_device()
    if dev not in _SMS:
        _SMS[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    n_tiles = (N + 127) // 128
    return max(1, min(ws.wide_split, round(_SMS[dev] / n_tiles), K // 64))


def device_error(clear: bool = True) -> int:
    """Non-zero when a kernel's bounded wait gave up (synchronises the current stream)."""
    import ctypes
    code = ctypes.c_int(0)
    _lib.call("dfl_device_error", ctypes.byref(code), int(clear), _stream())
    return code.value


def argmax_tiles(N: int) -> int:
    return int(_lib.query("dfl_gemm_argmax_tiles", N))


def rmsnorm(x: torch.Tensor, w: torch.Tensor | None, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(x, w, out)
    M, H = x.shape
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    _lib.call("dfl_rmsnorm_bf16", _ptr(x), _row_stride(x), _ptr(w), _ptr(out), _row_stride(out), M, H, float(eps),
              _stream())
    return out


def embed(tokens: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None,
          sumsq_out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(tokens, table, out, sumsq_out)
    if tokens.dtype != torch.int32 or not tokens.is_contiguous():
        raise ValueError("tokens must be contiguous int32")
    V, H = table.shape
    M = tokens.numel()
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=table.device)
    _lib.call("dfl_embed_bf16", _ptr(tokens), _ptr(table), _ptr(out), _row_stride(out), M, H, V, _ptr(sumsq_out),
              _stream())
    return out


def qkv_rope_append(qkv: torch.Tensor, pos: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                    inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, Hq: int, Hkv: int, hd: int,
                    rot_dim: int, eps: float, q_out: torch.Tensor | None = None, row_seq: torch.Tensor | None = None,
                    q_stride: int | None = None, do_q: bool = True, page_table: torch.Tensor | None = None,
                    page_size: int = 0) -> torch.Tensor | None:
    """q/k head norm + RoPE + cache append. Caches are [seq, Hkv, cap, hd] views (contiguous in the last 3 dims),
    or, with ``page_table`` [seq, pages] int32, page pools [n_pages, Hkv, page_size, hd]."""
    _need_cuda(qkv, pos, q_norm, k_norm, inv_freq, k_cache, v_cache, q_out, row_seq, page_table)
    M = qkv.shape[0]
    if do_q and q_out is None:
        q_out = torch.empty((M, Hq, hd), dtype=torch.bfloat16, device=qkv.device)
    if k_cache.dim() != 4 or k_cache.stride(3) != 1 or k_cache.stride(2) != hd:
        raise ValueError("k_cache must be a [seq, Hkv, cap, hd] view")
    if page_table is not None:
        _lib.call("dfl_qkv_rope_append_paged", _ptr(qkv), _row_stride(qkv), q_stride or hd, _ptr(pos),
                  _ptr(row_seq), _ptr(q_norm), _ptr(k_norm), _ptr(inv_freq), _ptr(q_out) if do_q else None,
                  _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), _ptr(page_table),
                  page_table.stride(0), int(page_size), M, Hq, Hkv, hd, rot_dim, float(eps), int(do_q), _stream())
        return q_out
    _lib.call("dfl_qkv_rope_append", _ptr(qkv), _row_stride(qkv), q_stride or hd, _ptr(pos), _ptr(row_seq),
              _ptr(q_norm), _ptr(k_norm), _ptr(inv_freq), _ptr(q_out) if do_q else None, _ptr(k_cache),
              _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), M, Hq, Hkv, hd, rot_dim, float(eps), int(do_q),
              _stream())
    return q_out


def gemm_qkv_rope(x: torch.Tensor, w: PackedWeight | torch.Tensor, qkv: torch.Tensor, pos: torch.Tensor, q_norm: torch.Tensor,
                  k_norm: torch.Tensor, inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  q_out: torch.Tensor, Hq: int, Hkv: int, hd: int, eps: float, norm_w: torch.Tensor | None = None,
                  sumsq_in: torch.Tensor | None = None, row_seq: torch.Tensor | None = None,
                  ws: Workspace | None = None, page_table: torch.Tensor | None = None, page_size: int = 0) -> None:
    """The QKV projection (input RMSNorm fused when norm_w is given) into ``qkv``, then the
    q/k head norm + RoPE (full rotary) + cache append of qkv_rope_append, as one call
    (dfl_gemm_qkv_rope): the same bits as gemm() followed by qkv_rope_append()."""
    if isinstance(w, torch.Tensor):  # convenience for tests: pack on the fly
        w = PackedWeight(w)
    _need_cuda(x, qkv, pos, q_norm, k_norm, inv_freq, k_cache, v_cache, q_out, norm_w, sumsq_in, row_seq, page_table)
    M, K = x.shape
    N = (Hq + 2 * Hkv) * hd
    if tuple(w.shape) != (N, K) or qkv.shape[0] < M or qkv.shape[1] < N:
        raise ValueError(f"gemm_qkv_rope shape mismatch x{tuple(x.shape)} w{tuple(w.shape)} qkv{tuple(qkv.shape)}")
    if k_cache.dim() != 4 or k_cache.stride(3) != 1 or k_cache.stride(2) != hd:
        raise ValueError("k_cache must be a [seq, Hkv, cap, hd] view (or a page pool)")
    ws = ws or workspace(x.device)
    if ws.wide:
        raise ValueError("gemm_qkv_rope runs the M <= 16 weight-streaming forms only")
    ws.ensure_gemm(int(_lib.query("dfl_gemm_workspace_bytes", M, N, K, EPI_STORE)))
    n_parts = 0
    if norm_w is not None:
        if sumsq_in is None or sumsq_in.dtype != torch.float32 or not sumsq_in.is_contiguous():
            raise ValueError("the fused RMSNorm needs contiguous fp32 sumsq_in partials [M, K/32]")
        n_parts = sumsq_in.shape[1]
    _lib.call("dfl_gemm_qkv_rope", _ptr(x), _row_stride(x), _ptr(w), M, K, _ptr(norm_w), _ptr(sumsq_in), n_parts,
              float(eps), _ptr(qkv), _row_stride(qkv), _ptr(pos), _ptr(row_seq), _ptr(q_norm), _ptr(k_norm),
              _ptr(inv_freq), _ptr(q_out), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1),
              _ptr(page_table), page_table.stride(0) if page_table is not None else 0, int(page_size), Hq, Hkv, hd,
              _ptr(ws.gemm), ws.gemm.numel(), _stream())


def gemm_kv_append_layers(x: torch.Tensor, w: PackedWeight | torch.Tensor, kv: torch.Tensor, pos: torch.Tensor,
                          k_norms: list[torch.Tensor], inv_freq: torch.Tensor, k_cache: torch.Tensor,
                          v_cache: torch.Tensor, Hkv: int, hd: int, eps: float, norm_w: torch.Tensor | None = None,
                          sumsq_in: torch.Tensor | None = None, row_seq: torch.Tensor | None = None,
                          ws: Workspace | None = None, page_table: torch.Tensor | None = None,
                          page_size: int = 0) -> None:
    """The stacked K/V projection of every layer's context rows (input RMSNorm fused when
    norm_w is given) into ``kv``, then each layer's k_norm + RoPE + append into
    k_cache[l] / v_cache[l] (caches [L, ...], one layer per leading index), as one call
    (dfl_gemm_kv_append_layers): the same bits as gemm() and a qkv_rope_append() per layer."""
    if isinstance(w, torch.Tensor):  # convenience for tests: pack on the fly
        w = PackedWeight(w)
    _need_cuda(x, kv, pos, inv_freq, k_cache, v_cache, norm_w, sumsq_in, row_seq, page_table, *k_norms)
    M, K = x.shape
    L = len(k_norms)
    N = L * 2 * Hkv * hd
    if tuple(w.shape) != (N, K) or kv.shape[0] < M or kv.shape[1] < N or k_cache.shape[0] < L:
        raise ValueError(f"gemm_kv_append_layers shape mismatch x{tuple(x.shape)} w{tuple(w.shape)} kv{tuple(kv.shape)}")
    if k_cache.dim() != 5 or k_cache.stride(4) != 1 or k_cache.stride(3) != hd or k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache / v_cache must be [L, seq, Hkv, cap, hd] (or [L, pages, Hkv, page_size, hd]) alike")
    ws = ws or workspace(x.device)
    if ws.wide:
        raise ValueError("gemm_kv_append_layers runs the M <= 16 weight-streaming forms only")
    ws.ensure_gemm(int(_lib.query("dfl_gemm_workspace_bytes", M, N, K, EPI_STORE)))
    n_parts = 0
    if norm_w is not None:
        if sumsq_in is None or sumsq_in.dtype != torch.float32 or not sumsq_in.is_contiguous():
            raise ValueError("the fused RMSNorm needs contiguous fp32 sumsq_in partials [M, K/32]")
        n_parts = sumsq_in.shape[1]
    norms = (ctypes.c_void_p * L)(*[t.data_ptr() for t in k_norms])
    _lib.call("dfl_gemm_kv_append_layers", _ptr(x), _row_stride(x), _ptr(w), M, K, _ptr(norm_w), _ptr(sumsq_in),
              n_parts, float(eps), _ptr(kv), _row_stride(kv), _ptr(pos), _ptr(row_seq), norms, _ptr(inv_freq),
              _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
              _ptr(page_table), page_table.stride(0) if page_table is not None else 0, int(page_size), L, Hkv, hd,
              _ptr(ws.gemm), ws.gemm.numel(), _stream())


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor, causal: bool,
              max_kv: int, kv_len: torch.Tensor | None = None, row_seq: torch.Tensor | None = None,
              scale: float | None = None, out: torch.Tensor | None = None, ws: Workspace | None = None,
              gate: torch.Tensor | None = None, gate_head_stride: int = 0, seq_rows: int = 0,
              key_chunk: int = 0, page_table: torch.Tensor | None = None, page_size: int = 0) -> torch.Tensor:
    """q [M, Hq, hd] against caches [seq, Hkv, cap, hd]; returns [M, Hq*hd] bf16.
    seq_rows: rows per sequence when row_seq groups contiguous runs (0 = any layout).
    key_chunk: keys per split (0 = the library default); results depend on it."""
    _need_cuda(q, k_cache, v_cache, pos, kv_len, row_seq, out)
    M, Hq, hd = q.shape
    Hkv = k_cache.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((M, Hq * hd), dtype=torch.bfloat16, device=q.device)
    ws = ws or workspace(q.device)
    need = int(_lib.query("dfl_attention_workspace_bytes", M, Hq, hd, max_kv, int(key_chunk)))
    ws.ensure_attn(need)
    if page_table is not None:
        _need_cuda(page_table)
        _lib.call("dfl_attention_paged", _ptr(q), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1),
                  _ptr(page_table), page_table.stride(0), int(page_size), _ptr(pos), _ptr(row_seq), _ptr(kv_len),
                  int(seq_rows), M, Hq, Hkv, hd, int(causal), float(scale), int(max_kv), int(key_chunk), _ptr(out),
                  _row_stride(out), _ptr(gate), _row_stride(gate) if gate is not None else 0, int(gate_head_stride),
                  _ptr(ws.attn), ws.attn.numel(), _stream())
        return out
    _lib.call("dfl_attention", _ptr(q), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1),
              _ptr(pos), _ptr(row_seq), _ptr(kv_len), int(seq_rows), M, Hq, Hkv, hd, int(causal), float(scale),
              int(max_kv), int(key_chunk),
              _ptr(out), _row_stride(out), _ptr(gate), _row_stride(gate) if gate is not None else 0,
              int(gate_head_stride), _ptr(ws.attn), ws.attn.numel(), _stream())
    return out


def fused_attention_ok(M: int, row_seq, seq_rows: int, hd: int, rot_dim: int) -> bool:
    """Whether attention_qkv applies: head_dim 128 with full rotary and every sequence's
    rows inside one 16-row tile."""
    if hd != 128 or rot_dim != 128:
        return False
    if row_seq is None:
        return M <= 16
    return 0 < seq_rows <= 16 and 16 % seq_rows == 0


def attention_qkv(qkv: torch.Tensor, pos: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                  inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, Hq: int, eps: float,
                  max_kv: int, row_seq: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  ws: Workspace | None = None, seq_rows: int = 0, key_chunk: int = 0,
                  scale: float | None = None) -> torch.Tensor:
    """qkv_rope_append + causal attention in one launch (head_dim 128, full rotary; every
    sequence's rows in one 16-row tile); the same bits as the two calls."""
    _need_cuda(qkv, pos, q_norm, k_norm, inv_freq, k_cache, v_cache, row_seq, out)
    M = qkv.shape[0]
    Hkv = k_cache.shape[1]
    if k_cache.dim() != 4 or k_cache.stride(3) != 1 or k_cache.stride(2) != 128:
        raise ValueError("k_cache must be a [seq, Hkv, cap, 128] view")
    if out is None:
        out = torch.empty((M, Hq * 128), dtype=torch.bfloat16, device=qkv.device)
    ws = ws or workspace(qkv.device)
    need = int(_lib.query("dfl_attention_workspace_bytes", M, Hq, 128, max_kv, int(key_chunk)))
    ws.ensure_attn(need)
    _lib.call("dfl_attention_qkv", _ptr(qkv), _row_stride(qkv), _ptr(q_norm), _ptr(k_norm), _ptr(inv_freq),
              float(eps), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), _ptr(pos),
              _ptr(row_seq), int(seq_rows), M, Hq, Hkv, float(scale if scale is not None else 1.0 / math.sqrt(128)),
              int(max_kv), int(key_chunk), _ptr(out), _row_stride(out), _ptr(ws.attn), ws.attn.numel(), _stream())
    return out


def argmax_reduce(partials: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(partials, out)
    M, ntiles = partials.shape[0], partials.shape[1]
    if out is None:
        out = torch.empty(M, dtype=torch.int32, device=partials.device)
    _lib.call("dfl_argmax_reduce", _ptr(partials), M, ntiles, _ptr(out), _stream())
    return out


def step_prepare(state, out_tokens, block, bs, mask_id, target_pos, draft_ctx_pos, draft_block_pos, draft_kv_len, B):
    _lib.call("dfl_step_prepare", _ptr(state), _ptr(out_tokens), out_tokens.stride(0), _ptr(block), bs, mask_id,
              _ptr(target_pos), _ptr(draft_ctx_pos), _ptr(draft_block_pos), _ptr(draft_kv_len), B, _stream())


_M64 = (1 << 64) - 1
SAMPLE_TAG_DRAFT, SAMPLE_TAG_TARGET = 1, 2


def mix64(z: int) -> int:
    """Host copy of the device splitmix64 finaliser (common.cuh)."""
    z = (z + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def sample_key(seed: int, tag: int, b: int, pos: int) -> int:
    """The key dfl_sample_keys gives sequence b's row predicting absolute position pos."""
    return mix64(mix64(mix64((seed ^ tag) & _M64) ^ b) ^ pos)


def _as_i64(k: int) -> int:
    return k - (1 << 64) if k >= 1 << 63 else k


def sample_keys(state, B, bs, seed, tag, offset, keys):
    """keys[b * bs + i] for the rows of a step (uint64 bits in an int64 tensor)."""
    _lib.call("dfl_sample_keys", _ptr(state), B, bs, ctypes.c_uint64(seed & _M64), tag, offset, _ptr(keys),
              _stream())


def keys_tensor(keys: list[int], device) -> torch.Tensor:
    return torch.tensor([_as_i64(k) for k in keys], dtype=torch.int64, device=device)


def sample_partials(logits: torch.Tensor, keys: torch.Tensor, temperature: float,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Gumbel-max partials of bf16 logits [M, V] at temperature (argmax_reduce gives the sample)."""
    _need_cuda(logits, keys, out)
    M, V = logits.shape
    if out is None:
        out = torch.empty((M, argmax_tiles(V), 2), dtype=torch.float32, device=logits.device)
    _lib.call("dfl_sample_partials", _ptr(logits), _row_stride(logits), M, V, _ptr(keys), float(1.0 / temperature),
              _ptr(out), _stream())
    return out


def draft_commit(state, partials, block, bs, B, inject_tokens=None, inject_len=None, inject_noise=None):
    _lib.call("dfl_draft_commit", _ptr(state), _ptr(partials), partials.shape[1], _ptr(block), bs,
              _ptr(inject_tokens), inject_tokens.stride(0) if inject_tokens is not None else 0, _ptr(inject_len),
              inject_len.stride(0) if inject_len is not None else 0, _ptr(inject_noise),
              inject_noise.stride(0) if inject_noise is not None else 0, B, _stream())


def verify_accept(state, partials, block, bs, out_tokens, B, stop_ids=None, n_stop=0, posterior=None,
                  accept_log=None):
    _lib.call("dfl_verify_accept", _ptr(state), _ptr(partials), partials.shape[1], _ptr(block), bs, _ptr(out_tokens),
              out_tokens.stride(0), _ptr(posterior), _ptr(stop_ids), n_stop, _ptr(accept_log),
              accept_log.stride(0) if accept_log is not None else 0, B, _stream())


def gdr_recurrence(q, k, v, g, beta, state_in, state_out=None, snapshots=None, o=None, state_slot=None,
                   state_in_bstride=None, tokens=None, tokens_stride: int = 1):
    """Gated-delta recurrence. q,k [B,T,Hk,Dk] bf16; v [B,T,Hv,Dv] bf16; g,beta [B,T,Hv] fp32;
    state_in [B,Hv,Dv,Dk] fp32 (or a snapshot array with state_slot). tokens (device
    int32, element b * tokens_stride): sequence b advances over that many tokens only."""
    _need_cuda(q, k, v, g, beta, state_in, state_out, snapshots, o, state_slot, tokens)
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2], v.shape[3]
    for t in (k, v, g, beta, state_in):
        if not t.is_contiguous():
            raise ValueError("gdr_recurrence inputs must be contiguous")
    if g.dtype != torch.float32 or beta.dtype != torch.float32 or state_in.dtype != torch.float32:
        raise ValueError("g, beta and the state are fp32")
    bstride = state_in_bstride if state_in_bstride is not None else Hv * Dv * Dk
    _lib.call("dfl_gdr_recurrence", _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(state_in), bstride,
              _ptr(state_slot), _ptr(state_out), _ptr(snapshots), _ptr(o), B, T, Hk, Hv, Dk, Dv, _ptr(tokens),
              int(tokens_stride), _stream())


def gdn_prep(proj: torch.Tensor, conv_w: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
             conv_state: torch.Tensor, B: int, T: int, Hk: int, Hv: int, Dk: int, Dv: int,
             window: torch.Tensor | None = None, eps: float = 1e-6, out: dict | None = None) -> dict:
    """Conv + SiLU + q/k scaling + g/beta for B sequences of T rows (proj rows are [qkv | z | b | a])."""
    _need_cuda(proj, conv_w, A_log, dt_bias, conv_state, window)
    dev = proj.device
    M = B * T
    o = out or {}
    q = o.get("q") if o.get("q") is not None else torch.empty((M, Hk, Dk), dtype=torch.bfloat16, device=dev)
    k = o.get("k") if o.get("k") is not None else torch.empty((M, Hk, Dk), dtype=torch.bfloat16, device=dev)
    v = o.get("v") if o.get("v") is not None else torch.empty((M, Hv, Dv), dtype=torch.bfloat16, device=dev)
    g = o.get("g") if o.get("g") is not None else torch.empty((M, Hv), dtype=torch.float32, device=dev)
    beta = o.get("beta") if o.get("beta") is not None else torch.empty((M, Hv), dtype=torch.float32, device=dev)
    _lib.call("dfl_gdn_prep", _ptr(proj), _row_stride(proj), _ptr(conv_w), _ptr(A_log), _ptr(dt_bias),
              _ptr(conv_state), _ptr(window), window.stride(0) if window is not None else 0, _ptr(q), _ptr(k),
              _ptr(v), _ptr(g), _ptr(beta), B, T, Hk, Hv, Dk, Dv, float(eps), _stream())
    return {"q": q, "k": k, "v": v, "g": g, "beta": beta}


def gdn_rollback(state, snapshots, conv_state, window, accepted, acc_stride, B, T, Hv, Dv, Dk, C):
    """state <- snapshots[accepted-1]; conv_state <- window rows [accepted, accepted+3) (device-side accepted)."""
    _lib.call("dfl_gdn_rollback", _ptr(state), _ptr(snapshots), _ptr(conv_state), _ptr(window),
              window.stride(0) if window is not None else 0, _ptr(accepted), acc_stride, B, T, Hv, Dv, Dk, C,
              _stream())


def gated_rmsnorm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, H: int, D: int, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(o, z, w, out)
    M = o.shape[0]
    if out is None:
        out = torch.empty((M, H * D), dtype=torch.bfloat16, device=o.device)
    _lib.call("dfl_gated_rmsnorm", _ptr(o), _row_stride(o), _ptr(z), _row_stride(z), _ptr(w), _ptr(out),
              _row_stride(out), M, H, D, float(eps), _stream())
    return out
