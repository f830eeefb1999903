"""GPU Qwen3 target and DFlash draft built from the C-ABI kernels.

HBM layout (per device):
  * target layer l: ``w_qkv`` [(Hq+2Hkv)*hd, H] (q, k, v projections stacked),
    ``w_o`` [H, Hq*hd], ``w_gu`` [2F, H] (gate/up packed per 64 rows as
    [32 gate | 32 up] for the fused SiLU*up epilogue), ``w_down`` [H, F];
  * KV cache: one tensor per K and V of shape [L, B, Hkv, cap, hd] bf16; the
    token at position p of sequence b lives in slot p (rollback = length update);
  * draft: per layer ``w_qkv``/``w_o``/``w_gu``/``w_down`` as above plus one
    ``w_ctx_kv`` [n_layers*2*Hkv*hd, H] stacking every layer's k/v projection so
    that the context rows (fc + hidden_norm of the target taps, the same input
    for every draft layer: draft.py:217-222) are projected for all layers with
    one weight stream.

Forward semantics follow the reference: the target forward with hidden-state
taps (adapters.py:611-631, mlx-lm qwen3 layers) and the DFlash draft
(draft.py:109-223).
"""
from __future__ import annotations

import os

from dataclasses import dataclass

import torch

from . import ops
from .config import DraftConfig, TargetConfig
from .weights import pack_gate_up, rope_inv_freq


@dataclass
class KVCache:
    """K/V of every layer, either contiguous slots [L, B, Hkv, cap, hd] bf16 (the token at
    position p of sequence b in slot p) or, with a page table, page pools
    [L, n_pages, Hkv, page_size, hd] and ``page_table`` [B, pages] int32 (position p of
    sequence b in page page_table[b, p // page_size], row p % page_size), so that each
    sequence holds pages for its own length only."""

    k: torch.Tensor
    v: torch.Tensor
    page_table: torch.Tensor | None = None
    page_size: int = 0
    cap_tokens: int = 0

    @property
    def cap(self) -> int:
        return self.cap_tokens if self.page_table is not None else self.k.shape[3]

    def layer(self, l: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[l], self.v[l]

    @property
    def paging(self) -> dict:
        """Keyword arguments of ops.qkv_rope_append / ops.attention for this cache."""
        if self.page_table is None:
            return {}
        return {"page_table": self.page_table, "page_size": self.page_size}

    def gather(self, l: int, b: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Keys and values of positions [0, n) of sequence b in layer l, as [Hkv, n, hd]."""
        if self.page_table is None:
            return self.k[l, b, :, :n], self.v[l, b, :, :n]
        ps = self.page_size
        pages = self.page_table[b, :(n + ps - 1) // ps].long()
        k = self.k[l, pages].permute(1, 0, 2, 3).reshape(self.k.shape[2], -1, self.k.shape[4])[:, :n]
        v = self.v[l, pages].permute(1, 0, 2, 3).reshape(self.v.shape[2], -1, self.v.shape[4])[:, :n]
        return k, v


def alloc_kv(n_layers: int, batch: int, n_kv: int, cap: int, hd: int, device) -> KVCache:
    shape = (n_layers, batch, n_kv, cap, hd)
    return KVCache(torch.zeros(shape, dtype=torch.bfloat16, device=device),
                   torch.zeros(shape, dtype=torch.bfloat16, device=device))


PAGE_SIZE = 64


def gemm_chain_enabled() -> bool:
    """GEMM chains are opt-in (DFLASH_B200_GEMM_CHAIN=1): on B200 the chained verify pass
    measured slower than one launch per projection (4.47 against 2.47 ms per Qwen3-4B
    verify pass): a split tile is finished by one last-arriving CTA that reads up to 15
    partial tiles two at a time, and each op then waits for all of them."""
    return os.environ.get("DFLASH_B200_GEMM_CHAIN", "0") == "1"


def qkv_rope_ok(ws, hd: int, rot_dim: int) -> bool:
    """Whether a decoder layer's QKV projection takes the fused q/k norm + RoPE + append
    call (ops.gemm_qkv_rope: the same bits as the separate calls): full rotary, the M <= 16
    GEMM forms (not a wide workspace), unless DFLASH_B200_FUSED_QKV_ROPE=0."""
    if os.environ.get("DFLASH_B200_FUSED_QKV_ROPE", "1") == "0":
        return False
    return rot_dim == hd and not (ws is not None and ws.wide)


def chain_ok(M: int, ws) -> bool:
    """Whether a forward over M rows uses GEMM chains: decode blocks of the one-sequence
    (weight-streaming) kernel forms; decided by M and the session's kernel forms only."""
    return M <= ops.CHAIN_MAX_ROWS and not (ws if ws is not None else ops.workspace()).wide


def page_plan(lengths: list[int], page_size: int = PAGE_SIZE) -> tuple[torch.Tensor, int]:
    """Page table for sequences that each need ``lengths[b]`` positions: sequence b gets
    consecutive pages; table entries past a sequence's need point at one spare page (the
    last), which no kernel reads. Returns (table [B, max pages] int32 on the host, n_pages)."""
    need = [(n + page_size - 1) // page_size for n in lengths]
    width = max(need) if need else 1
    total = sum(need)
    table = torch.full((len(lengths), width), total, dtype=torch.int32)
    base = 0
    for b, n in enumerate(need):
        table[b, :n] = torch.arange(base, base + n, dtype=torch.int32)
        base += n
    return table, total + 1


def alloc_kv_paged(n_layers: int, lengths: list[int], n_kv: int, hd: int, device,
                   page_table: torch.Tensor | None = None, page_size: int = PAGE_SIZE) -> KVCache:
    """Paged K/V for sequences of the given lengths (one shared page table may serve
    several caches: pass the device table of a previous call)."""
    table, n_pages = page_plan(lengths, page_size)
    if page_table is None:
        page_table = table.to(device)
    shape = (n_layers, n_pages, n_kv, page_size, hd)
    return KVCache(torch.zeros(shape, dtype=torch.bfloat16, device=device),
                   torch.zeros(shape, dtype=torch.bfloat16, device=device), page_table, page_size,
                   max(lengths) if lengths else 0)


class TargetModel:
    """Qwen3-family target: block forward with taps, KV append, fused lm_head argmax."""

    def __init__(self, cfg: TargetConfig, weights: dict, device="cuda"):
        if cfg.model_type != "qwen3":
            raise NotImplementedError("TargetModel runs the dense qwen3 family; the hybrid lives in hybrid.py")
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        P = ops.pack_weight
        self.embed_w = weights["embed"].to(dev).contiguous()  # row-major: the embedding gather
        self.lm_head_w = P(self.embed_w if cfg.tie_word_embeddings else weights["lm_head"].to(dev))
        self.norm_w = weights["norm"].to(dev)
        self.layers = []
        for lw in weights["layers"]:
            self.layers.append({
                "in_norm": lw["input_layernorm"].to(dev),
                "post_norm": lw["post_attention_layernorm"].to(dev),
                "w_qkv": P(torch.cat([lw["q_proj"].to(dev), lw["k_proj"].to(dev), lw["v_proj"].to(dev)], 0)),
                "w_o": P(lw["o_proj"].to(dev)),
                "w_gu": P(pack_gate_up(lw["gate_proj"].to(dev), lw["up_proj"].to(dev))),
                "w_down": P(lw["down_proj"].to(dev)),
                "q_norm": lw["q_norm"].to(dev),
                "k_norm": lw["k_norm"].to(dev),
            })
        self.inv_freq = rope_inv_freq(cfg.rope_dim, cfg.rope_theta, dev)
        # True (or DFLASH_B200_FUSED_ATTENTION=1): verify blocks whose sequences each sit in
        # one 16-row tile append K/V inside the attention launch (dfl_attention_qkv, the same
        # bits). Off by default: measured 3287 against 3217 us per Qwen3-4B verify step, the
        # in-CTA q/k preparation costing more than the append launch it removes.
        self.fuse_attention = os.environ.get("DFLASH_B200_FUSED_ATTENTION", "0") == "1"
        # decode blocks (M <= 16, one-sequence kernel forms) may run the projections between two
        # attention calls as one GEMM-chain launch (opt-in, see gemm_chain_enabled)
        self.use_chain = gemm_chain_enabled()
        self._bufs: dict[int, dict[str, torch.Tensor]] = {}

    # ------------------------------------------------------------------
    def make_cache(self, batch: int, cap: int, block: int = 16, lengths: list[int] | None = None,
                   page_table: torch.Tensor | None = None) -> KVCache:
        """Contiguous [L, batch, Hkv, cap, hd] slots, or, given each sequence's length,
        a paged cache holding pages for those lengths only."""
        c = self.cfg
        if lengths is not None:
            return alloc_kv_paged(c.num_hidden_layers, lengths, c.num_key_value_heads, c.head_dim, self.device,
                                  page_table)
        return alloc_kv(c.num_hidden_layers, batch, c.num_key_value_heads, cap, c.head_dim, self.device)

    def buffers(self, M: int) -> dict[str, torch.Tensor]:
        b = self._bufs.get(M)
        if b is None:
            c = self.cfg
            dev = self.device
            H, hd = c.hidden_size, c.head_dim
            b = {
                "h": torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                "xn": torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                "qkv": torch.empty((M, (c.num_attention_heads + 2 * c.num_key_value_heads) * hd), dtype=torch.bfloat16,
                                   device=dev),
                "q": torch.empty((M, c.num_attention_heads, hd), dtype=torch.bfloat16, device=dev),
                "attn": torch.empty((M, c.num_attention_heads * hd), dtype=torch.bfloat16, device=dev),
                "act": torch.empty((M, c.intermediate_size), dtype=torch.bfloat16, device=dev),
                "argmax": torch.empty((M, ops.argmax_tiles(c.vocab_size), 2), dtype=torch.float32, device=dev),
                "ss": torch.zeros((M, H // 32), dtype=torch.float32, device=dev),
            }
            self._bufs[M] = b
        return b

    def forward(self, tokens: torch.Tensor, pos: torch.Tensor, cache: KVCache, max_kv: int,
                layer_ids: list[int] | None = None, taps_out: torch.Tensor | None = None,
                row_seq: torch.Tensor | None = None, head: str = "argmax", ws: ops.Workspace | None = None,
                seq_rows: int = 0, key_chunk: int = 0):
        """Block forward over M rows (tokens int32 [M] at positions pos [M]).

        Appends K/V at each row's position, writes the residual stream after each
        layer in ``layer_ids`` into ``taps_out[:, i*H:(i+1)*H]`` (ascending layer
        order, adapters.py:624-630) and returns, by ``head``:
          "argmax": DFL_EPI_ARGMAX partials of the lm_head (fused, no logits in HBM)
          "logits": bf16 logits [M, V]
          "hidden": the final-normed hidden states [M, H]
        """
        c = self.cfg
        M = tokens.numel()
        b = self.buffers(M)
        H, hd = c.hidden_size, c.head_dim
        Hq, Hkv = c.num_attention_heads, c.num_key_value_heads
        tap_col = {}
        if layer_ids:
            for i, lid in enumerate(sorted(layer_ids)):
                tap_col[lid] = i
        h, ss = b["h"], b["ss"]
        eps = c.rms_norm_eps
        ops.embed(tokens, self.embed_w, out=h, sumsq_out=ss)
        fused = (self.fuse_attention and cache.page_table is None
                 and ops.fused_attention_ok(M, row_seq, seq_rows, hd, c.rope_dim))
        pg = cache.paging
        if self.use_chain and chain_ok(M, ws):
            return self._forward_chain(pos, cache, max_kv, tap_col, taps_out, row_seq, head, ws, seq_rows, key_chunk,
                                       fused, b)
        qkv_rope = not fused and qkv_rope_ok(ws, hd, c.rope_dim)
        for l, lw in enumerate(self.layers):
            kc, vc = cache.layer(l)
            if qkv_rope:  # input_layernorm, QKV projection, q/k norm + RoPE + append: one call
                ops.gemm_qkv_rope(h, lw["w_qkv"], b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc,
                                  b["q"], Hq, Hkv, hd, eps, norm_w=lw["in_norm"], sumsq_in=ss, row_seq=row_seq,
                                  ws=ws, **pg)
            else:  # input_layernorm fused into the QKV projection
                ops.gemm(h, lw["w_qkv"], out=b["qkv"], ws=ws, norm_w=lw["in_norm"], sumsq_in=ss, eps=eps)
            if fused:  # q/k norm + RoPE + append inside the attention launch (same bits)
                ops.attention_qkv(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, eps,
                                  max_kv, row_seq=row_seq, out=b["attn"], ws=ws, seq_rows=seq_rows,
                                  key_chunk=key_chunk)
            else:
                if not qkv_rope:
                    ops.qkv_rope_append(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, Hkv,
                                        hd, c.rope_dim, eps, q_out=b["q"], row_seq=row_seq, **pg)
                ops.attention(b["q"], kc, vc, pos, causal=True, max_kv=max_kv, row_seq=row_seq, out=b["attn"],
                              ws=ws, seq_rows=seq_rows, key_chunk=key_chunk, **pg)
            ops.gemm(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, ws=ws, sumsq_out=ss)
            # post_attention_layernorm fused into the gate/up projection
            ops.gemm(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], ws=ws, norm_w=lw["post_norm"], sumsq_in=ss,
                     eps=eps)
            tap = None
            if l in tap_col and taps_out is not None:
                i = tap_col[l]
                tap = taps_out[:, i * H:(i + 1) * H]
            ops.gemm(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, out2=tap, ws=ws, sumsq_out=ss)
        if head == "hidden":
            return ops.rmsnorm(h, self.norm_w, eps, out=b["xn"])
        if head == "logits":
            return ops.gemm(h, self.lm_head_w, ws=ws, norm_w=self.norm_w, sumsq_in=ss, eps=eps)
        return ops.gemm(h, self.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], ws=ws, norm_w=self.norm_w,
                        sumsq_in=ss, eps=eps)

    def _forward_chain(self, pos, cache, max_kv, tap_col, taps_out, row_seq, head, ws, seq_rows, key_chunk, fused, b):
        """forward() with every run of projections between two attention calls as one
        GEMM-chain launch: [qkv_0], then per layer [o, gate/up, down, next qkv or lm_head]."""
        c = self.cfg
        H, hd, Hq, Hkv = c.hidden_size, c.head_dim, c.num_attention_heads, c.num_key_value_heads
        h, ss, eps = b["h"], b["ss"], c.rms_norm_eps
        pg = cache.paging
        qkv_op = lambda lw: ops.chain_op(h, lw["w_qkv"], out=b["qkv"], norm_w=lw["in_norm"], sumsq_in=ss,  # noqa
                                         eps=eps)
        pending = [qkv_op(self.layers[0])] if self.layers else []
        for l, lw in enumerate(self.layers):
            ops.gemm_chain(pending, ws)
            kc, vc = cache.layer(l)
            if fused:
                ops.attention_qkv(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, eps,
                                  max_kv, row_seq=row_seq, out=b["attn"], ws=ws, seq_rows=seq_rows,
                                  key_chunk=key_chunk)
            else:
                ops.qkv_rope_append(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, Hkv, hd,
                                    c.rope_dim, eps, q_out=b["q"], row_seq=row_seq, **pg)
                ops.attention(b["q"], kc, vc, pos, causal=True, max_kv=max_kv, row_seq=row_seq, out=b["attn"],
                              ws=ws, seq_rows=seq_rows, key_chunk=key_chunk, **pg)
            tap = None
            if l in tap_col and taps_out is not None:
                tap = taps_out[:, tap_col[l] * H:(tap_col[l] + 1) * H]
            pending = [ops.chain_op(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss),
                       ops.chain_op(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], norm_w=lw["post_norm"],
                                    sumsq_in=ss, eps=eps),
                       ops.chain_op(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, out2=tap,
                                    sumsq_out=ss)]
            if l + 1 < len(self.layers):
                pending.append(qkv_op(self.layers[l + 1]))
        return chain_head(pending, h, ss, self.lm_head_w, self.norm_w, eps, head, b, ws)

    def verify_chains(self, M: int, ws: ops.Workspace | None = None) -> list[tuple]:
        """The GEMM-chain launches of one decode-block forward over M rows (M <= 16), as
        (callable, algorithmic bytes, FLOPs) triples on this model's buffers (roofline timing;
        the attention launches between them are left out)."""
        c = self.cfg
        b = self.buffers(M)
        h, ss, eps, H = b["h"], b["ss"], c.rms_norm_eps, c.hidden_size
        chains, cur = [], []

        def add(op, N, K, n_out, extra=0):
            cur.append((op, N * K * 2 + M * K * 2 + M * n_out * 2 + extra, 2 * M * N * K))

        def flush():
            if cur:
                lst = [o for o, _, _ in cur]
                chains.append((lambda lst=lst: ops.gemm_chain(lst, ws), sum(x for _, x, _ in cur),
                               sum(f for _, _, f in cur)))
                cur.clear()

        qkv = lambda lw: add(ops.chain_op(h, lw["w_qkv"], out=b["qkv"], norm_w=lw["in_norm"], sumsq_in=ss, eps=eps),  # noqa
                             lw["w_qkv"].N, H, lw["w_qkv"].N)
        if self.layers:
            qkv(self.layers[0])
        for l, lw in enumerate(self.layers):
            flush()
            Ko, Ng, F = lw["w_o"].K, lw["w_gu"].N, lw["w_down"].K
            add(ops.chain_op(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss), H, Ko, H,
                M * H * 2)
            add(ops.chain_op(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], norm_w=lw["post_norm"], sumsq_in=ss,
                             eps=eps), Ng, H, Ng // 2)
            add(ops.chain_op(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss), H, F, H,
                M * H * 2)
            if l + 1 < len(self.layers):
                qkv(self.layers[l + 1])
        V = self.lm_head_w.N
        add(ops.chain_op(h, self.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], norm_w=self.norm_w,
                         sumsq_in=ss, eps=eps), V, H, 0)
        flush()
        return chains

    def verify_gemms(self, M: int, ws: ops.Workspace | None = None) -> list[tuple]:
        """The GEMM launches of one forward over M rows, as (callable, algorithmic bytes,
        FLOPs) triples on this model's buffers (roofline timing)."""
        c = self.cfg
        b = self.buffers(M)
        h, ss, eps = b["h"], b["ss"], c.rms_norm_eps
        H = c.hidden_size
        out = []

        def nbytes(N, K, n_out, extra=0):
            return N * K * 2 + M * K * 2 + M * n_out * 2 + extra

        def fl(N, K):
            return 2 * M * N * K

        for lw in self.layers:
            Nq = lw["w_qkv"].shape[0]
            out.append((lambda lw=lw: ops.gemm(h, lw["w_qkv"], out=b["qkv"], ws=ws, norm_w=lw["in_norm"],
                                               sumsq_in=ss, eps=eps), nbytes(Nq, H, Nq), fl(Nq, H)))
            Ko = lw["w_o"].shape[1]
            out.append((lambda lw=lw: ops.gemm(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, ws=ws,
                                               sumsq_out=ss), nbytes(H, Ko, H, M * H * 2), fl(H, Ko)))
            Ng = lw["w_gu"].shape[0]
            out.append((lambda lw=lw: ops.gemm(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], ws=ws,
                                               norm_w=lw["post_norm"], sumsq_in=ss, eps=eps), nbytes(Ng, H, Ng // 2),
                        fl(Ng, H)))
            F = lw["w_down"].shape[1]
            out.append((lambda lw=lw: ops.gemm(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, ws=ws,
                                               sumsq_out=ss), nbytes(H, F, H, M * H * 2), fl(H, F)))
        V = self.lm_head_w.shape[0]
        out.append((lambda: ops.gemm(h, self.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], ws=ws,
                                     norm_w=self.norm_w, sumsq_in=ss, eps=eps), nbytes(V, H, 0), fl(V, H)))
        return out


def chain_head(pending: list, h: torch.Tensor, ss: torch.Tensor, lm_head, norm_w, eps: float, head: str, b: dict,
               ws) -> torch.Tensor:
    """Appends the head to the last GEMM chain of a forward and runs it: "argmax" (fused
    lm_head argmax partials), "logits" (bf16 logits) or "hidden" (final RMSNorm rows)."""
    M = h.shape[0]
    if head == "hidden":
        ops.gemm_chain(pending, ws)
        return ops.rmsnorm(h, norm_w, eps, out=b["xn"])
    if head == "logits":
        out = torch.empty((M, lm_head.N), dtype=torch.bfloat16, device=h.device)
        pending.append(ops.chain_op(h, lm_head, out=out, norm_w=norm_w, sumsq_in=ss, eps=eps))
        ops.gemm_chain(pending, ws)
        return out
    pending.append(ops.chain_op(h, lm_head, ops.EPI_ARGMAX, argmax_partials=b["argmax"], norm_w=norm_w, sumsq_in=ss,
                                eps=eps))
    ops.gemm_chain(pending, ws)
    return b["argmax"]


class DraftModel:
    """DFlash block-diffusion draft conditioned on target hidden-state taps (draft.py:190-223)."""

    def __init__(self, cfg: DraftConfig, weights: dict, target: TargetModel, mask_mode: str = "none"):
        self.cfg = cfg
        self.target = target
        self.device = target.device
        self.mask_mode = mask_mode
        dev = self.device
        P = ops.pack_weight
        self.fc = P(weights["fc"].to(dev))
        self.hidden_norm = weights["hidden_norm"].to(dev)
        self.norm_w = weights["norm"].to(dev)
        self.layers = []
        ctx_kv = []
        for lw in weights["layers"]:
            self.layers.append({
                "in_norm": lw["input_layernorm"].to(dev),
                "post_norm": lw["post_attention_layernorm"].to(dev),
                "w_qkv": P(torch.cat([lw["q_proj"].to(dev), lw["k_proj"].to(dev), lw["v_proj"].to(dev)], 0)),
                "w_o": P(lw["o_proj"].to(dev)),
                "w_gu": P(pack_gate_up(lw["gate_proj"].to(dev), lw["up_proj"].to(dev))),
                "w_down": P(lw["down_proj"].to(dev)),
                "q_norm": lw["q_norm"].to(dev),
                "k_norm": lw["k_norm"].to(dev),
            })
            ctx_kv += [lw["k_proj"].to(dev), lw["v_proj"].to(dev)]
        self.w_ctx_kv = P(torch.cat(ctx_kv, 0))
        self.inv_freq = rope_inv_freq(cfg.head_dim, cfg.rope_theta, dev)
        self.use_chain = gemm_chain_enabled()
        self._bufs: dict[tuple, dict[str, torch.Tensor]] = {}

    @property
    def block_size(self) -> int:
        return self.cfg.block_size

    @property
    def mask_token_id(self) -> int:
        return self.cfg.mask_token_id

    @property
    def target_layer_ids(self) -> list[int]:
        return list(self.cfg.target_layer_ids)

    def make_cache(self, batch: int, cap: int, lengths: list[int] | None = None,
                   page_table: torch.Tensor | None = None) -> KVCache:
        c = self.cfg
        if lengths is not None:
            return alloc_kv_paged(c.num_hidden_layers, lengths, c.num_key_value_heads, c.head_dim, self.device,
                                  page_table)
        return alloc_kv(c.num_hidden_layers, batch, c.num_key_value_heads, cap, c.head_dim, self.device)

    def buffers(self, M: int, kind: str) -> dict[str, torch.Tensor]:
        key = (M, kind)
        b = self._bufs.get(key)
        if b is None:
            c = self.cfg
            dev = self.device
            H, hd = c.hidden_size, c.head_dim
            Hq, Hkv = c.num_attention_heads, c.num_key_value_heads
            if kind == "ctx":
                b = {
                    "fc": torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                    "ss": torch.zeros((M, H // 32), dtype=torch.float32, device=dev),
                    "kv": torch.empty((M, c.num_hidden_layers * 2 * Hkv * hd), dtype=torch.bfloat16, device=dev),
                }
            else:
                b = {
                    "h": torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                    "xn": torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                    "qkv": torch.empty((M, (Hq + 2 * Hkv) * hd), dtype=torch.bfloat16, device=dev),
                    "q": torch.empty((M, Hq, hd), dtype=torch.bfloat16, device=dev),
                    "attn": torch.empty((M, Hq * hd), dtype=torch.bfloat16, device=dev),
                    "act": torch.empty((M, c.intermediate_size), dtype=torch.bfloat16, device=dev),
                    "argmax": torch.empty((M, ops.argmax_tiles(c.vocab_size), 2), dtype=torch.float32, device=dev),
                    "ss": torch.zeros((M, H // 32), dtype=torch.float32, device=dev),
                }
            self._bufs[key] = b
        return b

    def ingest_context(self, taps: torch.Tensor, pos: torch.Tensor, cache: KVCache,
                       row_seq: torch.Tensor | None = None, ws: ops.Workspace | None = None) -> None:
        """target_hidden = hidden_norm(fc(taps)) (draft.py:217); its K/V for every layer
        (k_norm + RoPE at the row's position, draft.py:128-147) go into the draft cache.
        Rows with pos < 0 are skipped."""
        c = self.cfg
        M = taps.shape[0]
        b = self.buffers(M, "ctx")
        H, hd, Hkv = c.hidden_size, c.head_dim, c.num_key_value_heads
        if self.use_chain and chain_ok(M, ws):
            ops.gemm_chain([ops.chain_op(taps, self.fc, out=b["fc"], sumsq_out=b["ss"]),
                            ops.chain_op(b["fc"], self.w_ctx_kv, out=b["kv"], norm_w=self.hidden_norm,
                                         sumsq_in=b["ss"], eps=c.rms_norm_eps)], ws)
        else:
            ops.gemm(taps, self.fc, out=b["fc"], ws=ws, sumsq_out=b["ss"])
            if qkv_rope_ok(ws, hd, hd) and len(self.layers) <= ops.KV_LAYERS_MAX:
                # hidden_norm, the stacked k/v projection of every layer and each layer's
                # k_norm + RoPE + append: one call (the same bits as the calls below)
                ops.gemm_kv_append_layers(b["fc"], self.w_ctx_kv, b["kv"], pos, [lw["k_norm"] for lw in self.layers],
                                          self.inv_freq, cache.k, cache.v, Hkv, hd, c.rms_norm_eps,
                                          norm_w=self.hidden_norm, sumsq_in=b["ss"], row_seq=row_seq, ws=ws,
                                          **cache.paging)
                return
            # hidden_norm fused into the stacked k/v projection of every layer
            ops.gemm(b["fc"], self.w_ctx_kv, out=b["kv"], ws=ws, norm_w=self.hidden_norm, sumsq_in=b["ss"],
                     eps=c.rms_norm_eps)
        per = 2 * Hkv * hd
        for l, lw in enumerate(self.layers):
            kc, vc = cache.layer(l)
            view = b["kv"][:, l * per:(l + 1) * per]
            ops.qkv_rope_append(view, pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, 0, Hkv, hd, hd,
                                c.rms_norm_eps, row_seq=row_seq, do_q=False, **cache.paging)

    def forward_block(self, tokens: torch.Tensor, pos: torch.Tensor, cache: KVCache, kv_len: torch.Tensor,
                      max_kv: int, row_seq: torch.Tensor | None = None, head: str = "argmax",
                      ws: ops.Workspace | None = None, seq_rows: int = 0, key_chunk: int = 0):
        """Block rows (the target embedding of [last, mask, ...] = the noise embedding,
        runtime.py:408-410) attend to the draft cache (context rows already ingested)
        plus the block itself; returns the lm_head argmax partials of the final-normed
        hidden states (or the hidden states)."""
        c = self.cfg
        M = tokens.numel()
        b = self.buffers(M, "blk")
        H, hd = c.hidden_size, c.head_dim
        Hq, Hkv = c.num_attention_heads, c.num_key_value_heads
        h, ss, eps = b["h"], b["ss"], c.rms_norm_eps
        ops.embed(tokens, self.target.embed_w, out=h, sumsq_out=ss)
        causal = self.mask_mode == "causal"
        if self.use_chain and chain_ok(M, ws):
            qkv_op = lambda lw: ops.chain_op(h, lw["w_qkv"], out=b["qkv"], norm_w=lw["in_norm"],  # noqa: E731
                                             sumsq_in=ss, eps=eps)
            pending = [qkv_op(self.layers[0])] if self.layers else []
            for l, lw in enumerate(self.layers):
                ops.gemm_chain(pending, ws)
                kc, vc = cache.layer(l)
                ops.qkv_rope_append(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, Hkv, hd,
                                    hd, eps, q_out=b["q"], row_seq=row_seq, **cache.paging)
                ops.attention(b["q"], kc, vc, pos, causal=causal, max_kv=max_kv, kv_len=kv_len, row_seq=row_seq,
                              seq_rows=seq_rows, key_chunk=key_chunk, out=b["attn"], ws=ws, **cache.paging)
                pending = [ops.chain_op(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss),
                           ops.chain_op(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], norm_w=lw["post_norm"],
                                        sumsq_in=ss, eps=eps),
                           ops.chain_op(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss)]
                if l + 1 < len(self.layers):
                    pending.append(qkv_op(self.layers[l + 1]))
            return chain_head(pending, h, ss, self.target.lm_head_w, self.norm_w, eps, head, b, ws)
        qkv_rope = qkv_rope_ok(ws, hd, hd)
        for l, lw in enumerate(self.layers):
            kc, vc = cache.layer(l)
            if qkv_rope:  # QKV projection + q/k norm + RoPE + append in one call (same bits)
                ops.gemm_qkv_rope(h, lw["w_qkv"], b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc,
                                  b["q"], Hq, Hkv, hd, eps, norm_w=lw["in_norm"], sumsq_in=ss, row_seq=row_seq,
                                  ws=ws, **cache.paging)
            else:
                ops.gemm(h, lw["w_qkv"], out=b["qkv"], ws=ws, norm_w=lw["in_norm"], sumsq_in=ss, eps=eps)
                ops.qkv_rope_append(b["qkv"], pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, Hkv, hd,
                                    hd, eps, q_out=b["q"], row_seq=row_seq, **cache.paging)
            ops.attention(b["q"], kc, vc, pos, causal=causal, max_kv=max_kv, kv_len=kv_len, row_seq=row_seq,
                          seq_rows=seq_rows, key_chunk=key_chunk, out=b["attn"], ws=ws, **cache.paging)
            ops.gemm(b["attn"], lw["w_o"], ops.EPI_RESIDUAL, residual=h, out=h, ws=ws, sumsq_out=ss)
            ops.gemm(h, lw["w_gu"], ops.EPI_SILU_MUL, out=b["act"], ws=ws, norm_w=lw["post_norm"], sumsq_in=ss,
                     eps=eps)
            ops.gemm(b["act"], lw["w_down"], ops.EPI_RESIDUAL, residual=h, out=h, ws=ws, sumsq_out=ss)
        if head == "hidden":
            return ops.rmsnorm(h, self.norm_w, eps, out=b["xn"])
        if head == "logits":
            return ops.gemm(h, self.target.lm_head_w, ws=ws, norm_w=self.norm_w, sumsq_in=ss, eps=eps)
        return ops.gemm(h, self.target.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], ws=ws,
                        norm_w=self.norm_w, sumsq_in=ss, eps=eps)
