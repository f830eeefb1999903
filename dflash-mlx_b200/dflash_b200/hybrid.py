"""GPU Qwen3.5 hybrid target: gated-delta-net (GDN) layers + gated full attention.

Layer i is full attention when (i + 1) % full_attention_interval == 0, otherwise a
GDN layer (custom_qwen35_model.py:818). Forward semantics follow the reference's
fork: GDN layer custom_qwen35_model.py:409-484, gated full attention :487-540,
hybrid forward with taps :883-1002.

HBM layout (per device):
  * GDN layer: ``w_in`` packed [qkv | z | b | a] rows (one weight stream, padded to a
    multiple of 32 rows), conv weight [C, 4], ``A_log`` / ``dt_bias`` fp32, gated-norm
    weight [Dv], ``w_out`` [H, Hv*Dv];
  * full-attention layer: ``w_qkv`` = [q_proj (q and output gate interleaved per head) |
    k_proj | v_proj], ``w_o``;
  * caches (``HybridCache``): KV [L_attn, B, Hkv, cap, hd] for the attention layers;
    per GDN layer the fp32 recurrent state [B, Hv, Dv, Dk], the conv state [B, 3, C], the
    conv window [B, 3 + T, C] and, by rollback mode, either per-token snapshots of the
    last verify block [B, T, Hv, Dv, Dk] (rollback = copy snapshot accepted-1) or the
    block's k, v, g, beta (rollback = re-advance the state over the accepted prefix,
    dfl_gdr_recurrence with per-sequence token counts). The conv state takes window rows
    [accepted, accepted + 3) (dfl_gdn_rollback). Both read the accepted length the device
    wrote: no host sync.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import ops
from .config import TargetConfig
from .model import KVCache, alloc_kv
from .weights import pack_gate_up, rope_inv_freq


@dataclass
class HybridCache:
    kv: KVCache                      # attention layers only (index = attention-layer ordinal)
    state: list[torch.Tensor]        # per GDN layer [B, Hv, Dv, Dk] fp32
    snaps: list[torch.Tensor]        # per GDN layer [B, T, Hv, Dv, Dk] fp32
    conv: list[torch.Tensor]         # per GDN layer [B, 3, C] bf16
    window: list[torch.Tensor]       # per GDN layer [B, 3 + Tw, C] bf16
    T: int                           # verify block rows per sequence (snapshot depth)
    Tw: int                          # window rows per sequence (max block / prefill chunk)
    kinds: list = field(default_factory=list)  # per layer "gdn" / "attn"
    last_block: int = 0              # rows of the last block forwarded with snapshots
    mode: str = "snapshot"           # rollback by per-token snapshots, or "replay" of the accepted prefix
    rec: list = field(default_factory=list)  # replay: per GDN layer the block's k, v, g, beta

    @property
    def cap(self) -> int:
        return self.kv.cap


class HybridTargetModel:
    """Qwen3.5-family target (GDN + gated attention) with the TargetModel interface."""

    has_recurrent_state = True

    def __init__(self, cfg: TargetConfig, weights: dict, device="cuda", tp=None):
        """``tp`` (a ``tp.TPComm``): tensor-parallel rank; ``cfg`` / ``weights`` are then
        this rank's shard (``tp.shard_config`` / ``tp.shard_weights``) and each
        row-parallel projection is followed by the peer-memory all-sum."""
        if cfg.model_type != "qwen3_5":
            raise ValueError("HybridTargetModel runs the qwen3_5 family")
        self.tp = tp
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        P = ops.pack_weight
        self.embed_w = weights["embed"].to(dev).contiguous()
        self.lm_head_w = P(self.embed_w if cfg.tie_word_embeddings else weights["lm_head"].to(dev))
        self.norm_w = weights["norm"].to(dev)
        c = cfg
        self.Hk, self.Hv = c.linear_num_key_heads, c.linear_num_value_heads
        self.Dk, self.Dv = c.linear_key_head_dim, c.linear_value_head_dim
        self.C = 2 * self.Hk * self.Dk + self.Hv * self.Dv
        self.vd = self.Hv * self.Dv
        n_in = self.C + self.vd + 2 * self.Hv
        self.n_in_pad = (n_in + 31) // 32 * 32
        self.layers = []
        self.kinds = []
        for i, lw in enumerate(weights["layers"]):
            common = {
                "in_norm": lw["input_layernorm"].to(dev),
                "post_norm": lw["post_attention_layernorm"].to(dev),
                "w_gu": P(pack_gate_up(lw["gate_proj"].to(dev), lw["up_proj"].to(dev))),
                "w_down": P(lw["down_proj"].to(dev)),
            }
            if c.is_linear_layer(i):
                w_in = torch.cat([lw["in_proj_qkv"].to(dev), lw["in_proj_z"].to(dev), lw["in_proj_b"].to(dev),
                                  lw["in_proj_a"].to(dev)], 0)
                if w_in.shape[0] < self.n_in_pad:
                    w_in = torch.cat([w_in, w_in.new_zeros(self.n_in_pad - w_in.shape[0], w_in.shape[1])], 0)
                common.update({
                    "w_in": P(w_in),
                    "conv_w": lw["conv1d"].to(dev).to(torch.bfloat16).contiguous(),
                    "A_log": lw["A_log"].to(dev).float().contiguous(),
                    "dt_bias": lw["dt_bias"].to(dev).float().contiguous(),
                    "gnorm": lw["norm"].to(dev),
                    "w_out": P(lw["out_proj"].to(dev)),
                })
                self.kinds.append("gdn")
            else:
                common.update({
                    "w_qkv": P(torch.cat([lw["q_proj"].to(dev), lw["k_proj"].to(dev), lw["v_proj"].to(dev)], 0)),
                    "w_o": P(lw["o_proj"].to(dev)),
                    "q_norm": lw["q_norm"].to(dev),
                    "k_norm": lw["k_norm"].to(dev),
                })
                self.kinds.append("attn")
            self.layers.append(common)
        self.attn_index = {}
        self.gdn_index = {}
        for i, k in enumerate(self.kinds):
            (self.gdn_index if k == "gdn" else self.attn_index)[i] = len(self.gdn_index if k == "gdn"
                                                                        else self.attn_index)
        self.inv_freq = rope_inv_freq(cfg.rope_dim, cfg.rope_theta, dev)
        self._bufs: dict[int, dict[str, torch.Tensor]] = {}

    # ------------------------------------------------------------------
    def make_cache(self, batch: int, cap: int, block: int = 16, window_rows: int = 128,
                   rollback: str = "snapshot") -> HybridCache:
        """rollback="snapshot": the verify forward writes the state after every token
        (a rollback is a copy; the adapter contract's "advance the whole block, then roll
        back" needs it). rollback="replay": the verify forward keeps the block's k, v, g,
        beta and the rollback re-advances the state over each sequence's accepted prefix
        (the reference's own method, adapters.py:505-560): T-fold less state traffic."""
        if rollback not in ("snapshot", "replay"):
            raise ValueError(f"rollback must be 'snapshot' or 'replay', not {rollback!r}")
        c, dev = self.cfg, self.device
        kv = alloc_kv(max(1, len(self.attn_index)), batch, c.num_key_value_heads, cap, c.head_dim, dev)
        n = len(self.gdn_index)
        S = (self.Hv, self.Dv, self.Dk)
        Tw = max(block, window_rows)
        f32 = dict(dtype=torch.float32, device=dev)
        bf = dict(dtype=torch.bfloat16, device=dev)
        rec = [] if rollback == "snapshot" else [
            {"k": torch.zeros((batch, block, self.Hk, self.Dk), **bf), "v": torch.zeros((batch, block, self.Hv, self.Dv), **bf),
             "g": torch.zeros((batch, block, self.Hv), **f32), "beta": torch.zeros((batch, block, self.Hv), **f32)}
            for _ in range(n)]
        snaps = [torch.zeros((batch, block, *S), **f32) for _ in range(n)] if rollback == "snapshot" else []
        return HybridCache(
            kv=kv,
            state=[torch.zeros((batch, *S), dtype=torch.float32, device=dev) for _ in range(n)],
            snaps=snaps, mode=rollback, rec=rec,
            conv=[torch.zeros((batch, 3, self.C), dtype=torch.bfloat16, device=dev) for _ in range(n)],
            window=[torch.zeros((batch, 3 + Tw, self.C), dtype=torch.bfloat16, device=dev) for _ in range(n)],
            T=block, Tw=Tw, kinds=list(self.kinds))

    def buffers(self, M: int) -> dict[str, torch.Tensor]:
        b = self._bufs.get(M)
        if b is None:
            c, dev = self.cfg, self.device
            H, hd = c.hidden_size, c.head_dim
            bf = dict(dtype=torch.bfloat16, device=dev)
            b = {
                "h": torch.empty((M, H), **bf),
                "xn": torch.empty((M, H), **bf),
                "qkv": torch.empty((M, (2 * c.num_attention_heads + 2 * c.num_key_value_heads) * hd), **bf),
                "q": torch.empty((M, c.num_attention_heads, hd), **bf),
                "attn": torch.empty((M, c.num_attention_heads * hd), **bf),
                "act": torch.empty((M, c.intermediate_size), **bf),
                "proj": torch.empty((M, self.n_in_pad), **bf),
                "gq": torch.empty((M, self.Hk, self.Dk), **bf),
                "gk": torch.empty((M, self.Hk, self.Dk), **bf),
                "gv": torch.empty((M, self.Hv, self.Dv), **bf),
                "gg": torch.empty((M, self.Hv), dtype=torch.float32, device=dev),
                "gbeta": torch.empty((M, self.Hv), dtype=torch.float32, device=dev),
                "go": torch.empty((M, self.vd), **bf),
                "gon": torch.empty((M, self.vd), **bf),
                "argmax": torch.empty((M, ops.argmax_tiles(c.vocab_size), 2), dtype=torch.float32, device=dev),
                "ss": torch.zeros((M, H // 32), dtype=torch.float32, device=dev),
                "xtp": torch.empty((M, H), **bf),  # tensor parallel: the all-sum's normed rows
            }
            self._bufs[M] = b
        return b

    def _normed_gemm(self, h, xn, w, norm_w, ss, ws, epilogue=ops.EPI_STORE, out=None):
        """A projection of RMSNorm(h) * norm_w: from the all-sum's normed rows ``xn`` when
        tensor parallelism produced them (the same bits), else with the GEMM's own norm."""
        eps = self.cfg.rms_norm_eps
        if xn is not None:
            return ops.gemm(xn, w, epilogue, out=out, ws=ws)
        return ops.gemm(h, w, epilogue, out=out, ws=ws, norm_w=norm_w, sumsq_in=ss, eps=eps)

    def _gdn_layer(self, lw, h, ss, b, cache: HybridCache, gi: int, seqs: slice, T: int, verify: bool, ws,
                   xn=None, next_norm=None):
        """One GDN layer over rows [B_s * T] (sequences `seqs` of the cache, T tokens each);
        returns the all-sum's normed rows for ``next_norm`` under tensor parallelism."""
        c = self.cfg
        eps = c.rms_norm_eps
        Bs = (seqs.stop - seqs.start)
        M = Bs * T
        proj = b["proj"]
        self._normed_gemm(h, xn, lw["w_in"], lw["in_norm"], ss, ws, out=proj)
        win = cache.window[gi][seqs]
        replay = verify and cache.mode == "replay"
        if replay:
            if T != cache.T:
                raise ValueError(f"a replay-rollback cache takes verify blocks of exactly {cache.T} rows")
            r = {k: t[seqs] for k, t in cache.rec[gi].items()}
            kvgb = {"k": r["k"].view(M, self.Hk, self.Dk), "v": r["v"].view(M, self.Hv, self.Dv),
                    "g": r["g"].view(M, self.Hv), "beta": r["beta"].view(M, self.Hv)}
        else:
            kvgb = {"k": b["gk"], "v": b["gv"], "g": b["gg"], "beta": b["gbeta"]}
        ops.gdn_prep(proj, lw["conv_w"], lw["A_log"], lw["dt_bias"], cache.conv[gi][seqs], Bs, T, self.Hk, self.Hv,
                     self.Dk, self.Dv, window=win if T <= cache.Tw else None, eps=1e-6,
                     out={"q": b["gq"], **kvgb})
        st = cache.state[gi][seqs]
        o = b["go"].view(M, self.Hv, self.Dv)
        if replay:  # outputs only: the state advances at the rollback, over the accepted prefix
            ops.gdr_recurrence(b["gq"].view(Bs, T, self.Hk, self.Dk), r["k"], r["v"], r["g"], r["beta"], st,
                               o=o.view(Bs, T, self.Hv, self.Dv))
        elif verify:
            ops.gdr_recurrence(b["gq"].view(Bs, T, self.Hk, self.Dk), b["gk"].view(Bs, T, self.Hk, self.Dk),
                               b["gv"].view(Bs, T, self.Hv, self.Dv), b["gg"].view(Bs, T, self.Hv),
                               b["gbeta"].view(Bs, T, self.Hv), st, snapshots=cache.snaps[gi][seqs],
                               o=o.view(Bs, T, self.Hv, self.Dv))
        else:
            ops.gdr_recurrence(b["gq"].view(Bs, T, self.Hk, self.Dk), b["gk"].view(Bs, T, self.Hk, self.Dk),
                               b["gv"].view(Bs, T, self.Hv, self.Dv), b["gg"].view(Bs, T, self.Hv),
                               b["gbeta"].view(Bs, T, self.Hv), st, state_out=st, o=o.view(Bs, T, self.Hv, self.Dv))
        z = proj[:, self.C:self.C + self.vd]
        ops.gated_rmsnorm(b["go"], z, lw["gnorm"], self.Hv, self.Dv, eps, out=b["gon"])
        return self._row_parallel(b["gon"], lw["w_out"], h, ss, None, ws, parity=0, next_norm=next_norm,
                                  xn_out=b["xtp"])

    def _row_parallel(self, x, w, h, ss, tap, ws, parity: int, next_norm=None, xn_out=None):
        """h <- h + x @ w.T (out_proj / o_proj / down_proj): fused residual epilogue on one
        GPU; with tensor parallelism this rank's partial, then the all-sum + residual, which
        also writes RMSNorm(h) * next_norm into ``xn_out`` for the projection that follows
        (returned; None on one GPU, where that projection norms its own input)."""
        if self.tp is None:
            ops.gemm(x, w, ops.EPI_RESIDUAL, residual=h, out=h, out2=tap, ws=ws, sumsq_out=ss)
            return None
        M = x.shape[0]
        # one fp32 partial per rank: a split-K GEMM sums its K ranges locally first, so
        # the peers read one slab each over NVLink (handing them the unsummed K-range
        # slabs, DFL_EPI_PARTIALS, saves that launch but multiplies the NVLink bytes by
        # the split: slower from 2 ranks on, 0.7x at 4)
        ops.gemm(x, w, ops.EPI_STORE_F32, out=self.tp.partial(parity, M), ws=ws)
        if next_norm is None or xn_out is None:
            self.tp.reduce_residual(parity, h, tap, ss, M)
            return None
        self.tp.reduce_residual(parity, h, tap, ss, M, norm_w=next_norm, eps=self.cfg.rms_norm_eps, xn=xn_out[:M])
        return xn_out[:M]

    def forward(self, tokens: torch.Tensor, pos: torch.Tensor, cache: HybridCache, max_kv: int,
                layer_ids: list[int] | None = None, taps_out: torch.Tensor | None = None,
                row_seq: torch.Tensor | None = None, head: str = "argmax", ws: ops.Workspace | None = None,
                seqs: slice | None = None, verify: bool = True, T: int | None = None, seq_rows: int = 0,
                key_chunk: int = 0):
        """Block forward over M = B_s * T rows of sequences ``seqs`` (default: all, T = M / B).
        verify=True writes per-token snapshots + the conv window (a later dfl_gdn_rollback
        picks the accepted prefix); verify=False advances the GDN state in place (prefill)
        and leaves the new conv state to ``commit_prefill``."""
        c = self.cfg
        M = tokens.numel()
        b = self.buffers(M)
        H, hd = c.hidden_size, c.head_dim
        Hq, Hkv = c.num_attention_heads, c.num_key_value_heads
        if seqs is None:
            seqs = slice(0, cache.state[0].shape[0] if cache.state else 1)
        Bs = seqs.stop - seqs.start
        T = T or M // Bs
        tap_col = {lid: i for i, lid in enumerate(sorted(layer_ids or []))}
        h, ss, eps = b["h"], b["ss"], c.rms_norm_eps
        ops.embed(tokens, self.embed_w, out=h, sumsq_out=ss)
        xn = None  # tensor parallel: the all-sum's normed rows for the next projection
        for l, lw in enumerate(self.layers):
            if self.kinds[l] == "gdn":
                xn = self._gdn_layer(lw, h, ss, b, cache, self.gdn_index[l], seqs, T, verify, ws, xn=xn,
                                     next_norm=lw["post_norm"])
            else:
                kc, vc = cache.kv.layer(self.attn_index[l])
                self._normed_gemm(h, xn, lw["w_qkv"], lw["in_norm"], ss, ws, out=b["qkv"])
                qkv = b["qkv"][:, :(2 * Hq + 2 * Hkv) * hd]
                ops.qkv_rope_append(qkv, pos, lw["q_norm"], lw["k_norm"], self.inv_freq, kc, vc, Hq, Hkv, hd,
                                    c.rope_dim, eps, q_out=b["q"], row_seq=row_seq, q_stride=2 * hd)
                ops.attention(b["q"], kc, vc, pos, causal=True, max_kv=max_kv, row_seq=row_seq, out=b["attn"],
                              seq_rows=seq_rows or T, key_chunk=key_chunk,
                              ws=ws, gate=qkv[:, hd:], gate_head_stride=2 * hd)
                xn = self._row_parallel(b["attn"], lw["w_o"], h, ss, None, ws, parity=0, next_norm=lw["post_norm"],
                                        xn_out=b["xtp"])
            self._normed_gemm(h, xn, lw["w_gu"], lw["post_norm"], ss, ws, ops.EPI_SILU_MUL, out=b["act"])
            tap = None
            if l in tap_col and taps_out is not None:
                i = tap_col[l]
                tap = taps_out[:, i * H:(i + 1) * H]
            nxt = self.layers[l + 1]["in_norm"] if l + 1 < len(self.layers) else (
                self.norm_w if head != "hidden" else None)
            xn = self._row_parallel(b["act"], lw["w_down"], h, ss, tap, ws, parity=1, next_norm=nxt, xn_out=b["xtp"])
        if head == "hidden":
            return ops.rmsnorm(h, self.norm_w, eps, out=b["xn"])
        if head == "logits":
            return self._normed_gemm(h, xn, self.lm_head_w, self.norm_w, ss, ws)
        if xn is not None:
            return ops.gemm(xn, self.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], ws=ws)
        return ops.gemm(h, self.lm_head_w, ops.EPI_ARGMAX, argmax_partials=b["argmax"], ws=ws, norm_w=self.norm_w,
                        sumsq_in=ss, eps=eps)

    def rollback(self, cache: HybridCache, accepted: torch.Tensor, acc_stride: int, T: int | None = None) -> None:
        """After a verify block: every GDN layer keeps the state after `accepted` tokens
        (accepted[b * acc_stride], read on the device)."""
        T = T or cache.T
        B = cache.state[0].shape[0] if cache.state else 0
        for gi in range(len(cache.state)):
            if cache.mode == "replay":
                r = cache.rec[gi]
                ops.gdr_recurrence(None, r["k"], r["v"], r["g"], r["beta"], cache.state[gi], state_out=cache.state[gi],
                                   tokens=accepted, tokens_stride=acc_stride)
                ops.gdn_rollback(None, None, cache.conv[gi], cache.window[gi], accepted, acc_stride, B, T, self.Hv,
                                 self.Dv, self.Dk, self.C)
            else:
                ops.gdn_rollback(cache.state[gi], cache.snaps[gi], cache.conv[gi], cache.window[gi], accepted,
                                 acc_stride, B, T, self.Hv, self.Dv, self.Dk, self.C)

    def commit_prefill(self, cache: HybridCache, seqs: slice, n_rows: torch.Tensor, T: int) -> None:
        """After a prefill chunk of T rows: conv state <- last three rows of the window."""
        Bs = seqs.stop - seqs.start
        for gi in range(len(cache.state)):
            ops.gdn_rollback(None, None, cache.conv[gi][seqs], cache.window[gi][seqs], n_rows, 1, Bs, T, self.Hv,
                             self.Dv, self.Dk, self.C)
