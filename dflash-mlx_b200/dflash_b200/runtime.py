"""Speculative DFlash decode loop with the step state kept on the device.

Reference: dflash_mlx/runtime.py:360-589 (``dflash_generate_stream`` /
``dflash_generate``) with the default ``parallel-replay`` verify
(runtime.py:117-163). The reference pulls drafted and posterior tokens to the
host twice per step; here one step is a fixed kernel sequence

    step_prepare -> draft context ingest -> draft block forward -> draft commit
    -> target verify forward (taps into the draft conditioning buffer)
    -> verify accept (argmax, longest prefix, bonus, commit, stop checks)

that reads and writes a per-sequence ``dfl_seq_state`` record, so it can be
captured once in a CUDA graph and replayed. The host polls the state of step k-1
while step k runs. At temperature 0 every verify mode of the reference produces
the same tokens; all of them map onto this path.
"""
from __future__ import annotations

import time
from collections.abc import Iterator
from dataclasses import dataclass
from typing import Any

import torch

from . import ops
from .model import DraftModel, TargetModel

STATE_INTS = 16  # sizeof(dfl_seq_state) / 4
S_START, S_PENDING, S_DRAFT_LEN, S_ACCEPTED, S_BONUS, S_FINISHED, S_STOP, S_STEPS, S_TOTAL, S_PROMPT = range(10)

VERIFY_MODES = ("parallel-replay", "parallel-lazy-logits", "parallel-greedy-argmax", "stream", "chunked")


@dataclass
class DFlashRuntimeEvent:
    token_ids: list[int]
    output_tokens: list[int]
    metrics: dict[str, Any] | None = None
    finished: bool = False


def longest_prefix_match(draft_tokens: list[int], verifier_tokens: list[int]) -> int:
    """Host restatement of runtime.py:41-47 (the device kernel does the same per step)."""
    matched = 0
    for d, v in zip(draft_tokens, verifier_tokens):
        if d != v:
            break
        matched += 1
    return matched


def sample_tokens(logits: torch.Tensor, temperature: float, seed: int | None = None) -> torch.Tensor:
    """runtime.py:22-29: argmax below temperature 1e-5, else a categorical sample of
    softmax(logits / temperature) (Gumbel-max on the device; fresh keys from torch's
    generator unless ``seed`` is given)."""
    flat = logits.reshape(-1, logits.shape[-1])
    if temperature < 1e-5:
        return torch.argmax(flat, dim=-1).reshape(logits.shape[:-1]).to(torch.int32)
    if seed is None:
        seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    keys = ops.keys_tensor([ops.sample_key(seed, 0, 0, r) for r in range(flat.shape[0])], flat.device)
    part = ops.sample_partials(flat.to(torch.bfloat16).contiguous(), keys, temperature)
    return ops.argmax_reduce(part).reshape(logits.shape[:-1]).to(torch.int32)


def _packed_weights(model) -> list:
    """Every packed GEMM weight a target / draft model holds (workspace sizing)."""
    out = []
    for v in vars(model).values():
        items = v if isinstance(v, list) else [v]
        for it in items:
            if isinstance(it, ops.PackedWeight):
                out.append(it)
            elif isinstance(it, dict):
                out.extend(x for x in it.values() if isinstance(x, ops.PackedWeight))
    return out


class SpecSession:
    """Device buffers and the captured step for B sequences decoded together."""

    def __init__(self, target: TargetModel, draft: DraftModel | None, batch: int, max_total: int,
                 block_size: int, stop_token_ids: set[int] | None = None, use_graph: bool = True,
                 max_steps: int | None = None, prefill_chunk: int = 128, temperature: float = 0.0,
                 seed: int = 0, profile: bool = False, paged: bool = True):
        """temperature >= 1e-5 samples (Gumbel-max on the bf16 logits, keyed by sequence and
        absolute position: the speculative decode reproduces the plain sampled decode of the
        same seed token for token); below it decoding is greedy (fused lm_head argmax)."""
        self.sampled = temperature >= 1e-5
        # profile=True: the verify half is captured as three graphs (forward, accept,
        # rollback) so that step(events=5 events) can time each part on the device
        self.profile = profile
        self.profile_events: list[tuple] = []
        self.temperature = float(temperature)
        self.seed = int(seed)
        self.target = target
        self.draft = draft
        self.B = batch
        self.bs = block_size
        self.dev = target.device
        self.use_graph = use_graph
        self.prefill_chunk = prefill_chunk
        tc = target.cfg
        B, bs = batch, block_size
        self.cap = max_total + 2 * bs + 1
        # batched sessions (4+ sequences) switch two kernel forms, both chosen from the
        # batch size alone so that a batch's plain decode and its speculative decode
        # use the same arithmetic: attention splits keys every 1024 positions (a batch
        # already fills the SMs; long splits cut the partial-result traffic) instead of
        # every 64 (one 64-key block per CTA: the most SMs on a single stream's keys,
        # measured fastest on B200 at config 3's contexts), and every GEMM runs whole-K
        # tensor-core tiles (weights read once for all rows) instead of the M <= 16
        # weight-streaming split-K form
        self.batched = batch >= 4
        self.key_chunk = 1024 if self.batched else 64
        self.out_cap = self.cap
        self.max_steps = max_steps or (max_total + 1)
        # under 16 sequences, weights with few 128-row tiles also split K (fixed ranges)
        self.ws = ops.Workspace(self.dev, wide=self.batched, wide_split=4 if batch < 16 else 1)
        dev = self.dev
        i32 = dict(dtype=torch.int32, device=dev)
        self.state = torch.zeros((B, STATE_INTS), **i32)
        self.out_tokens = torch.zeros((B, self.out_cap), **i32)
        self.block = torch.zeros(B * bs, **i32)
        self.tpos = torch.zeros(B * bs, **i32)
        self.dpos_ctx = torch.zeros(B * bs, **i32)
        self.dpos_blk = torch.zeros(B * bs, **i32)
        self.dkv_len = torch.zeros(B, **i32)
        self.row_seq = (torch.arange(B * bs, device=dev, dtype=torch.int32) // bs) if B > 1 else None
        self.accept_log = torch.zeros((B, self.max_steps), **i32)
        stops = sorted(stop_token_ids or [])
        self.n_stop = len(stops)
        self.stop_ids = torch.tensor(stops or [0], **i32)
        self.hybrid = bool(getattr(target, "has_recurrent_state", False))
        # hybrid targets roll back by replaying the accepted prefix (no per-token snapshots)
        # dense targets keep paged K/V (pages for each sequence's own length, allocated at
        # prefill when the lengths are known); the hybrid's attention layers stay contiguous
        self.paged = paged and not self.hybrid
        self.tcache = None
        if self.hybrid:
            self.tcache = target.make_cache(B, self.cap, block=bs, rollback="replay")
        elif not self.paged:
            self.tcache = target.make_cache(B, self.cap, block=bs)
        self.layer_ids = sorted(draft.target_layer_ids) if draft is not None else []
        ntaps = max(1, len(self.layer_ids))
        self.taps = torch.zeros((B * bs, ntaps * tc.hidden_size), dtype=torch.bfloat16, device=dev)
        self.dcache = None
        if draft is not None and not self.paged:
            self.dcache = draft.make_cache(B, self.cap)
        self.inject_tokens = self.inject_len = self.inject_noise = None
        self.graph: torch.cuda.CUDAGraph | None = None
        self.host_state = torch.zeros((B, STATE_INTS), dtype=torch.int32, pin_memory=True)
        if self.sampled:
            self.keys = torch.zeros(B * bs, dtype=torch.int64, device=dev)
            self.spart = torch.empty((B * bs, ops.argmax_tiles(tc.vocab_size), 2), dtype=torch.float32, device=dev)
        self._reserve_workspace()

    def _reserve_workspace(self) -> None:
        """Sizes the scratch for every launch shape up front: a captured graph holds raw
        pointers into it, so it must never be reallocated afterwards."""
        tc = self.target.cfg
        q = ops._lib.query
        gemm_need = 0
        attn_need = 0
        wide_need = 0
        shapes = [self.B * self.bs, self.prefill_chunk]
        nk = {(w.N, w.K) for w in _packed_weights(self.target)}
        if self.draft is not None:
            nk |= {(w.N, w.K) for w in _packed_weights(self.draft)}
        for M in shapes:
            for N, K in nk:
                gemm_need = max(gemm_need, int(q("dfl_gemm_workspace_bytes", M, N, K, 0)))
                wide_need = max(wide_need, int(q("dfl_gemm_wide_workspace_bytes", M, N, K, 1,
                                                   ops.wide_split(N, K, self.ws))))
            attn_need = max(attn_need, int(q("dfl_attention_workspace_bytes", M, tc.num_attention_heads,
                                               tc.head_dim, self.cap, self.key_chunk)))
        self.ws.ensure_gemm(gemm_need)
        self.ws.ensure_attn(attn_need)
        if self.ws.wide:
            self.ws.ensure_wide(wide_need)

    # ------------------------------------------------------------------
    def set_injection(self, trace: torch.Tensor, lengths: torch.Tensor, noise: torch.Tensor) -> None:
        """Oracle-injected drafts: block[1+i] = trace[start+1+i] for i < lengths[step], else noise."""
        self.inject_tokens = trace.to(self.dev, torch.int32).contiguous()
        self.inject_len = lengths.to(self.dev, torch.int32).contiguous()
        self.inject_noise = noise.to(self.dev, torch.int32).contiguous()
        self.graph = None

    def prefill(self, prompts: list[list[int]], max_new_tokens: int | list[int]) -> list[int]:
        """Target forward over each prompt (taps for the draft context, runtime.py:384-390);
        returns the first greedy token of every sequence."""
        B = self.B
        tc = self.target.cfg
        dev = self.dev
        if len(prompts) != B:
            raise ValueError(f"expected {B} prompts")
        if isinstance(max_new_tokens, int):
            max_new_tokens = [max_new_tokens] * B
        if self.paged:
            # pages for each sequence's own length (prompt + new tokens + two blocks of slack:
            # the bound the capacity check below applies)
            lengths = [min(self.cap, len(p) + m + 2 * self.bs + 1) for p, m in zip(prompts, max_new_tokens)]
            self.tcache = self.target.make_cache(B, self.cap, block=self.bs, lengths=lengths)
            if self.draft is not None:
                self.dcache = self.draft.make_cache(B, self.cap, lengths=lengths, page_table=self.tcache.page_table)
            self.graph = None  # a recorded step holds the previous caches' pointers
        firsts = []
        st = torch.zeros((B, STATE_INTS), dtype=torch.int32)
        head = "logits" if self.sampled else "argmax"
        for b, prompt in enumerate(prompts):
            P = len(prompt)
            if P == 0:
                raise ValueError("empty prompt")
            if P + max_new_tokens[b] + 2 * self.bs + 1 > self.cap:
                raise ValueError("prompt + max_new_tokens exceeds the session capacity")
            toks = torch.tensor(prompt, dtype=torch.int32, device=dev)
            seq = torch.full((self.prefill_chunk,), b, dtype=torch.int32, device=dev) if B > 1 else None
            last_part = None
            for c0 in range(0, P, self.prefill_chunk):
                c1 = min(P, c0 + self.prefill_chunk)
                n = c1 - c0
                pos = torch.arange(c0, c1, dtype=torch.int32, device=dev)
                rs = seq[:n] if seq is not None else None
                taps = torch.empty((n, self.taps.shape[1]), dtype=torch.bfloat16, device=dev)
                if self.hybrid:
                    # recurrent layers advance in place over the chunk; conv state from the window
                    part = self.target.forward(toks[c0:c1], pos, self.tcache, max_kv=c1, layer_ids=self.layer_ids,
                                               taps_out=taps, row_seq=rs, ws=self.ws, seqs=slice(b, b + 1),
                                               verify=False, T=n, seq_rows=n, key_chunk=self.key_chunk,
                                               head=head)
                    self.target.commit_prefill(self.tcache, slice(b, b + 1),
                                               torch.full((1,), n, dtype=torch.int32, device=dev), n)
                else:
                    part = self.target.forward(toks[c0:c1], pos, self.tcache, max_kv=c1, layer_ids=self.layer_ids,
                                               taps_out=taps, row_seq=rs, ws=self.ws, seq_rows=n,
                                               key_chunk=self.key_chunk, head=head)
                if self.sampled:  # part holds logits: sample the token at position P
                    key = ops.keys_tensor([ops.sample_key(self.seed, ops.SAMPLE_TAG_TARGET, b, P)], dev)
                    last_part = ops.sample_partials(part[n - 1:n], key, self.temperature)
                else:
                    last_part = part[n - 1:n]
                if self.draft is not None:
                    self.draft.ingest_context(taps, pos, self.dcache, row_seq=rs, ws=self.ws)
            first = int(ops.argmax_reduce(last_part).item())
            firsts.append(first)
            self.out_tokens[b, :P] = toks
            self.out_tokens[b, P] = first
            total_max = P + max_new_tokens[b]
            stop_index = P if first in set(self.stop_ids.tolist()[: self.n_stop]) else -1
            # like runtime.py:406, a stop token sampled at prefill still runs one decode step
            finished = int(P + 1 > total_max)
            st[b, S_START] = P
            st[b, S_PENDING] = 0
            st[b, S_DRAFT_LEN] = P
            st[b, S_FINISHED] = finished
            st[b, S_STOP] = stop_index
            st[b, S_TOTAL] = total_max
            st[b, S_PROMPT] = P
        self.state.copy_(st.to(dev))
        self.accept_log.zero_()
        return firsts

    # ------------------------------------------------------------------
    def _draft_kernels(self) -> None:
        """step_prepare + draft proposal (runtime.py:407-423)."""
        B, bs = self.B, self.bs
        ops.step_prepare(self.state, self.out_tokens, self.block, bs,
                         self.draft.mask_token_id if self.draft is not None else 0,
                         self.tpos, self.dpos_ctx if self.draft else None, self.dpos_blk if self.draft else None,
                         self.dkv_len if self.draft else None, B)
        if self.draft is not None:
            d = self.draft
            d.ingest_context(self.taps, self.dpos_ctx, self.dcache, row_seq=self.row_seq, ws=self.ws)
            part = d.forward_block(self.block, self.dpos_blk, self.dcache, self.dkv_len, self.cap,
                                   row_seq=self.row_seq, ws=self.ws, seq_rows=bs, key_chunk=self.key_chunk,
                                   head="logits" if self.sampled else "argmax")
            if self.sampled:  # draft row i proposes the token at position start + i
                ops.sample_keys(self.state, B, bs, self.seed, ops.SAMPLE_TAG_DRAFT, 0, self.keys)
                part = ops.sample_partials(part, self.keys, self.temperature, out=self.spart)
            ops.draft_commit(self.state, part, self.block, bs, B, self.inject_tokens, self.inject_len,
                             self.inject_noise)

    def _verify_kernels(self) -> None:
        """Target verify forward + accept (parallel-replay, runtime.py:117-163)."""
        self._verify_forward()
        self._verify_accept()
        self._verify_rollback()

    def _verify_forward(self) -> None:
        part = self.target.forward(self.block, self.tpos, self.tcache, max_kv=self.cap, layer_ids=self.layer_ids,
                                   taps_out=self.taps, row_seq=self.row_seq, ws=self.ws, seq_rows=self.bs,
                                   key_chunk=self.key_chunk, head="logits" if self.sampled else "argmax")
        if self.sampled:  # verify row i predicts the token at position start + i + 1
            ops.sample_keys(self.state, self.B, self.bs, self.seed, ops.SAMPLE_TAG_TARGET, 1, self.keys)
            part = ops.sample_partials(part, self.keys, self.temperature, out=self.spart)
        self._verify_part = part

    def _verify_accept(self) -> None:
        ops.verify_accept(self.state, self._verify_part, self.block, self.bs, self.out_tokens, self.B,
                          stop_ids=self.stop_ids, n_stop=self.n_stop, accept_log=self.accept_log)

    def _verify_rollback(self) -> None:
        if self.hybrid:
            # recurrent layers keep the state after the accepted prefix (snapshot restore);
            # attention KV needs no truncation: the next block overwrites rows past start
            self.target.rollback(self.tcache, self.state[:, S_ACCEPTED], STATE_INTS, self.bs)

    def capture(self) -> None:
        """Captures the draft half and the verify half of a step as two CUDA graphs."""
        # the step's activation buffers exist before the capture: one first made inside it
        # would put its zero fill into the graph, to run again at every replay
        M = self.B * self.bs
        self.target.buffers(M)
        if self.draft is not None:
            for kind in ("ctx", "blk"):
                self.draft.buffers(M, kind)
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        parts = [self._draft_kernels]
        parts += [self._verify_forward, self._verify_accept, self._verify_rollback] if self.profile \
            else [self._verify_kernels]
        graphs = [torch.cuda.CUDAGraph() for _ in parts]
        with torch.cuda.stream(s):
            for g, fn in zip(graphs, parts):
                with torch.cuda.graph(g, stream=s):
                    fn()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = tuple(graphs)

    def step(self, events: tuple | None = None) -> None:
        """One speculative step. ``events`` = (before, between, after) CUDA events to time
        the draft and the verify halves; a session made with profile=True takes five
        (before, after draft, after verify forward, after accept, after rollback)."""
        if self.use_graph and self.graph is None:
            self.capture()
        fine = events is not None and len(events) == 5
        if fine and not self.profile:
            raise ValueError("five step events need a session made with profile=True")
        if self.use_graph:
            parts = [g.replay for g in self.graph]
        else:
            parts = [self._draft_kernels] + ([self._verify_forward, self._verify_accept, self._verify_rollback]
                                             if self.profile else [self._verify_kernels])
        if events is not None:
            events[0].record()
        for i, fn in enumerate(parts):
            fn()
            if events is not None and (fine or i == 0):
                events[i + 1].record()
        if events is not None and not fine:
            events[2].record()

    def poll_state(self) -> torch.Tensor:
        self.host_state.copy_(self.state, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return self.host_state.clone()

    def run_iter(self, max_steps: int, copy_tokens: bool = True, before_step=None, first_index: int = 0):
        """Launches up to ``max_steps`` steps keeping one step in flight: after launching
        step k the host waits only for the state (and tokens) of step k-1, copied into
        pinned memory, and yields ``(state, tokens)`` for it. Stops once every sequence
        is finished (the step already in flight then runs as a no-op). ``before_step(i)``
        is called before launching the step with global index ``first_index + i`` (for
        per-step host-to-device input copies on the same stream)."""
        if not hasattr(self, "_ring"):
            self._ring = [(torch.empty_like(self.host_state).pin_memory(),
                           torch.empty(self.out_tokens.shape, dtype=torch.int32).pin_memory(),
                           torch.cuda.Event()) for _ in range(2)]
        stream = torch.cuda.current_stream(self.dev)
        inflight: list[int] = []
        launched = 0
        done = False
        while not done and (launched < max_steps or inflight):
            if launched < max_steps:
                if before_step is not None:
                    before_step(first_index + launched)
                if self.profile:
                    evs = tuple(torch.cuda.Event(enable_timing=True) for _ in range(5))
                    self.profile_events.append(evs)
                    self.step(events=evs)
                else:
                    self.step()
                hs, ht, ev = self._ring[launched % 2]
                hs.copy_(self.state, non_blocking=True)
                if copy_tokens:
                    ht.copy_(self.out_tokens, non_blocking=True)
                ev.record(stream)
                inflight.append(launched % 2)
                launched += 1
                if len(inflight) < 2 and launched < max_steps:
                    continue
            slot = inflight.pop(0)
            hs, ht, ev = self._ring[slot]
            ev.synchronize()
            done = bool((hs[:, S_FINISHED] != 0).all())
            yield hs, ht
        stream.synchronize()
        self.steps_launched = launched

    def profile_times(self) -> dict[str, float]:
        """Device time of each part of the profiled steps, summed (seconds), under the
        reference's profile keys (runtime.py:61-71, 117-163, 406-518)."""
        keys = ("draft_time_s", "verify_forward_logits_time_s", "verify_prefix_time_s", "verify_rollback_time_s")
        out = dict.fromkeys(keys, 0.0)
        for evs in self.profile_events:
            evs[-1].synchronize()
            for i, k in enumerate(keys):
                out[k] += evs[i].elapsed_time(evs[i + 1]) * 1e-3
        out["verify_time_s"] = sum(out[k] for k in keys[1:])
        return out

    def run(self, max_steps: int, copy_tokens: bool = False) -> int:
        for _ in self.run_iter(max_steps, copy_tokens):
            pass
        return self.steps_launched

    def outputs(self) -> tuple[list[list[int]], list[list[int]], torch.Tensor]:
        """Committed tokens (truncated like runtime.py:499-507, 518) and acceptance lengths."""
        st = self.state.cpu()
        toks = self.out_tokens.cpu()
        log = self.accept_log.cpu()
        outs, accs = [], []
        for b in range(self.B):
            start, stop, total, steps = (int(st[b, S_START]), int(st[b, S_STOP]), int(st[b, S_TOTAL]),
                                         int(st[b, S_STEPS]))
            n = start + 1
            if stop >= 0:
                n = min(n, stop + 1)
            n = min(n, total)
            outs.append(toks[b, :n].tolist())
            accs.append(log[b, :steps].tolist())
        return outs, accs, st


def dflash_generate_stream(target: TargetModel, draft: DraftModel, prompt_tokens, max_new_tokens: int,
                           temperature: float, stop_token_ids: set[int], layer_ids: list[int] | None,
                           speculative_tokens: int | None, verify_mode: str = "parallel-replay",
                           verify_chunk_size: int = 4, profile: bool = False,
                           use_graph: bool = True, seed: int = 0) -> Iterator[DFlashRuntimeEvent]:
    """Single-sequence generator with the reference's event and metrics shape (runtime.py:360-555).
    temperature >= 1e-5 samples (sample_tokens, runtime.py:22-29) with noise keyed by
    ``seed`` and absolute position, so the output equals the plain sampled decode."""
    if verify_mode not in VERIFY_MODES:
        raise ValueError(f"unknown verify_mode {verify_mode!r}")
    if layer_ids is not None and draft is not None and sorted(layer_ids) != sorted(draft.target_layer_ids):
        raise ValueError("layer_ids must match the draft's target_layer_ids")
    prompt = prompt_tokens.tolist() if hasattr(prompt_tokens, "tolist") else list(prompt_tokens)
    prompt = [int(t) for t in prompt]
    prompt_len = len(prompt)
    bs_max = draft.block_size if draft is not None else 1
    block_size = bs_max if speculative_tokens is None else max(1, min(speculative_tokens, bs_max))
    use_draft = draft if block_size > 1 else None
    total_max = prompt_len + max_new_tokens
    sess = SpecSession(target, use_draft, 1, total_max, block_size, stop_token_ids, use_graph=use_graph,
                       temperature=temperature, seed=seed, profile=profile)

    torch.cuda.synchronize(target.device)
    t0 = time.perf_counter()
    first = sess.prefill([prompt], max_new_tokens)[0]
    torch.cuda.synchronize(target.device)
    prefill_time = time.perf_counter() - t0

    output_tokens = prompt + [first]
    streamed_len = prompt_len
    if max_new_tokens > 0:
        yield DFlashRuntimeEvent(token_ids=output_tokens[streamed_len:], output_tokens=list(output_tokens))
        streamed_len = len(output_tokens)

    decode_start = time.perf_counter()
    bookkeeping = 0.0
    finished = bool(sess.state[0, S_FINISHED].item()) or max_new_tokens <= 0
    if not finished:
        # a step commits at least one token, so max_new_tokens + 1 steps always finish
        for host_state, host_tokens in sess.run_iter(max_new_tokens + 1):
            t_book = time.perf_counter()
            start = int(host_state[0, S_START])
            stop = int(host_state[0, S_STOP])
            n = min(start + 1, total_max)
            if stop >= 0:
                n = min(n, stop + 1)
            if n > streamed_len:
                toks = host_tokens[0, :n].tolist()
                bookkeeping += time.perf_counter() - t_book
                yield DFlashRuntimeEvent(token_ids=toks[streamed_len:], output_tokens=toks)
                streamed_len = n
            else:
                bookkeeping += time.perf_counter() - t_book
    torch.cuda.synchronize(target.device)
    decode_time = time.perf_counter() - decode_start
    outs, accs, st = sess.outputs()
    output_tokens = outs[0]
    acceptance_lengths = accs[0]
    stop_index = int(st[0, S_STOP])
    generated = max(len(output_tokens) - prompt_len, 0)
    total_time = prefill_time + decode_time
    metrics = {
        "num_input_tokens": prompt_len,
        "num_output_tokens": generated,
        "prefill_time_s": prefill_time,
        "decode_time_s": decode_time,
        "total_time_s": total_time,
        "prompt_tps": prompt_len / max(prefill_time, 1e-9),
        "generation_tps": generated / max(decode_time, 1e-9),
        "end_to_end_tps": generated / max(total_time, 1e-9),
        "avg_acceptance_length": sum(acceptance_lengths) / max(len(acceptance_lengths), 1),
        "acceptance_lengths": acceptance_lengths,
        "peak_memory_gb": torch.cuda.max_memory_allocated(target.device) / 1e9,
        "target_cache_summary": f"kv_len={int(sess.state[0, S_START].item())} x {target.cfg.num_hidden_layers} layers",
        "speculative_tokens": block_size,
        # why decoding ended: a stop token inside the length limit, else the limit
        "finish_reason": "stop" if 0 <= stop_index < total_max else "max_tokens",
    }
    if profile:
        # device time of the draft and verify parts (CUDA events around each captured part),
        # host time spent reading back and committing tokens, and the remainder of the
        # decode wall time; the device parts of step k overlap the host's work on step k-1
        prof = sess.profile_times()
        prof["bookkeeping_time_s"] = bookkeeping
        profiled = prof["draft_time_s"] + prof["verify_time_s"] + bookkeeping
        metrics["profile"] = {**prof, "unattributed_decode_time_s": decode_time - profiled,
                              "steps": len(acceptance_lengths), "verify_mode": verify_mode}
    yield DFlashRuntimeEvent(token_ids=[], output_tokens=list(output_tokens), metrics=metrics, finished=True)


@dataclass
class BatchStreamEvent:
    """New committed tokens of sequence ``index`` of a batched decode; ``finished`` marks its
    last event, with ``finish_reason`` "stop" (a stop token) or "max_tokens" (the limit)."""
    index: int
    token_ids: list[int]
    finished: bool = False
    finish_reason: str | None = None
    acceptance_lengths: list[int] | None = None


def dflash_generate_batch_stream(target: TargetModel, draft: DraftModel | None, prompts: list[list[int]],
                                 max_new_tokens: list[int], temperature: float, stop_token_ids: set[int],
                                 speculative_tokens: int | None = None, use_graph: bool = True,
                                 seed: int = 0) -> Iterator[list[BatchStreamEvent]]:
    """Decodes several prompts together in one batched session (per-sequence acceptance,
    stop and length rules of runtime.py:405-518 applied to every row) and yields, after
    each step, the events of the sequences that committed tokens or finished in it."""
    B = len(prompts)
    if B == 0:
        return
    if len(max_new_tokens) != B:
        raise ValueError("one max_new_tokens per prompt")
    prompts = [[int(t) for t in p] for p in prompts]
    bs_max = draft.block_size if draft is not None else 1
    block_size = bs_max if speculative_tokens is None else max(1, min(speculative_tokens, bs_max))
    use_draft = draft if block_size > 1 else None
    totals = [len(p) + m for p, m in zip(prompts, max_new_tokens)]
    sess = SpecSession(target, use_draft, B, max(totals), block_size, stop_token_ids, use_graph=use_graph,
                       temperature=temperature, seed=seed)
    firsts = sess.prefill(prompts, max_new_tokens)
    streamed = [len(p) for p in prompts]
    done = [False] * B
    events = []
    for b in range(B):
        if max_new_tokens[b] <= 0:
            done[b] = True
            events.append(BatchStreamEvent(b, [], True, "max_tokens", []))
        else:
            events.append(BatchStreamEvent(b, [firsts[b]]))
            streamed[b] += 1
    if events:
        yield events

    def finish(b: int, host_state) -> BatchStreamEvent:
        stop = int(host_state[b, S_STOP])
        steps = int(host_state[b, S_STEPS])
        return BatchStreamEvent(b, [], True, "stop" if 0 <= stop < totals[b] else "max_tokens",
                                sess.accept_log[b, :steps].tolist())

    if not all(done):
        for host_state, host_tokens in sess.run_iter(max(max_new_tokens) + 1):
            events = []
            for b in range(B):
                if done[b]:
                    continue
                start, stop = int(host_state[b, S_START]), int(host_state[b, S_STOP])
                n = min(start + 1, totals[b])
                if stop >= 0:
                    n = min(n, stop + 1)
                if n > streamed[b]:
                    events.append(BatchStreamEvent(b, host_tokens[b, streamed[b]:n].tolist()))
                    streamed[b] = n
                if int(host_state[b, S_FINISHED]):
                    done[b] = True
                    events.append(finish(b, host_state))
            if events:
                yield events
    if not all(done):  # every sequence is finished once the steps run out
        st = sess.state.cpu()
        yield [finish(b, st) for b in range(B) if not done[b]]


def dflash_generate(target: TargetModel, draft: DraftModel, prompt_tokens, max_new_tokens: int, temperature: float,
                    stop_token_ids: set[int], layer_ids: list[int] | None, speculative_tokens: int | None,
                    verify_mode: str = "parallel-replay", verify_chunk_size: int = 4, profile: bool = False,
                    use_graph: bool = True, seed: int = 0) -> tuple[list[int], dict[str, Any]]:
    final = None
    for event in dflash_generate_stream(target, draft, prompt_tokens, max_new_tokens, temperature, stop_token_ids,
                                        layer_ids, speculative_tokens, verify_mode, verify_chunk_size, profile,
                                        use_graph, seed):
        if event.finished:
            final = event
    if final is None or final.metrics is None:
        raise RuntimeError("DFlash generation did not produce a final event.")
    return final.output_tokens, final.metrics
