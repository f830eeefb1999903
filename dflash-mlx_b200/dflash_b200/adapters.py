"""Target-adapter contract of the reference, on B200 tensors.

Mirrors ``MLXTargetAdapter`` (dflash_mlx/adapters.py:246-338), the adapter
registry (adapters.py:719-726) and the ``LoadedTargetModel`` facade
(adapters.py:729-826). The rules kept verbatim:

  * tap rule: ``target_hidden`` is the residual stream after each layer in
    ``layer_ids``, concatenated in ascending layer order (adapters.py:624-630);
  * cache types: one KV cache per full-attention layer (and, for the hybrid,
    a conv + recurrent state per gated-delta layer);
  * rollback: KV trim by ``block - accepted`` (adapters.py:697-700); Qwen3 has no
    linear-layer state to roll back (adapters.py:702-709).

The per-call methods here run the same kernels as the fused step in
``runtime.py`` and are what a caller written against the reference's adapter
API uses; ``runtime.SpecSession`` is the graph-captured fast path.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from . import ops
from .config import PRESETS
from .model import KVCache, TargetModel
from .weights import random_target_weights


@dataclass
class TargetCache:
    """Per-sequence KV slots plus the length (mlx-lm KVCache.offset) of every layer."""

    kv: KVCache
    offset: int = 0

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n


class ByteTokenizer:
    """Stand-in tokenizer for random-init models: UTF-8 bytes folded into the vocabulary."""

    def __init__(self, vocab_size: int, eos_token_ids: tuple[int, ...] = ()):
        self.vocab_size = vocab_size
        self.eos_token_ids = list(eos_token_ids)

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")]

    def decode(self, tokens, skip_special_tokens: bool = False) -> str:
        return bytes(int(t) % 256 for t in tokens).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True, **_):
        return "".join(m["content"] for m in messages)


class TargetAdapter:
    family: str = "unknown"

    def build_prompt(self, tokenizer, prompt_text: str) -> torch.Tensor:
        messages = [{"role": "user", "content": prompt_text}]
        try:
            prompt = tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                                   enable_thinking=False)
        except TypeError:
            prompt = tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
        return torch.tensor(tokenizer.encode(prompt, add_special_tokens=False), dtype=torch.int32)

    def stop_token_ids(self, tokenizer) -> set[int]:
        eos = tokenizer.eos_token_ids
        return {eos} if isinstance(eos, int) else set(eos)

    def make_cache(self, model, cap: int = 8192) -> TargetCache:
        return TargetCache(model.make_cache(1, cap))

    def embed_tokens(self, model: TargetModel, tokens: torch.Tensor) -> torch.Tensor:
        t = tokens.reshape(-1).to(model.device, torch.int32).contiguous()
        return ops.embed(t, model.embed_w).reshape(*tokens.shape, -1)

    def lm_head_logits(self, model: TargetModel, hidden: torch.Tensor) -> torch.Tensor:
        h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
        return ops.gemm(h, model.lm_head_w).reshape(*hidden.shape[:-1], -1)

    def lm_head_argmax(self, model: TargetModel, hidden: torch.Tensor) -> torch.Tensor:
        """The fused top-1 lm_head hook of adapters.py:264-271: logits never reach HBM."""
        h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
        part = ops.gemm(h, model.lm_head_w, ops.EPI_ARGMAX)
        return ops.argmax_reduce(part).reshape(hidden.shape[:-1])

    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records=False):
        raise NotImplementedError

    def forward_verifier_states(self, model, inputs, cache, layer_ids):
        raise NotImplementedError

    def forward_accept_all_block(self, model, inputs, cache, layer_ids):
        logits, hidden = self.forward_with_hidden_states(model, inputs, cache, layer_ids)
        return logits[:, -1:, :], hidden

    def snapshot_linear_caches(self, model, cache) -> dict:
        return {}

    def restore_linear_caches(self, model, cache, snapshots) -> None:
        return None

    def rewind_kv_caches(self, cache: TargetCache, num_tokens: int) -> None:
        cache.trim(num_tokens)

    def rollback_linear_caches(self, model, cache, rollback_records, accepted_inputs) -> None:
        return None

    def cache_summary(self, cache: TargetCache) -> str:
        return f"kv={cache.offset}"


class Qwen3TargetAdapter(TargetAdapter):
    family = "qwen3"

    def _forward_states(self, model: TargetModel, inputs: torch.Tensor, cache: TargetCache, layer_ids):
        toks = inputs.reshape(-1).to(model.device, torch.int32).contiguous()
        T = toks.numel()
        pos = torch.arange(cache.offset, cache.offset + T, dtype=torch.int32, device=model.device)
        H = model.cfg.hidden_size
        taps = torch.empty((T, len(layer_ids) * H), dtype=torch.bfloat16, device=model.device)
        if cache.offset + T > cache.kv.cap:
            raise ValueError("KV cache capacity exceeded")
        norm_h = model.forward(toks, pos, cache.kv, max_kv=cache.offset + T, layer_ids=list(layer_ids),
                               taps_out=taps, head="hidden").clone()
        cache.offset += T
        return norm_h[None], taps[None]

    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records=False):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids)
        logits = self.lm_head_logits(model, norm_h)
        if return_rollback_records:
            return logits, taps, {}
        return logits, taps

    def forward_verifier_states(self, model, inputs, cache, layer_ids):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids)
        return norm_h, taps, {}

    def forward_accept_all_block(self, model, inputs, cache, layer_ids):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids)
        return self.lm_head_logits(model, norm_h[:, -1:, :]), taps


class Qwen35TargetAdapter(TargetAdapter):
    """Qwen3.5 hybrid adapter (adapters.py:341-570). Differences of mechanism, same
    cache semantics: a forward that returns rollback records leaves every gated-delta
    layer's state advanced over the whole block (as the reference does) and keeps the
    per-token snapshots and the conv window on the device; ``rollback_linear_caches``
    restores snapshot ``accepted - 1`` instead of replaying the recurrence over the
    accepted prefix (adapters.py:505-560)."""

    family = "qwen3_5"

    def make_cache(self, model, cap: int = 8192, block: int = 16) -> TargetCache:
        return TargetCache(model.make_cache(1, cap, block=block))

    def _forward_states(self, model, inputs: torch.Tensor, cache: TargetCache, layer_ids, records: bool):
        toks = inputs.reshape(-1).to(model.device, torch.int32).contiguous()
        T = toks.numel()
        hc = cache.kv
        H = model.cfg.hidden_size
        if cache.offset + T > hc.cap:
            raise ValueError("KV cache capacity exceeded")
        if records and T > hc.T:
            raise ValueError(f"a block with rollback records holds at most {hc.T} tokens")
        taps = torch.empty((T, len(layer_ids) * H), dtype=torch.bfloat16, device=model.device)
        outs = []
        step = T if records else hc.Tw
        one = slice(0, 1)
        for c0 in range(0, T, step):
            c1 = min(T, c0 + step)
            n = c1 - c0
            pos = torch.arange(cache.offset + c0, cache.offset + c1, dtype=torch.int32, device=model.device)
            nrow = torch.full((1,), n, dtype=torch.int32, device=model.device)
            outs.append(model.forward(toks[c0:c1], pos, hc, max_kv=cache.offset + c1, layer_ids=list(layer_ids),
                                      taps_out=taps[c0:c1], head="hidden", seqs=one, verify=records, T=n).clone())
            if records:
                model.rollback(hc, nrow, 1, n)  # advance over the whole block; snapshots stay for rollback
                hc.last_block = n
            else:
                model.commit_prefill(hc, one, nrow, n)
        cache.offset += T
        return torch.cat(outs, 0)[None], taps[None]

    def forward_with_hidden_states(self, model, inputs, cache, layer_ids, return_rollback_records=False):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids, return_rollback_records)
        logits = self.lm_head_logits(model, norm_h)
        if return_rollback_records:
            return logits, taps, self._records(model, cache)
        return logits, taps

    def forward_verifier_states(self, model, inputs, cache, layer_ids):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids, True)
        return norm_h, taps, self._records(model, cache)

    def forward_accept_all_block(self, model, inputs, cache, layer_ids):
        norm_h, taps = self._forward_states(model, inputs, cache, layer_ids, False)
        return self.lm_head_logits(model, norm_h[:, -1:, :]), taps

    @staticmethod
    def _records(model, cache: TargetCache) -> dict:
        """Layer index -> record of the block just verified (its snapshots live in the cache)."""
        T = cache.kv.last_block
        return {l: {"block_tokens": T} for l, k in enumerate(model.kinds) if k == "gdn"}

    def snapshot_linear_caches(self, model, cache: TargetCache) -> dict:
        hc = cache.kv
        return {l: [hc.conv[gi].clone(), hc.state[gi].clone()] for l, gi in model.gdn_index.items()}

    def restore_linear_caches(self, model, cache: TargetCache, snapshots: dict) -> None:
        hc = cache.kv
        for l, (conv, state) in snapshots.items():
            gi = model.gdn_index[l]
            hc.conv[gi].copy_(conv)
            hc.state[gi].copy_(state)

    def rewind_kv_caches(self, cache: TargetCache, num_tokens: int) -> None:
        cache.trim(num_tokens)

    def rollback_linear_caches(self, model, cache: TargetCache, rollback_records: dict, accepted_inputs: int) -> None:
        if not rollback_records:
            return
        T = next(iter(rollback_records.values()))["block_tokens"]
        if not 1 <= accepted_inputs <= T:
            raise ValueError(f"accepted_inputs {accepted_inputs} outside [1, {T}]")
        acc = torch.full((1,), int(accepted_inputs), dtype=torch.int32, device=model.device)
        model.rollback(cache.kv, acc, 1, T)

    def cache_summary(self, cache: TargetCache) -> str:
        hc = cache.kv
        parts = []
        for l, k in enumerate(cache_model_kinds(hc)):
            parts.append(f"{l}:kv={cache.offset}" if k == "attn" else f"{l}:ssm={tuple(hc.state[0].shape[1:])}")
        return " ".join(parts)


def cache_model_kinds(hc) -> list[str]:
    return list(getattr(hc, "kinds", []))


ADAPTERS: dict[str, type[TargetAdapter]] = {
    "qwen3": Qwen3TargetAdapter,
    "qwen3_5": Qwen35TargetAdapter,
}


def adapter_for_model_type(model_type: str) -> type[TargetAdapter] | None:
    return ADAPTERS.get(model_type)


@dataclass
class LoadedTargetModel:
    requested_model: str
    resolved_model_path: Path | None
    model: Any
    tokenizer: Any
    adapter: TargetAdapter

    def build_prompt(self, prompt_text: str):
        return self.adapter.build_prompt(self.tokenizer, prompt_text)

    def stop_token_ids(self) -> set[int]:
        return self.adapter.stop_token_ids(self.tokenizer)

    def make_cache(self, cap: int = 8192):
        return self.adapter.make_cache(self.model, cap)

    def embed_tokens(self, tokens):
        return self.adapter.embed_tokens(self.model, tokens)

    def lm_head_logits(self, hidden_states):
        return self.adapter.lm_head_logits(self.model, hidden_states)

    def lm_head_argmax(self, hidden_states):
        return self.adapter.lm_head_argmax(self.model, hidden_states)

    def forward_with_hidden_states(self, inputs, cache, layer_ids, return_rollback_records=False):
        return self.adapter.forward_with_hidden_states(self.model, inputs, cache, layer_ids,
                                                       return_rollback_records=return_rollback_records)

    def forward_verifier_states(self, inputs, cache, layer_ids):
        return self.adapter.forward_verifier_states(self.model, inputs, cache, layer_ids)

    def forward_accept_all_block(self, inputs, cache, layer_ids):
        return self.adapter.forward_accept_all_block(self.model, inputs, cache, layer_ids)

    def snapshot_linear_caches(self, cache):
        return self.adapter.snapshot_linear_caches(self.model, cache)

    def restore_linear_caches(self, cache, snapshots):
        self.adapter.restore_linear_caches(self.model, cache, snapshots)

    def rewind_kv_caches(self, cache, num_tokens: int):
        self.adapter.rewind_kv_caches(cache, num_tokens)

    def rollback_linear_caches(self, cache, rollback_records, accepted_inputs: int):
        self.adapter.rollback_linear_caches(self.model, cache, rollback_records, accepted_inputs)

    def cache_summary(self, cache) -> str:
        return self.adapter.cache_summary(cache)


def load_target_model(path_or_spec: str | tuple, device="cuda", seed: int = 0) -> LoadedTargetModel:
    """Builds a target. ``"random:<preset>"`` (presets: tiny, qwen3-4b, tiny-hybrid,
    qwen3.5-27b) draws seeded random weights; a ``(TargetConfig, weights)`` tuple uses the
    given weights; a checkpoint directory (config.json + model*.safetensors, Hugging Face
    or MLX layout) is read by ``checkpoint.load_target_checkpoint`` (adapters.py:829-852)."""
    tok = None
    resolved = None
    if isinstance(path_or_spec, tuple):
        cfg, w = path_or_spec
        name = "custom"
    elif isinstance(path_or_spec, str) and path_or_spec.startswith("random:"):
        preset = path_or_spec.split(":", 1)[1]
        if preset not in PRESETS:
            raise ValueError(f"unknown preset {preset!r}; choose from {sorted(PRESETS)}")
        cfg = PRESETS[preset]()[0]
        w = random_target_weights(cfg, seed, device="cpu" if cfg.num_hidden_layers * cfg.hidden_size < 20000 else device)
        name = path_or_spec
    else:
        from .checkpoint import load_target_checkpoint, load_tokenizer
        cfg, w, resolved = load_target_checkpoint(path_or_spec)
        tok = load_tokenizer(resolved, cfg.vocab_size, cfg.eos_token_ids)
        name = str(path_or_spec)
    adapter_cls = adapter_for_model_type(cfg.model_type)
    if adapter_cls is None:
        registered = ", ".join(sorted(ADAPTERS))
        raise NotImplementedError(f"Unsupported DFlash target model_type={cfg.model_type!r}. Current adapters: "
                                  f"{registered}.")
    if cfg.model_type == "qwen3_5":
        from .hybrid import HybridTargetModel
        model = HybridTargetModel(cfg, w, device)
    else:
        model = TargetModel(cfg, w, device)
    tok = tok or ByteTokenizer(cfg.vocab_size, cfg.eos_token_ids)
    return LoadedTargetModel(name, resolved, model, tok, adapter_cls())
