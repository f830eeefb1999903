"""Public API with the reference's signatures (dflash_mlx/api.py:21-212)."""
from __future__ import annotations

from collections.abc import Iterator
from dataclasses import dataclass
from typing import Any

import torch

from .adapters import LoadedTargetModel, load_target_model
from .config import PRESETS
from .model import DraftModel
from .runtime import dflash_generate, dflash_generate_stream
from .weights import random_draft_weights

DEFAULT_TARGET_MODEL = "random:qwen3-4b"
DEFAULT_DRAFT_MODEL = "random:qwen3-4b"


@dataclass
class DFlashResult:
    text: str
    output_tokens: list[int]
    generated_tokens: list[int]
    metrics: dict[str, Any]


@dataclass
class DFlashStreamEvent:
    delta: str
    text: str
    token_ids: list[int]
    output_tokens: list[int]
    generated_tokens: list[int]
    metrics: dict[str, Any] | None = None
    finished: bool = False


def load_draft_model(spec, target: LoadedTargetModel, seed: int = 0, mask_mode: str = "none") -> DraftModel:
    """``"random:<preset>"``, a ``(DraftConfig, weights)`` tuple, or a DFlash draft checkpoint
    directory (config.json + model*.safetensors, draft.py:226-238)."""
    if isinstance(spec, DraftModel):
        return spec
    if isinstance(spec, tuple):
        cfg, w = spec
    elif isinstance(spec, str) and spec.startswith("random:"):
        cfg = PRESETS[spec.split(":", 1)[1]]()[1]
        w = random_draft_weights(cfg, seed)
    else:
        from .checkpoint import load_draft_checkpoint
        cfg, w, _ = load_draft_checkpoint(spec)
    return DraftModel(cfg, w, target.model, mask_mode=mask_mode)


class DFlashGenerator:
    def __init__(self, target_model=DEFAULT_TARGET_MODEL, draft_model=DEFAULT_DRAFT_MODEL,
                 draft_attention_mask: str = "auto", draft_quant_bits: int | None = None,
                 draft_quant_group_size: int = 64, seed: int = 0, device: str = "cuda"):
        if draft_quant_bits is not None:
            raise NotImplementedError("draft quantisation is not part of this build")
        torch.manual_seed(seed)
        self.seed = int(seed)  # default sampling seed of generate / stream
        self.requested_target_model = target_model
        self.requested_draft_model = draft_model
        self.target: LoadedTargetModel = (target_model if isinstance(target_model, LoadedTargetModel)
                                          else load_target_model(target_model, device=device, seed=seed))
        if draft_attention_mask == "auto":
            draft_attention_mask = "causal" if self.target.adapter.family == "qwen3_5" else "none"
        self.draft_attention_mask = draft_attention_mask
        self.draft = load_draft_model(draft_model, self.target, seed=seed, mask_mode=draft_attention_mask)
        self.draft.mask_mode = draft_attention_mask
        self.draft_quantization = None

    @property
    def target_model_path(self):
        return self.target.resolved_model_path

    def encode_prompt(self, prompt_text: str):
        return self.target.build_prompt(prompt_text)

    def generate_from_tokens(self, prompt_tokens, max_new_tokens: int = 256, temperature: float = 0.0,
                             speculative_tokens: int | None = None, verify_mode: str = "parallel-replay",
                             verify_chunk_size: int = 4, reset_peak_memory: bool = True,
                             skip_special_tokens: bool = False, profile: bool = False,
                             seed: int | None = None) -> DFlashResult:
        if reset_peak_memory:
            torch.cuda.reset_peak_memory_stats(self.target.model.device)
        output_tokens, metrics = dflash_generate(
            target=self.target.model, draft=self.draft, prompt_tokens=prompt_tokens, max_new_tokens=max_new_tokens,
            temperature=temperature, stop_token_ids=self.target.stop_token_ids(),
            layer_ids=self.draft.target_layer_ids, speculative_tokens=speculative_tokens, verify_mode=verify_mode,
            verify_chunk_size=verify_chunk_size, profile=profile,
            seed=self.seed if seed is None else seed)
        generated = output_tokens[metrics["num_input_tokens"]:]
        text = self.target.tokenizer.decode(generated, skip_special_tokens=skip_special_tokens)
        return DFlashResult(text=text, output_tokens=output_tokens, generated_tokens=generated, metrics=metrics)

    def stream_from_tokens(self, prompt_tokens, max_new_tokens: int = 256, temperature: float = 0.0,
                           speculative_tokens: int | None = None, verify_mode: str = "parallel-replay",
                           verify_chunk_size: int = 4, reset_peak_memory: bool = True,
                           skip_special_tokens: bool = False, profile: bool = False,
                           seed: int | None = None) -> Iterator[DFlashStreamEvent]:
        """Incremental detokenisation as in api.py:116-164."""
        prompt_len = int(len(prompt_tokens))
        decoded = ""
        if reset_peak_memory and torch.cuda.is_available():
            torch.cuda.reset_peak_memory_stats(self.target.model.device)
        for event in dflash_generate_stream(
                target=self.target.model, draft=self.draft, prompt_tokens=prompt_tokens,
                max_new_tokens=max_new_tokens, temperature=temperature, stop_token_ids=self.target.stop_token_ids(),
                layer_ids=self.draft.target_layer_ids, speculative_tokens=speculative_tokens, verify_mode=verify_mode,
                verify_chunk_size=verify_chunk_size, profile=profile, seed=self.seed if seed is None else seed):
            generated = event.output_tokens[prompt_len:]
            text = self.target.tokenizer.decode(generated, skip_special_tokens=skip_special_tokens)
            delta = text[len(decoded):] if text.startswith(decoded) else text
            decoded = text
            yield DFlashStreamEvent(delta=delta, text=text, token_ids=list(event.token_ids),
                                    output_tokens=list(event.output_tokens), generated_tokens=list(generated),
                                    metrics=event.metrics, finished=event.finished)

    def generate(self, prompt_text: str, **kw) -> DFlashResult:
        return self.generate_from_tokens(prompt_tokens=self.encode_prompt(prompt_text), **kw)

    def stream(self, prompt_text: str, **kw) -> Iterator[DFlashStreamEvent]:
        return self.stream_from_tokens(prompt_tokens=self.encode_prompt(prompt_text), **kw)
