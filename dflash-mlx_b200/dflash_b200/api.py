"""Public API with the reference's signatures (dflash_mlx/api.py:21-212)."""
from __future__ import annotations

from collections.abc import Iterator
from dataclasses import dataclass
from pathlib import Path
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


@dataclass
class DraftCheckpoint:
    """A DFlash draft as loaded, before it is placed on a target's device: its config,
    its weights in checkpoint layout and the draft contract fields the runtime reads
    (draft.py:190-223). ``bind(target)`` builds the GPU draft, which shares the target's
    embedding and lm_head as the reference's draft does."""
    cfg: Any
    weights: dict
    attention_mask_mode: str = "none"

    @property
    def block_size(self) -> int:
        return self.cfg.block_size

    @property
    def mask_token_id(self) -> int:
        return self.cfg.mask_token_id

    @property
    def target_layer_ids(self) -> list[int]:
        return list(self.cfg.target_layer_ids)

    def bind(self, target) -> DraftModel:
        model = target.model if isinstance(target, LoadedTargetModel) else target
        return DraftModel(self.cfg, self.weights, model, mask_mode=self.attention_mask_mode)


def load_draft_model(path_or_repo, seed: int = 0) -> tuple[DraftCheckpoint, Any]:
    """Reference signature and return (draft.py:224-236): ``(draft, model_path)``.
    ``path_or_repo`` is a DFlash draft checkpoint directory (config.json +
    model*.safetensors; local only, there is no network here), ``"random:<preset>"``
    (seeded random weights of a preset's shape) or a ``(DraftConfig, weights)`` tuple. The
    draft is placed on the GPU by ``DFlashGenerator`` (or ``draft.bind(target)``), because
    it reads the target's embedding."""
    if isinstance(path_or_repo, tuple):
        cfg, w = path_or_repo
        return DraftCheckpoint(cfg, w), None
    if isinstance(path_or_repo, str) and path_or_repo.startswith("random:"):
        cfg = PRESETS[path_or_repo.split(":", 1)[1]]()[1]
        return DraftCheckpoint(cfg, random_draft_weights(cfg, seed)), path_or_repo
    from .checkpoint import load_draft_checkpoint
    cfg, w, path = load_draft_checkpoint(path_or_repo)
    return DraftCheckpoint(cfg, w), Path(path)


QUANT_BITS = (2, 3, 4, 5, 6, 8)
QUANT_GROUPS = (32, 64, 128)


def quantize_dequantize(w: torch.Tensor, bits: int, group_size: int) -> torch.Tensor:
    """Affine group quantization of a [N, K] weight, returned dequantized (bf16): per group
    of ``group_size`` consecutive inputs, scale = (max - min) / (2^bits - 1) and
    bias = min, q = round((w - bias) / scale) clamped to [0, 2^bits - 1], w' = q * scale +
    bias, with scale and bias stored in bf16. This is the published affine scheme behind
    the reference's ``quantize_model`` of the draft (draft.py:239-252, api.py:62-66): the
    draft then computes with w'. The weights stay bf16 in HBM (no packed low-bit GEMM)."""
    N, K = w.shape
    if K % group_size:
        raise ValueError(f"input dimension {K} is not a multiple of the group size {group_size}")
    x = w.float().reshape(N, K // group_size, group_size)
    lo, hi = x.amin(-1, keepdim=True), x.amax(-1, keepdim=True)
    levels = (1 << bits) - 1
    scale = ((hi - lo) / levels).to(torch.bfloat16).float()
    bias = lo.to(torch.bfloat16).float()
    safe = torch.where(scale > 0, scale, torch.ones_like(scale))
    q = torch.clamp(torch.round((x - bias) / safe), 0, levels)
    return (q * scale + bias).reshape(N, K).to(torch.bfloat16)


def maybe_quantize_draft_model(draft: DraftCheckpoint, bits: int | None, group_size: int) -> dict | None:
    """draft.py:239-252: quantize every projection of the draft (fc, q/k/v/o, gate/up/down;
    the draft owns no embedding) and return the quantization record ``{"group_size",
    "bits"}``, or None when ``bits`` is None."""
    if bits is None:
        return None
    if bits not in QUANT_BITS:
        raise ValueError(f"draft_quant_bits must be one of {QUANT_BITS}")
    if group_size not in QUANT_GROUPS:
        raise ValueError(f"draft_quant_group_size must be one of {QUANT_GROUPS}")
    w = dict(draft.weights)
    w["fc"] = quantize_dequantize(w["fc"], bits, group_size)
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    w["layers"] = [{k: (quantize_dequantize(v, bits, group_size) if k in names else v) for k, v in lw.items()}
                   for lw in w["layers"]]
    draft.weights = w
    return {"group_size": group_size, "bits": bits}


class DFlashGenerator:
    def __init__(self, target_model=DEFAULT_TARGET_MODEL, draft_model=DEFAULT_DRAFT_MODEL,
                 draft_attention_mask: str = "auto", draft_quant_bits: int | None = None,
                 draft_quant_group_size: int = 64, seed: int = 0, device: str = "cuda"):
        torch.manual_seed(seed)
        self.seed = int(seed)  # default sampling seed of generate / stream
        self.requested_target_model = target_model
        self.requested_draft_model = draft_model
        self.target: LoadedTargetModel = (target_model if isinstance(target_model, LoadedTargetModel)
                                          else load_target_model(target_model, device=device, seed=seed))
        if draft_attention_mask == "auto":
            draft_attention_mask = "causal" if self.target.adapter.family == "qwen3_5" else "none"
        self.draft_attention_mask = draft_attention_mask
        if isinstance(draft_model, DraftModel):
            self.draft, self.draft_path = draft_model, None
            self.draft_quantization = None
            if draft_quant_bits is not None:
                raise ValueError("draft_quant_bits needs a draft checkpoint or spec, not a built DraftModel")
        else:
            ckpt, self.draft_path = load_draft_model(draft_model, seed=seed)
            ckpt.attention_mask_mode = draft_attention_mask
            self.draft_quantization = maybe_quantize_draft_model(ckpt, draft_quant_bits, draft_quant_group_size)
            self.draft = ckpt.bind(self.target)
        self.draft.mask_mode = draft_attention_mask

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
