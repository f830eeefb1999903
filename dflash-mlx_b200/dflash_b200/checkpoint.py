"""Checkpoint loading: Hugging Face / MLX safetensors directories for the targets and
the DFlash draft, into the weight dictionaries the device models take.

Follows what the reference loads:

* target: ``config.json`` (``model_type`` ``qwen3`` or ``qwen3_5``; a Qwen3.5
  multimodal config nests the text model under ``text_config``) and
  ``model*.safetensors`` (reference ``adapters.py:829-852`` through mlx-lm ``load``;
  Qwen3.5 key remapping and norm handling ``custom_qwen35_model.py:1156-1180,
  1270-1284``: vision tower dropped, ``model.language_model.`` prefix accepted, a
  Hugging Face checkpoint (conv1d stored [C, 1, K]) has zero-centred RMSNorm weights
  that are shifted by +1, the gated-delta output norm is not);
* draft: ``config.json`` with ``dflash_config.target_layer_ids`` / ``mask_token_id`` and
  ``block_size`` (``draft.py:26-66, 195, 204``) and ``model*.safetensors`` named like the
  draft module tree (``draft.py:226-238``).

Directories only: this build has no network, so hub repository ids are not fetched.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch

from .config import DraftConfig, TargetConfig


def _resolve(path_or_repo: str | Path) -> Path:
    p = Path(path_or_repo)
    if not (p / "config.json").exists():
        raise FileNotFoundError(
            f"{path_or_repo!r} is not a local checkpoint directory with a config.json (this build does not "
            "download from the Hugging Face hub)")
    return p


def _tensors(path: Path) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file
    files = sorted(path.glob("model*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no model*.safetensors in {path}")
    out: dict[str, torch.Tensor] = {}
    for f in files:
        out.update(load_file(str(f)))
    return out


def target_config_from_dict(config: dict[str, Any]) -> TargetConfig:
    """TargetConfig from a qwen3 / qwen3_5 ``config.json``."""
    model_type = config.get("model_type", "qwen3")
    text = config.get("text_config", config) if model_type == "qwen3_5" else config
    rope = text.get("rope_parameters") or text.get("rope_scaling") or {}
    H = text["hidden_size"]
    nq = text["num_attention_heads"]
    eos = config.get("eos_token_id", text.get("eos_token_id"))
    eos = tuple(eos) if isinstance(eos, list) else ((eos,) if isinstance(eos, int) else ())
    kw = dict(
        model_type=model_type, hidden_size=H, num_hidden_layers=text["num_hidden_layers"],
        num_attention_heads=nq, num_key_value_heads=text.get("num_key_value_heads", nq),
        head_dim=text.get("head_dim", H // nq), intermediate_size=text["intermediate_size"],
        vocab_size=text["vocab_size"], rms_norm_eps=text.get("rms_norm_eps", 1e-6),
        rope_theta=float(text.get("rope_theta", rope.get("rope_theta", 1e6))),
        partial_rotary_factor=float(text.get("partial_rotary_factor", rope.get("partial_rotary_factor", 1.0))),
        tie_word_embeddings=bool(config.get("tie_word_embeddings", text.get("tie_word_embeddings", False))),
        eos_token_ids=eos)
    if model_type == "qwen3_5":
        types = text.get("layer_types")
        interval = text.get("full_attention_interval", 4)
        if types:  # the interval rule of custom_qwen35_model.py:818 must describe the listed types
            full = [i for i, t in enumerate(types) if t == "full_attention"]
            interval = full[0] + 1 if full else len(types) + 1
            expect = [(i + 1) % interval == 0 for i in range(len(types))]
            if [t == "full_attention" for t in types] != expect:
                raise NotImplementedError("layer_types that are not every n-th layer full attention")
        kw.update(full_attention_interval=interval, linear_num_key_heads=text["linear_num_key_heads"],
                  linear_num_value_heads=text["linear_num_value_heads"],
                  linear_key_head_dim=text["linear_key_head_dim"],
                  linear_value_head_dim=text["linear_value_head_dim"],
                  linear_conv_kernel_dim=text.get("linear_conv_kernel_dim", 4))
    return TargetConfig(**kw)


def _strip(key: str) -> str:
    for pre in ("model.language_model.", "language_model.model.", "language_model.", "model."):
        if key.startswith(pre):
            return key[len(pre):]
    return key


def target_weights_from_tensors(cfg: TargetConfig, tensors: dict[str, torch.Tensor]) -> dict[str, Any]:
    """The device models' weight dictionary from checkpoint tensors (bf16 matrices,
    fp32 A_log / dt_bias, conv [C, 4])."""
    t = {}
    for k, v in tensors.items():
        if "visual" in k or "vision_tower" in k or k.startswith("mtp.") or ".mtp." in k:
            continue
        t[_strip(k)] = v
    hf_layout = cfg.model_type == "qwen3_5" and any(k.endswith("conv1d.weight") and v.dim() == 3 and v.shape[1] == 1
                                                    for k, v in t.items())
    bf = lambda x: x.to(torch.bfloat16).contiguous()  # noqa: E731

    def norm(x):  # Hugging Face Qwen3.5 stores (weight - 1) for these RMSNorms
        x = x.float()
        return bf(x + 1.0 if hf_layout else x)

    w: dict[str, Any] = {"embed": bf(t["embed_tokens.weight"]), "norm": norm(t["norm.weight"]), "layers": []}
    if not cfg.tie_word_embeddings:
        w["lm_head"] = bf(t["lm_head.weight"])
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        lw = {"input_layernorm": norm(t[p + "input_layernorm.weight"]),
              "post_attention_layernorm": norm(t[p + "post_attention_layernorm.weight"]),
              "gate_proj": bf(t[p + "mlp.gate_proj.weight"]), "up_proj": bf(t[p + "mlp.up_proj.weight"]),
              "down_proj": bf(t[p + "mlp.down_proj.weight"])}
        if cfg.is_linear_layer(i):
            la = p + "linear_attn."
            conv = t[la + "conv1d.weight"]
            conv = conv.reshape(conv.shape[0], -1) if conv.dim() == 3 else conv  # [C,1,K] or [C,K,1] -> [C,K]
            lw.update({"in_proj_qkv": bf(t[la + "in_proj_qkv.weight"]), "in_proj_z": bf(t[la + "in_proj_z.weight"]),
                       "in_proj_b": bf(t[la + "in_proj_b.weight"]), "in_proj_a": bf(t[la + "in_proj_a.weight"]),
                       "conv1d": bf(conv), "dt_bias": t[la + "dt_bias"].float().contiguous(),
                       "A_log": t[la + "A_log"].float().contiguous(), "norm": bf(t[la + "norm.weight"]),
                       "out_proj": bf(t[la + "out_proj.weight"])})
        else:
            sa = p + "self_attn."
            lw.update({k: bf(t[sa + k + ".weight"]) for k in ("q_proj", "k_proj", "v_proj", "o_proj")})
            lw.update({"q_norm": norm(t[sa + "q_norm.weight"]), "k_norm": norm(t[sa + "k_norm.weight"])})
        w["layers"].append(lw)
    return w


def load_target_checkpoint(path_or_repo: str | Path) -> tuple[TargetConfig, dict[str, Any], Path]:
    path = _resolve(path_or_repo)
    cfg = target_config_from_dict(json.loads((path / "config.json").read_text()))
    return cfg, target_weights_from_tensors(cfg, _tensors(path)), path


def load_draft_checkpoint(path_or_repo: str | Path) -> tuple[DraftConfig, dict[str, Any], Path]:
    """A DFlash draft directory (draft.py:226-238)."""
    path = _resolve(path_or_repo)
    cfg = DraftConfig.from_dict(json.loads((path / "config.json").read_text()))
    t = {(k[len("model."):] if k.startswith("model.") else k): v for k, v in _tensors(path).items()}
    bf = lambda x: x.to(torch.bfloat16).contiguous()  # noqa: E731
    w: dict[str, Any] = {"fc": bf(t["fc.weight"]), "hidden_norm": bf(t["hidden_norm.weight"]),
                         "norm": bf(t["norm.weight"]), "layers": []}
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        w["layers"].append({
            "input_layernorm": bf(t[p + "input_layernorm.weight"]),
            "post_attention_layernorm": bf(t[p + "post_attention_layernorm.weight"]),
            **{k: bf(t[p + "self_attn." + k + ".weight"]) for k in ("q_proj", "k_proj", "v_proj", "o_proj",
                                                                    "q_norm", "k_norm")},
            **{k: bf(t[p + "mlp." + k + ".weight"]) for k in ("gate_proj", "up_proj", "down_proj")},
        })
    return cfg, w, path


def load_tokenizer(path: Path, vocab_size: int, eos: tuple[int, ...]):
    """The checkpoint's tokenizer when its files are present, else a byte tokenizer."""
    if any((path / f).exists() for f in ("tokenizer.json", "tokenizer_config.json", "vocab.json")):
        try:
            from transformers import AutoTokenizer
            tok = AutoTokenizer.from_pretrained(str(path))
            if not hasattr(tok, "eos_token_ids"):
                tok.eos_token_ids = list(eos) or ([tok.eos_token_id] if tok.eos_token_id is not None else [])
            return tok
        except Exception as exc:  # unusable tokenizer files: say so, then fall back to bytes
            import warnings
            warnings.warn(f"tokenizer files in {path} could not be loaded ({exc}); using a byte tokenizer",
                          RuntimeWarning, stacklevel=2)
    from .adapters import ByteTokenizer
    return ByteTokenizer(vocab_size, eos)
