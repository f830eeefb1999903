"""Model configurations of the target / draft pairs this build runs.

Field names follow the checkpoint ``config.json`` keys that the reference reads:
the target's ``TextModelArgs`` / mlx-lm ``qwen3.ModelArgs`` and the draft's
``DraftArgs`` (dflash_mlx/draft.py:26-66, with ``dflash_config.target_layer_ids``
and ``mask_token_id`` at draft.py:195, 204).
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict
from typing import Any


@dataclass
class TargetConfig:
    model_type: str = "qwen3"  # "qwen3" or "qwen3_5" (hybrid gated-delta)
    hidden_size: int = 2560
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    partial_rotary_factor: float = 1.0
    tie_word_embeddings: bool = True
    # qwen3_5 hybrid fields (custom_qwen35_model.py:637-696)
    full_attention_interval: int = 4
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 48
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    eos_token_ids: tuple[int, ...] = ()

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def is_linear_layer(self, idx: int) -> bool:
        """GDN layer test of custom_qwen35_model.py:818 ((i+1) % interval != 0)."""
        if self.model_type != "qwen3_5":
            return False
        return (idx + 1) % self.full_attention_interval != 0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass
class DraftConfig:
    hidden_size: int = 2560
    num_hidden_layers: int = 5
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    block_size: int = 16
    target_layer_ids: list[int] = field(default_factory=lambda: [1, 9, 17, 25, 33])
    mask_token_id: int = 151669

    @classmethod
    def from_dict(cls, config: dict[str, Any]) -> "DraftConfig":
        """Reads a DFlash draft ``config.json`` (draft.py:46-66, 195, 204)."""
        dcfg = config.get("dflash_config") or {}
        return cls(
            hidden_size=config["hidden_size"],
            num_hidden_layers=config["num_hidden_layers"],
            num_attention_heads=config["num_attention_heads"],
            num_key_value_heads=config["num_key_value_heads"],
            head_dim=config.get("head_dim", config["hidden_size"] // config["num_attention_heads"]),
            intermediate_size=config["intermediate_size"],
            vocab_size=config["vocab_size"],
            rms_norm_eps=config.get("rms_norm_eps", 1e-6),
            rope_theta=config.get("rope_theta", 1e6),
            block_size=config.get("block_size", 16),
            target_layer_ids=list(dcfg["target_layer_ids"]),
            mask_token_id=int(dcfg["mask_token_id"]),
        )


def evenly_spaced_layers(num_layers: int, n: int) -> list[int]:
    """n tap layers spread over the depth, ascending (the DFlash draft convention)."""
    if n == 1:
        return [num_layers // 2]
    start, end = 1, num_layers - 3
    return [int(round(start + i * (end - start) / (n - 1))) for i in range(n)]


# ---------------------------------------------------------------------------
# Presets: the benchmark configurations (random-init, seeded)
# ---------------------------------------------------------------------------
def tiny_pair() -> tuple[TargetConfig, DraftConfig]:
    """Config 1: 4 layers, hidden 256, 4 q / 2 kv heads of 64, FFN 768, vocab 4096;
    draft of 1 layer conditioned on target layers 1 and 3, block 8."""
    t = TargetConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                     head_dim=64, intermediate_size=768, vocab_size=4096)
    d = DraftConfig(hidden_size=256, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
                    head_dim=64, intermediate_size=768, vocab_size=4096, block_size=8,
                    target_layer_ids=[1, 3], mask_token_id=4095)
    return t, d


def qwen3_4b_pair() -> tuple[TargetConfig, DraftConfig]:
    """Config 3/4: Qwen3-4B shape; DFlash draft of 5 layers, block 16, 5 taps."""
    t = TargetConfig()
    d = DraftConfig(target_layer_ids=evenly_spaced_layers(36, 5))
    return t, d


def qwen3_4b_small_pair(num_layers: int = 4, draft_layers: int = 1) -> tuple[TargetConfig, DraftConfig]:
    """Full-width Qwen3-4B layers at reduced depth (parity tests against the CPU oracle)."""
    t = TargetConfig(num_hidden_layers=num_layers)
    taps = [1, num_layers - 1] if num_layers >= 3 else [num_layers - 1]
    d = DraftConfig(num_hidden_layers=draft_layers, target_layer_ids=taps)
    return t, d


def tiny_hybrid_pair() -> tuple[TargetConfig, DraftConfig]:
    """Tiny Qwen3.5-style hybrid: 4 layers (GDN, GDN, GDN, gated attention), hidden 256,
    attention 4 q / 2 kv heads of 256 with RoPE on the first 64 dims, GDN 2 key heads /
    4 value heads of 64, FFN 768, vocab 4096; draft of 1 layer on target layers 1 and 3."""
    t = TargetConfig(model_type="qwen3_5", hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                     num_key_value_heads=2, head_dim=256, partial_rotary_factor=0.25, intermediate_size=768,
                     vocab_size=4096, linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64,
                     linear_value_head_dim=64)
    d = DraftConfig(hidden_size=256, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
                    head_dim=64, intermediate_size=768, vocab_size=4096, block_size=8,
                    target_layer_ids=[1, 3], mask_token_id=4095)
    return t, d


def qwen35_27b_pair(num_layers: int = 64) -> tuple[TargetConfig, DraftConfig]:
    """Config 5: Qwen3.5-27B shape (64 layers, every 4th gated full attention 24 q / 4 kv
    heads of 256 with partial RoPE 0.25; 48 GDN layers of 16 key / 48 value heads of 128;
    hidden 5120, FFN 17408, vocab 151936); DFlash draft of 5 layers, block 16.
    ``num_layers`` < 64 gives the same widths at reduced depth (parity tests)."""
    t = TargetConfig(model_type="qwen3_5", hidden_size=5120, num_hidden_layers=num_layers, num_attention_heads=24,
                     num_key_value_heads=4, head_dim=256, partial_rotary_factor=0.25, intermediate_size=17408,
                     vocab_size=151936, linear_num_key_heads=16,
                     linear_num_value_heads=48, linear_key_head_dim=128, linear_value_head_dim=128)
    n_taps = 5 if num_layers >= 8 else 2
    d = DraftConfig(hidden_size=5120, num_hidden_layers=5 if num_layers >= 8 else 1, num_attention_heads=32,
                    num_key_value_heads=8, head_dim=128, intermediate_size=17408, vocab_size=151936,
                    target_layer_ids=evenly_spaced_layers(num_layers, n_taps) if num_layers >= 8
                    else [1, num_layers - 1])
    return t, d


PRESETS = {
    "tiny": tiny_pair,
    "qwen3-4b": qwen3_4b_pair,
    "tiny-hybrid": tiny_hybrid_pair,
    "qwen3.5-27b": qwen35_27b_pair,
}
