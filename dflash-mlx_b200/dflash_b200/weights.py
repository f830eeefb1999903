"""Weights of the target and draft in their natural (checkpoint) layout.

Names follow the checkpoint keys the reference loads (mlx-lm qwen3 and the
DFlash draft, draft.py:75-223): ``q_proj``/``k_proj``/``v_proj``/``o_proj`` are
[out, in] matrices, norms are vectors, ``embed`` is [vocab, hidden] and is also
the tied lm_head (adapters.py:606-609). Random initialisation is N(0, std) from a
seeded CPU generator, so the same seed gives the same bf16 weights on any
machine; norm weights are ones (the nn.RMSNorm initial value).

The GPU model (``model.py``) repacks these into its own HBM layout; the CPU
oracle used by the tests reads them as they are.
"""
from __future__ import annotations

from typing import Any

import torch

from .config import DraftConfig, TargetConfig


def _randn(gen: torch.Generator, shape, std: float, device: str) -> torch.Tensor:
    if device == "cpu":
        return (torch.randn(shape, generator=gen, dtype=torch.float32) * std).to(torch.bfloat16)
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    # fill in slabs to bound the fp32 temporary
    flat = out.view(-1)
    step = 1 << 26
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = (torch.randn(n, generator=gen, dtype=torch.float32, device=device) * std).to(torch.bfloat16)
    return out


def _ones(n: int, device: str) -> torch.Tensor:
    return torch.ones(n, dtype=torch.bfloat16, device=device)


def random_target_weights(cfg: TargetConfig, seed: int, std: float = 0.02, device: str = "cpu",
                          layer_hook=None) -> dict[str, Any]:
    """Seeded N(0, std) target weights. device='cuda' draws them on the GPU (large models).
    ``layer_hook(i, layer_weights) -> layer_weights`` transforms each layer as soon as it is
    drawn (a tensor-parallel rank keeps only its shard: one full layer is live at a time)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    H, hd = cfg.hidden_size, cfg.head_dim
    w: dict[str, Any] = {"embed": _randn(gen, (cfg.vocab_size, H), std, device), "norm": _ones(H, device), "layers": []}
    for i in range(cfg.num_hidden_layers):
        lw: dict[str, torch.Tensor] = {
            "input_layernorm": _ones(H, device),
            "post_attention_layernorm": _ones(H, device),
            "gate_proj": _randn(gen, (cfg.intermediate_size, H), std, device),
            "up_proj": _randn(gen, (cfg.intermediate_size, H), std, device),
            "down_proj": _randn(gen, (H, cfg.intermediate_size), std, device),
        }
        if cfg.is_linear_layer(i):
            kd = cfg.linear_key_head_dim * cfg.linear_num_key_heads
            vd = cfg.linear_value_head_dim * cfg.linear_num_value_heads
            hv = cfg.linear_num_value_heads
            lw.update({
                "in_proj_qkv": _randn(gen, (2 * kd + vd, H), std, device),
                "in_proj_z": _randn(gen, (vd, H), std, device),
                "in_proj_b": _randn(gen, (hv, H), std, device),
                "in_proj_a": _randn(gen, (hv, H), std, device),
                "conv1d": _randn(gen, (2 * kd + vd, cfg.linear_conv_kernel_dim), 0.2, device),
                "dt_bias": torch.ones(hv, dtype=torch.float32, device=device),
                "A_log": torch.log(torch.linspace(1.0, 16.0, hv, dtype=torch.float32, device=device)),
                "norm": _ones(cfg.linear_value_head_dim, device),
                "out_proj": _randn(gen, (H, vd), std, device),
            })
        else:
            qmul = 2 if cfg.model_type == "qwen3_5" else 1  # qwen3_5 q_proj also emits the output gate
            lw.update({
                "q_proj": _randn(gen, (qmul * cfg.num_attention_heads * hd, H), std, device),
                "k_proj": _randn(gen, (cfg.num_key_value_heads * hd, H), std, device),
                "v_proj": _randn(gen, (cfg.num_key_value_heads * hd, H), std, device),
                "o_proj": _randn(gen, (H, cfg.num_attention_heads * hd), std, device),
                "q_norm": _ones(hd, device),
                "k_norm": _ones(hd, device),
            })
        w["layers"].append(layer_hook(i, lw) if layer_hook is not None else lw)
    return w


def random_draft_weights(cfg: DraftConfig, seed: int, std: float = 0.02, device: str = "cpu") -> dict[str, Any]:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 7919)
    H, hd = cfg.hidden_size, cfg.head_dim
    n_taps = len(cfg.target_layer_ids)
    w: dict[str, Any] = {
        "fc": _randn(gen, (H, n_taps * H), std, device),
        "hidden_norm": _ones(H, device),
        "norm": _ones(H, device),
        "layers": [],
    }
    for _ in range(cfg.num_hidden_layers):
        w["layers"].append({
            "input_layernorm": _ones(H, device),
            "post_attention_layernorm": _ones(H, device),
            "q_proj": _randn(gen, (cfg.num_attention_heads * hd, H), std, device),
            "k_proj": _randn(gen, (cfg.num_key_value_heads * hd, H), std, device),
            "v_proj": _randn(gen, (cfg.num_key_value_heads * hd, H), std, device),
            "o_proj": _randn(gen, (H, cfg.num_attention_heads * hd), std, device),
            "q_norm": _ones(hd, device),
            "k_norm": _ones(hd, device),
            "gate_proj": _randn(gen, (cfg.intermediate_size, H), std, device),
            "up_proj": _randn(gen, (cfg.intermediate_size, H), std, device),
            "down_proj": _randn(gen, (H, cfg.intermediate_size), std, device),
        })
    return w


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F,H] gate and up -> [2F,H] packed per 64 rows as [32 gate | 32 up] (DFL_EPI_SILU_MUL)."""
    F, H = gate.shape
    if F % 32:
        raise ValueError("intermediate size must be a multiple of 32")
    g = gate.reshape(F // 32, 32, H)
    u = up.reshape(F // 32, 32, H)
    return torch.stack([g, u], dim=1).reshape(2 * F, H).contiguous()


def rope_inv_freq(rot_dim: int, theta: float, device="cpu") -> torch.Tensor:
    """inv_freq[i] = theta^(-2i/rot_dim), fp32 (non-interleaved RoPE, traditional=False)."""
    exps = torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim
    return (1.0 / (theta ** exps)).to(torch.float32).to(device)
