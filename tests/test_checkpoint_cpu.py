"""Checkpoint loading (CPU): Hugging Face-layout safetensors directories written from
seeded random weights load back into the device models' weight dictionaries — Qwen3
target, Qwen3.5 hybrid target (zero-centred norms shifted by +1, conv1d [C, 1, K]) in
both the bare and the multimodal key layouts, and the DFlash draft."""
import json

import pytest
import torch

safetensors = pytest.importorskip("safetensors.torch")


def _save(path, tensors, config):
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(config))
    safetensors.save_file({k: v.contiguous() for k, v in tensors.items()}, str(path / "model.safetensors"))


def _hf_target(cfg, w, prefix, shift):
    t = {prefix + "embed_tokens.weight": w["embed"], prefix + "norm.weight": w["norm"].float() - shift}
    for i, lw in enumerate(w["layers"]):
        p = f"{prefix}layers.{i}."
        t[p + "input_layernorm.weight"] = lw["input_layernorm"].float() - shift
        t[p + "post_attention_layernorm.weight"] = lw["post_attention_layernorm"].float() - shift
        for k in ("gate_proj", "up_proj", "down_proj"):
            t[p + f"mlp.{k}.weight"] = lw[k]
        if "q_proj" in lw:
            for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
                t[p + f"self_attn.{k}.weight"] = lw[k]
            t[p + "self_attn.q_norm.weight"] = lw["q_norm"].float() - shift
            t[p + "self_attn.k_norm.weight"] = lw["k_norm"].float() - shift
        else:
            for k in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj", "norm"):
                t[p + f"linear_attn.{k}.weight"] = lw[k]
            t[p + "linear_attn.conv1d.weight"] = lw["conv1d"][:, None, :]
            t[p + "linear_attn.dt_bias"] = lw["dt_bias"]
            t[p + "linear_attn.A_log"] = lw["A_log"]
    return t


def _same(a, b):
    assert a.shape == b.shape, (a.shape, b.shape)
    assert torch.equal(a.float(), b.float())


def _check(w, got):
    _same(w["embed"], got["embed"])
    _same(w["norm"], got["norm"])
    for lw, gl in zip(w["layers"], got["layers"]):
        assert set(lw) == set(gl)
        for k in lw:
            _same(lw[k], gl[k])


def test_qwen3_checkpoint_roundtrip(tmp_path):
    from dflash_b200.checkpoint import load_target_checkpoint
    from dflash_b200.config import tiny_pair
    from dflash_b200.weights import random_target_weights
    cfg, _ = tiny_pair()
    w = random_target_weights(cfg, 3)
    config = {"model_type": "qwen3", "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_hidden_layers,
              "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
              "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate_size, "vocab_size": cfg.vocab_size,
              "rms_norm_eps": 1e-6, "rope_theta": 1e6, "tie_word_embeddings": True, "eos_token_id": 7}
    _save(tmp_path / "q3", _hf_target(cfg, w, "model.", 0.0), config)
    got_cfg, got, path = load_target_checkpoint(tmp_path / "q3")
    assert got_cfg == cfg.__class__(**{**cfg.__dict__, "eos_token_ids": (7,)})
    _check(w, got)


@pytest.mark.parametrize("prefix,multimodal", [("model.", False), ("model.language_model.", True)])
def test_qwen35_hf_checkpoint_roundtrip(tmp_path, prefix, multimodal):
    from dflash_b200.checkpoint import load_target_checkpoint
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.weights import random_target_weights
    cfg, _ = tiny_hybrid_pair()
    w = random_target_weights(cfg, 4)
    for lw in w["layers"]:  # non-trivial norm weights: the +1 shift must be exact in bf16
        for k in ("input_layernorm", "post_attention_layernorm"):
            lw[k] = (1 + 0.25 * torch.randint(-2, 3, lw[k].shape)).to(torch.bfloat16)
    text = {"hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_hidden_layers,
            "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
            "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate_size, "vocab_size": cfg.vocab_size,
            "rms_norm_eps": 1e-6, "rope_parameters": {"rope_theta": 1e6, "partial_rotary_factor": 0.25},
            "linear_num_key_heads": cfg.linear_num_key_heads, "linear_num_value_heads": cfg.linear_num_value_heads,
            "linear_key_head_dim": cfg.linear_key_head_dim, "linear_value_head_dim": cfg.linear_value_head_dim,
            "layer_types": ["linear_attention"] * 3 + ["full_attention"]}
    config = {"model_type": "qwen3_5", "tie_word_embeddings": True,
              **({"text_config": text} if multimodal else text)}
    tensors = _hf_target(cfg, w, prefix, 1.0)
    if multimodal:
        tensors["model.visual.patch_embed.weight"] = torch.zeros(4, 4)
    _save(tmp_path / "q35", tensors, config)
    got_cfg, got, _ = load_target_checkpoint(tmp_path / "q35")
    assert got_cfg.model_type == "qwen3_5" and got_cfg.rope_dim == cfg.rope_dim
    assert [got_cfg.is_linear_layer(i) for i in range(4)] == [True, True, True, False]
    _check(w, got)


def test_draft_checkpoint_roundtrip(tmp_path):
    from dflash_b200.checkpoint import load_draft_checkpoint
    from dflash_b200.config import tiny_pair
    from dflash_b200.weights import random_draft_weights
    _, dcfg = tiny_pair()
    dw = random_draft_weights(dcfg, 5)
    t = {"fc.weight": dw["fc"], "hidden_norm.weight": dw["hidden_norm"], "norm.weight": dw["norm"]}
    for i, lw in enumerate(dw["layers"]):
        p = f"layers.{i}."
        t[p + "input_layernorm.weight"] = lw["input_layernorm"]
        t[p + "post_attention_layernorm.weight"] = lw["post_attention_layernorm"]
        for k in ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"):
            t[p + f"self_attn.{k}.weight"] = lw[k]
        for k in ("gate_proj", "up_proj", "down_proj"):
            t[p + f"mlp.{k}.weight"] = lw[k]
    config = {"hidden_size": dcfg.hidden_size, "num_hidden_layers": dcfg.num_hidden_layers,
              "num_attention_heads": dcfg.num_attention_heads, "num_key_value_heads": dcfg.num_key_value_heads,
              "head_dim": dcfg.head_dim, "intermediate_size": dcfg.intermediate_size,
              "vocab_size": dcfg.vocab_size, "block_size": dcfg.block_size,
              "dflash_config": {"target_layer_ids": dcfg.target_layer_ids, "mask_token_id": dcfg.mask_token_id}}
    _save(tmp_path / "d", t, config)
    got_cfg, got, _ = load_draft_checkpoint(tmp_path / "d")
    assert got_cfg == dcfg
    for k in ("fc", "hidden_norm", "norm"):
        _same(dw[k], got[k])
    for lw, gl in zip(dw["layers"], got["layers"]):
        for k in lw:
            _same(lw[k], gl[k])


def test_missing_directory_is_reported(tmp_path):
    from dflash_b200.checkpoint import load_target_checkpoint
    with pytest.raises(FileNotFoundError):
        load_target_checkpoint(tmp_path / "nope")
