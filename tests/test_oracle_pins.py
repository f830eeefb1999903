"""Pins the CPU oracle to the reference: golden fixtures produced by running the
reference's own runtime.py / adapters.py / custom_qwen35_model.py (see
tests/golden/make_golden.py), plus a cross-check of the model mathematics
against transformers' Qwen3 and Qwen3-Next implementations."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import dflash_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def tiny():
    from dflash_b200.config import tiny_pair
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    tw, dw = random_target_weights(tcfg, 0), random_draft_weights(dcfg, 0)
    ot = O.OracleTarget(tcfg, tw)
    return tcfg, dcfg, ot, O.OracleDraft(dcfg, dw, ot)


@pytest.fixture(scope="module")
def runtime_fx():
    with open(os.path.join(GOLD, "runtime_loop.json")) as f:
        return json.load(f)


def test_oracle_trace_is_reproducible(tiny, runtime_fx):
    tcfg, dcfg, ot, od = tiny
    prompt = runtime_fx["prompt"]
    trace = O.plain_greedy(ot, prompt, len(runtime_fx["trace"]) - len(prompt))
    assert trace == runtime_fx["trace"]


@pytest.mark.parametrize("case", ["real_draft", "injected", "injected_stream", "injected_chunked", "injected_stop",
                                  "injected_short", "injected_spec4", "zero_new", "one_new"])
def test_oracle_loop_matches_reference_runtime(tiny, runtime_fx, case):
    """The oracle's decode loop reproduces the reference dflash_generate (run on the
    same oracle models) token for token, with the same acceptance lengths."""
    tcfg, dcfg, ot, od = tiny
    c = next(x for x in runtime_fx["cases"] if x["name"] == case)
    inj = None
    if c["injected"]:
        inj = O.Injection(runtime_fx["trace"] + [0] * (4 * dcfg.block_size), runtime_fx["inject_lengths"],
                          runtime_fx["inject_noise"])
    bs = dcfg.block_size if c["speculative_tokens"] is None else max(1, min(c["speculative_tokens"],
                                                                          dcfg.block_size))
    out, accs = O.spec_generate(ot, od, runtime_fx["prompt"], c["max_new_tokens"], bs, set(c["stops"]), inj)
    assert out == c["output_tokens"]
    assert accs == c["acceptance_lengths"]


def test_lossless_property_in_reference_runs(runtime_fx):
    """Every reference run's output is a prefix of the plain greedy trace."""
    trace = runtime_fx["trace"]
    for c in runtime_fx["cases"]:
        out = c["output_tokens"]
        assert out == trace[:len(out)], c["name"]


def test_gdr_snapshot_restore_equals_reference_replay():
    """State after `a` accepted tokens from the per-token snapshots equals the
    reference's rollback replay (custom_qwen35_model.py:1029-1074 ->
    advance_gated_delta_states fp32 loop); the conv state equals the last K-1 rows
    of concat(initial_conv_state, qkv[:a])."""
    fx = np.load(os.path.join(GOLD, "gdr_rollback.npz"))
    n_layers, T = int(fx["meta"][0]), int(fx["meta"][1])
    for l in range(n_layers):
        g = lambda k: torch.from_numpy(fx[f"l{l}_{k}"])  # noqa: E731
        _, snaps, final = O.gdr_recurrence(g("q"), g("k"), g("v"), g("g"), g("beta"), g("initial_state"))
        for acc in (1, 3, T):
            ref_state = fx[f"acc{acc}_l{l}_state"]
            got = snaps[:, acc - 1].numpy()
            np.testing.assert_allclose(got, ref_state, rtol=1e-5, atol=1e-6)
            conv = torch.cat([g("initial_conv_state"), g("qkv")[:, :acc]], 1)[:, -3:].numpy()
            np.testing.assert_array_equal(conv, fx[f"acc{acc}_l{l}_conv"])
    _, _, final0 = O.gdr_recurrence(*(torch.from_numpy(fx[f"l0_{k}"]) for k in ("q", "k", "v", "g", "beta",
                                                                                 "initial_state")))
    np.testing.assert_allclose(final0.numpy(), fx["replay_full"], rtol=1e-5, atol=1e-6)


def test_gdr_matches_transformers_recurrence():
    """Cross-check against transformers' torch_recurrent_gated_delta_rule (qwen3_next):
    log-decay g, state [Dk, Dv], q scaled by Dk^-1/2 inside."""
    tr = pytest.importorskip("transformers.models.qwen3_next.modeling_qwen3_next")
    gen = torch.Generator().manual_seed(5)
    B, T, H, D = 1, 7, 4, 16
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1)
    v = torch.randn(B, T, H, D, generator=gen)
    logg = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    S0 = torch.randn(B, H, D, D, generator=gen) * 0.1  # [Dk, Dv] in transformers
    o_t, S_t = tr.torch_recurrent_gated_delta_rule(q, k, v, logg, beta, S0, True)
    o_o, _, S_o = O.gdr_recurrence(q * D ** -0.5, k, v, torch.exp(logg), beta, S0.transpose(-1, -2))
    torch.testing.assert_close(o_o, o_t, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(S_o.transpose(-1, -2), S_t, rtol=1e-4, atol=1e-5)


def test_qwen3_layers_match_transformers():
    """The restated mlx-lm qwen3 forward agrees with transformers' Qwen3Model on the
    same (bf16) weights: final hidden states within bf16 tolerance."""
    tq = pytest.importorskip("transformers.models.qwen3.modeling_qwen3")
    from transformers import Qwen3Config
    from dflash_b200.config import tiny_pair
    from dflash_b200.weights import random_target_weights
    tcfg, _ = tiny_pair()
    w = random_target_weights(tcfg, 11, std=0.05)
    hf_cfg = Qwen3Config(vocab_size=tcfg.vocab_size, hidden_size=tcfg.hidden_size,
                         intermediate_size=tcfg.intermediate_size, num_hidden_layers=tcfg.num_hidden_layers,
                         num_attention_heads=tcfg.num_attention_heads, num_key_value_heads=tcfg.num_key_value_heads,
                         head_dim=tcfg.head_dim, rms_norm_eps=tcfg.rms_norm_eps, rope_theta=tcfg.rope_theta,
                         max_position_embeddings=4096, tie_word_embeddings=True, attention_bias=False)
    hf_cfg._attn_implementation = "eager"
    model = tq.Qwen3Model(hf_cfg).eval()
    sd = {"embed_tokens.weight": w["embed"], "norm.weight": w["norm"]}
    names = {"input_layernorm": "input_layernorm", "post_attention_layernorm": "post_attention_layernorm",
             "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
             "o_proj": "self_attn.o_proj", "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm",
             "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}
    for i, lw in enumerate(w["layers"]):
        for k, hk in names.items():
            sd[f"layers.{i}.{hk}.weight"] = lw[k]
    model.load_state_dict({k: v.float() for k, v in sd.items()}, strict=False)
    g = torch.Generator().manual_seed(1)
    toks = torch.randint(0, tcfg.vocab_size, (1, 24), generator=g)
    with torch.no_grad():
        hf = model(toks).last_hidden_state[0]
    ot = O.OracleTarget(tcfg, w)
    ours, _ = ot.forward_states(toks[0].tolist(), ot.make_cache(), [])
    err = (ours - hf).abs().max().item()
    assert err < 0.05 * hf.abs().max().item(), err


def test_qwen35_hybrid_layers_match_transformers(monkeypatch):
    """The restated hybrid stack (GDN layers + gated partial-RoPE attention) agrees with
    transformers' Qwen3_5TextModel on the same weights, with the oracle's bf16
    roundings switched off so that the comparison is of the mathematics (fp32 both
    sides, 1e-3 relative). transformers keeps the
    zero-centred RMSNorm weights (applies 1 + w); the mlx checkpoint layout the
    reference loads stores them shifted, so the oracle's w maps to w - 1 there."""
    tq = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.weights import random_target_weights
    tcfg, _ = tiny_hybrid_pair()
    w = random_target_weights(tcfg, 12, std=0.05)
    hf_cfg = Qwen3_5TextConfig(
        vocab_size=tcfg.vocab_size, hidden_size=tcfg.hidden_size, intermediate_size=tcfg.intermediate_size,
        num_hidden_layers=tcfg.num_hidden_layers, num_attention_heads=tcfg.num_attention_heads,
        num_key_value_heads=tcfg.num_key_value_heads, head_dim=tcfg.head_dim, rms_norm_eps=tcfg.rms_norm_eps,
        linear_key_head_dim=tcfg.linear_key_head_dim, linear_value_head_dim=tcfg.linear_value_head_dim,
        linear_num_key_heads=tcfg.linear_num_key_heads, linear_num_value_heads=tcfg.linear_num_value_heads,
        layer_types=["linear_attention" if tcfg.is_linear_layer(i) else "full_attention"
                     for i in range(tcfg.num_hidden_layers)],
        rope_parameters={"rope_type": "default", "rope_theta": tcfg.rope_theta,
                         "partial_rotary_factor": tcfg.partial_rotary_factor})
    hf_cfg._attn_implementation = "eager"
    model = tq.Qwen3_5TextModel(hf_cfg).eval()
    sd = {"embed_tokens.weight": w["embed"], "norm.weight": w["norm"].float() - 1}
    for i, lw in enumerate(w["layers"]):
        p = f"layers.{i}."
        sd[p + "input_layernorm.weight"] = lw["input_layernorm"].float() - 1
        sd[p + "post_attention_layernorm.weight"] = lw["post_attention_layernorm"].float() - 1
        for k in ("gate_proj", "up_proj", "down_proj"):
            sd[p + f"mlp.{k}.weight"] = lw[k]
        if tcfg.is_linear_layer(i):
            for k in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj", "A_log", "dt_bias"):
                sd[p + f"linear_attn.{k}" + ("" if k in ("A_log", "dt_bias") else ".weight")] = lw[k]
            sd[p + "linear_attn.conv1d.weight"] = lw["conv1d"][:, None, :]
            sd[p + "linear_attn.norm.weight"] = lw["norm"]
        else:
            for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
                sd[p + f"self_attn.{k}.weight"] = lw[k]
            sd[p + "self_attn.q_norm.weight"] = lw["q_norm"].float() - 1
            sd[p + "self_attn.k_norm.weight"] = lw["k_norm"].float() - 1
    missing = set(model.state_dict()) - set(sd)
    assert not missing, missing
    model.load_state_dict({k: v.float() for k, v in sd.items()})
    g = torch.Generator().manual_seed(1)
    toks = torch.randint(0, tcfg.vocab_size, (1, 24), generator=g)
    with torch.no_grad():
        hf = model(toks).last_hidden_state[0]
    monkeypatch.setattr(O, "bf16", lambda x: x.float())
    ot = O.OracleHybridTarget(tcfg, w)
    ours, _ = ot.forward_states(toks[0].tolist(), ot.make_cache(), [])
    err = (ours - hf).abs().max().item()
    assert err < 1e-3 * hf.abs().max().item(), err


def test_hybrid_oracle_spec_is_lossless():
    """Hybrid oracle decode loop with injected drafts (snapshot rollback of every GDN
    layer after each partial accept) reproduces its plain greedy decode."""
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_hybrid_pair()
    ot = O.OracleHybridTarget(tcfg, random_target_weights(tcfg, 0, std=0.05))
    od = O.OracleDraft(dcfg, random_draft_weights(dcfg, 0), ot)
    od.mask_mode = "causal"
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, tcfg.vocab_size, (24,), generator=g).tolist()
    bs = dcfg.block_size
    trace = O.plain_greedy(ot, prompt, 24 + 3 * bs)
    lens = torch.randint(0, bs, (40,), generator=g).tolist()
    noise = torch.randint(0, tcfg.vocab_size, (40, bs), generator=g).tolist()
    out, accs = O.spec_generate(ot, od, prompt, 24, bs, set(), O.Injection(trace + [0] * 4 * bs, lens, noise))
    assert out == trace[:len(out)]
    assert len(out) >= len(prompt) + 24
    assert any(1 < a < bs for a in accs)


@pytest.mark.parametrize("mode", ["none", "causal"])
def test_oracle_draft_matches_reference_draft(monkeypatch, mode):
    """The oracle's DFlash draft forward equals the reference's own DFlashDraftModel
    (draft.py:68-223, run on numpy restatements of its mlx layers by
    tests/golden/make_golden.py) over three cached calls, mask none and causal
    (fp32: the oracle's bf16 roundings switched off; 1e-5 relative)."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import draft_fixture_config
    from dflash_b200.weights import random_draft_weights
    monkeypatch.setattr(O, "bf16", lambda x: x.float())
    fx = np.load(os.path.join(GOLD, "draft_forward.npz"))
    dcfg = draft_fixture_config()
    od = O.OracleDraft(dcfg, random_draft_weights(dcfg, int(fx["meta"][1]), std=0.05), None)
    od.mask_mode = mode
    cache = od.make_cache(256)
    for i in range(int(fx["meta"][0])):
        noise = torch.from_numpy(fx[f"call{i}_noise"][0]).float()
        hidden = torch.from_numpy(fx[f"call{i}_hidden"][0]).float()
        got = od(noise, hidden, cache)
        ref = torch.from_numpy(fx[f"{mode}_call{i}_out"][0]).float()
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
        for c in cache:
            c.trim(noise.shape[0])


def test_oracle_hybrid_layers_match_reference(monkeypatch):
    """The oracle's gated-delta layer and gated full-attention layer equal the reference's
    own forward_linear_layer_explicit_with_record / forward_full_attention_layer_explicit
    (custom_qwen35_model.py:409-540, run under the numpy shim by
    tests/golden/make_golden.py): layer output, new conv state, new recurrent state, new
    keys / values (fp32; 1e-5)."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import hybrid_fixture_weights
    monkeypatch.setattr(O, "bf16", lambda x: x.float())
    fx = np.load(os.path.join(GOLD, "hybrid_layers.npz"))
    cfg, w = hybrid_fixture_weights()
    ot = O.OracleHybridTarget(cfg, w)
    t = lambda k: torch.from_numpy(fx[k]).float()  # noqa: E731
    cache = ot.make_cache(64)
    g0 = cache[0]
    g0.conv, g0.state = t("gdn_conv0")[0], t("gdn_state0")[0]
    h = ot.gdn_layer(w["layers"][0], t("gdn_in")[0], g0)
    torch.testing.assert_close(h, t("gdn_out")[0], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(g0.conv, t("gdn_conv1")[0], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(g0.state, t("gdn_state1")[0], rtol=1e-5, atol=1e-6)
    offset, T = int(fx["meta"][2]), int(fx["meta"][1])
    kv = cache[3]
    kv.k[:, :offset] = t("attn_k0")[0]
    kv.v[:, :offset] = t("attn_v0")[0]
    kv.offset = offset
    h = ot.attn_layer(w["layers"][3], t("attn_in")[0], torch.arange(offset, offset + T), kv)
    torch.testing.assert_close(h, t("attn_out")[0], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(kv.k[:, offset:offset + T], t("attn_k1")[0], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(kv.v[:, offset:offset + T], t("attn_v1")[0], rtol=1e-5, atol=1e-5)
