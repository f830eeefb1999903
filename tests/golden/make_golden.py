"""Generates the golden fixtures under tests/golden/ by running the REFERENCE's own
Python code (dflash_mlx/runtime.py, adapters.py, custom_qwen35_model.py from the
read-only reference tree) under the numpy stand-in for mlx (oracle/refshim.py).

Run in the build container (the reference tree is not present on GPU boxes):

    python tests/golden/make_golden.py /path/to/reference

Fixtures:
  runtime_loop.json   reference dflash_generate outputs / acceptance lengths for the
                      tiny config-1 pair (weights regenerated from their seeds), with
                      the real draft and with injected drafts, several verify modes,
                      stop tokens and length limits;
  gdr_rollback.npz    reference advance_gated_delta_states (adapters.py:93-135) and
                      Qwen3_5TextModel.rollback_linear_caches
                      (custom_qwen35_model.py:1029-1074) on seeded random records;
  draft_forward.npz   reference DFlashDraftModel (draft.py:68-223), 2 layers of the
                      tiny draft width with seeded random weights, run over three
                      calls with its KV cache (context appended, block trimmed as the
                      runtime does at runtime.py:420), mask none and causal;
  hybrid_layers.npz   reference forward_linear_layer_explicit_with_record and
                      forward_full_attention_layer_explicit (custom_qwen35_model.py:
                      409-540) on a gated-delta and a gated-attention layer of the tiny
                      hybrid with seeded random weights, states and cached keys.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "dflash-mlx_b200"))

from oracle import dflash_oracle as O  # noqa: E402
from oracle import refshim  # noqa: E402
from dflash_b200.config import tiny_pair  # noqa: E402
from dflash_b200.weights import random_draft_weights, random_target_weights  # noqa: E402

SENTINEL = -1.0e6


class FakeTarget:
    """LoadedTargetModel-shaped wrapper over the oracle target (numpy in/out)."""

    def __init__(self, ot: O.OracleTarget, stops: set[int]):
        self.ot = ot
        self.stops = stops
        self.rewinds: list[int] = []

    def make_cache(self):
        return self.ot.make_cache()

    def stop_token_ids(self):
        return set(self.stops)

    def embed_tokens(self, tokens):
        return self.ot.embed_tokens(np.asarray(tokens).reshape(-1).tolist()).numpy()[None]

    def lm_head_logits(self, hidden):
        h = torch.from_numpy(np.asarray(hidden, dtype=np.float32))
        V = self.ot.cfg.vocab_size
        flat = h.reshape(-1, h.shape[-1])
        out = torch.empty((flat.shape[0], V))
        for i, row in enumerate(flat):
            if row[0] <= SENTINEL / 2:  # injected draft proposal: one-hot logits
                out[i] = 0.0
                out[i, int(round(SENTINEL - float(row[0])))] = 1.0
            else:
                out[i] = self.ot.lm_head_logits(row[None])[0]
        return out.reshape(*h.shape[:-1], V).numpy()

    def forward_with_hidden_states(self, inputs, cache, layer_ids, return_rollback_records=False):
        toks = np.asarray(inputs).reshape(-1).tolist()
        logits, taps = self.ot.forward_with_hidden_states(toks, cache, layer_ids)
        res = (logits.numpy()[None], taps.numpy()[None])
        return (*res, {}) if return_rollback_records else res

    def snapshot_linear_caches(self, cache):
        return {}

    def restore_linear_caches(self, cache, snapshots):
        return None

    def rewind_kv_caches(self, cache, n):
        self.rewinds.append(int(n))
        for c in cache:
            c.trim(n)

    def rollback_linear_caches(self, cache, records, accepted):
        return None

    def cache_summary(self, cache):
        return " ".join(f"{i}:kv={c.offset}" for i, c in enumerate(cache))


class FakeDraft:
    """DFlashDraftModel-shaped wrapper over the oracle draft; optionally injects proposals."""

    def __init__(self, od: O.OracleDraft, inject: O.Injection | None):
        self.od = od
        self.inject = inject
        self.step = 0
        self.block_size = od.block_size
        self.mask_token_id = od.mask_token_id
        self.target_layer_ids = list(od.cfg.target_layer_ids)

    def make_cache(self):
        return self.od.make_cache()

    def __call__(self, noise_embedding, target_hidden, cache):
        start = cache[0].offset + int(np.asarray(target_hidden).shape[1])
        h = self.od(torch.from_numpy(np.asarray(noise_embedding[0], dtype=np.float32)),
                    torch.from_numpy(np.asarray(target_hidden[0], dtype=np.float32)), cache).numpy()[None]
        if self.inject is not None:
            L = self.inject.lengths[self.step]
            for i in range(1, h.shape[1]):
                tok = self.inject.trace[start + i] if i - 1 < L else self.inject.noise[self.step][i]
                h[0, i, :] = 0.0
                h[0, i, 0] = SENTINEL - tok
        self.step += 1
        return h


def run_reference(rt, ot, od, prompt, max_new, stops, inject, mode, spec_tokens=None):
    target = FakeTarget(ot, stops)
    draft = FakeDraft(od, inject)
    out, metrics = rt.dflash_generate(target=target, draft=draft, prompt_tokens=np.array(prompt, dtype=np.uint32),
                                      max_new_tokens=max_new, temperature=0.0, stop_token_ids=set(stops),
                                      layer_ids=draft.target_layer_ids, speculative_tokens=spec_tokens,
                                      verify_mode=mode, verify_chunk_size=3)
    return [int(t) for t in out], [int(a) for a in metrics["acceptance_lengths"]], target.rewinds


def make_runtime_fixture(ref_root: str) -> dict:
    rt = refshim.import_reference(ref_root, ("runtime",))["runtime"]
    tcfg, dcfg = tiny_pair()
    tw, dw = random_target_weights(tcfg, 0), random_draft_weights(dcfg, 0)
    ot = O.OracleTarget(tcfg, tw)
    od = O.OracleDraft(dcfg, dw, ot)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, tcfg.vocab_size, (64,), generator=g).tolist()
    max_new = 48
    trace = O.plain_greedy(ot, prompt, max_new + 3 * dcfg.block_size)
    bs = dcfg.block_size
    steps = max_new + 2
    lengths = torch.randint(0, bs, (steps,), generator=g).tolist()
    noise = torch.randint(0, tcfg.vocab_size, (steps, bs), generator=g).tolist()
    inj = O.Injection(trace + [0] * (4 * bs), lengths, noise)
    cases = []
    stop_mid = trace[len(prompt) + 20]
    for name, stops, inject, mode, mn, spec in [
        ("real_draft", [], None, "parallel-replay", max_new, None),
        ("injected", [], inj, "parallel-replay", max_new, None),
        ("injected_stream", [], inj, "stream", max_new, None),
        ("injected_chunked", [], inj, "chunked", max_new, None),
        ("injected_stop", [stop_mid], inj, "parallel-replay", max_new, None),
        ("injected_short", [], inj, "parallel-replay", 5, None),
        ("injected_spec4", [], inj, "parallel-replay", max_new, 4),
        ("zero_new", [], None, "parallel-replay", 0, None),
        ("one_new", [], inj, "parallel-replay", 1, None),
    ]:
        out, accs, rewinds = run_reference(rt, ot, od, prompt, mn, stops, inject, mode, spec)
        cases.append({"name": name, "stops": stops, "injected": inject is not None, "verify_mode": mode,
                      "max_new_tokens": mn, "speculative_tokens": spec, "output_tokens": out,
                      "acceptance_lengths": accs, "kv_rewinds": rewinds})
    return {"seed_target": 0, "seed_draft": 0, "prompt": prompt, "trace": trace, "inject_lengths": lengths,
            "inject_noise": noise, "cases": cases}


def make_gdr_fixture(ref_root: str) -> dict:
    mods = refshim.import_reference(ref_root, ("adapters", "custom_qwen35_model"))
    adv = mods["adapters"].advance_gated_delta_states
    model_cls = mods["custom_qwen35_model"].Qwen3_5TextModel
    rng = np.random.default_rng(1)
    n_layers, T, Hk, Hv, Dk, Dv, conv_dim = 3, 6, 2, 4, 16, 16, 40
    out: dict[str, np.ndarray] = {}
    recs = {}
    for l in range(n_layers):
        q = rng.standard_normal((1, T, Hk, Dk)).astype(np.float32)
        k = rng.standard_normal((1, T, Hk, Dk)).astype(np.float32)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((1, T, Hv, Dv)).astype(np.float32)
        gl = np.exp(-np.log1p(np.exp(rng.standard_normal((1, T, Hv))))).astype(np.float32)
        beta = (1 / (1 + np.exp(-rng.standard_normal((1, T, Hv))))).astype(np.float32)
        s0 = (rng.standard_normal((1, Hv, Dv, Dk)) * 0.1).astype(np.float32)
        conv0 = rng.standard_normal((1, 3, conv_dim)).astype(np.float32)
        qkv = rng.standard_normal((1, T, conv_dim)).astype(np.float32)
        recs[l] = {"initial_conv_state": conv0, "initial_state": s0, "qkv": qkv, "k": k, "v": v, "g": gl,
                   "beta": beta, "repeat_factor": Hv // Hk}
        for key, val in recs[l].items():
            if key != "repeat_factor":
                out[f"l{l}_{key}"] = val
        out[f"l{l}_q"] = q
    for acc in (1, 3, T):
        cache = [[None, None] for _ in range(n_layers)]
        model_cls.rollback_linear_caches(None, cache, recs, acc)
        for l in range(n_layers):
            out[f"acc{acc}_l{l}_conv"] = np.asarray(cache[l][0])
            out[f"acc{acc}_l{l}_state"] = np.asarray(cache[l][1])
    # direct call of the replay kernel's CPU branch on the full block
    ks = np.repeat(recs[0]["k"], Hv // Hk, axis=2)
    out["replay_full"] = np.asarray(adv(recs[0]["initial_state"], ks, recs[0]["v"], recs[0]["g"], recs[0]["beta"]))
    out["meta"] = np.array([n_layers, T, Hk, Hv, Dk, Dv, conv_dim])
    return out


def draft_fixture_config():
    """The draft geometry of draft_forward.npz: the tiny draft width with 2 layers."""
    from dflash_b200.config import DraftConfig
    return DraftConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=64, intermediate_size=768, vocab_size=4096, block_size=8, target_layer_ids=[1, 3],
                       mask_token_id=4095)


def make_draft_fixture(ref_root: str) -> dict:
    draft_mod = refshim.import_reference(ref_root, ("draft",))["draft"]
    dcfg = draft_fixture_config()
    dw = random_draft_weights(dcfg, 6, std=0.05)
    f64 = lambda t: t.double().numpy()  # noqa: E731
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(6)
    calls = [(24, 8), (5, 8), (3, 8)]  # (context rows appended, block rows) per call
    for mode in ("none", "causal"):
        args = draft_mod.DraftArgs(model_type="qwen3", hidden_size=dcfg.hidden_size,
                                   num_hidden_layers=dcfg.num_hidden_layers,
                                   intermediate_size=dcfg.intermediate_size,
                                   num_attention_heads=dcfg.num_attention_heads, rms_norm_eps=dcfg.rms_norm_eps,
                                   vocab_size=dcfg.vocab_size, num_key_value_heads=dcfg.num_key_value_heads,
                                   max_position_embeddings=4096, rope_theta=dcfg.rope_theta, head_dim=dcfg.head_dim,
                                   tie_word_embeddings=True, block_size=dcfg.block_size,
                                   dflash_config={"target_layer_ids": dcfg.target_layer_ids,
                                                  "mask_token_id": dcfg.mask_token_id})
        model = draft_mod.DFlashDraftModel(args)
        model.attention_mask_mode = mode
        model.fc.weight, model.hidden_norm.weight, model.norm.weight = f64(dw["fc"]), f64(dw["hidden_norm"]), \
            f64(dw["norm"])
        for layer, lw in zip(model.layers, dw["layers"]):
            a = layer.self_attn
            a.q_proj.weight, a.k_proj.weight, a.v_proj.weight = f64(lw["q_proj"]), f64(lw["k_proj"]), f64(lw["v_proj"])
            a.o_proj.weight, a.q_norm.weight, a.k_norm.weight = f64(lw["o_proj"]), f64(lw["q_norm"]), f64(lw["k_norm"])
            layer.mlp.gate_proj.weight, layer.mlp.up_proj.weight = f64(lw["gate_proj"]), f64(lw["up_proj"])
            layer.mlp.down_proj.weight = f64(lw["down_proj"])
            layer.input_layernorm.weight = f64(lw["input_layernorm"])
            layer.post_attention_layernorm.weight = f64(lw["post_attention_layernorm"])
        cache = model.make_cache()
        for i, (ctx, bs) in enumerate(calls):
            if mode == "none":
                out[f"call{i}_noise"] = rng.standard_normal((1, bs, dcfg.hidden_size)) * 0.5
                out[f"call{i}_hidden"] = rng.standard_normal((1, ctx, 2 * dcfg.hidden_size)) * 0.5
            h = model(out[f"call{i}_noise"], out[f"call{i}_hidden"], cache)
            out[f"{mode}_call{i}_out"] = np.asarray(h)
            for c in cache:  # the runtime trims the block rows after each proposal (runtime.py:420)
                c.trim(bs)
    out["meta"] = np.array([len(calls), 6])
    return out


def hybrid_fixture_weights():
    """The tiny hybrid's seeded random weights of hybrid_layers.npz (non-trivial norms)."""
    from dflash_b200.config import tiny_hybrid_pair
    cfg, _ = tiny_hybrid_pair()
    w = random_target_weights(cfg, 7, std=0.05)
    g = torch.Generator().manual_seed(7)
    for lw in w["layers"]:
        for k in ("input_layernorm", "post_attention_layernorm", "q_norm", "k_norm", "norm"):
            if k in lw:
                lw[k] = (1 + 0.2 * torch.randn(lw[k].shape, generator=g)).to(torch.bfloat16)
    return cfg, w


def make_hybrid_layer_fixture(ref_root: str) -> dict:
    from types import SimpleNamespace
    cq = refshim.import_reference(ref_root, ("custom_qwen35_model",))["custom_qwen35_model"]
    nn = sys.modules["mlx.nn"]
    qn = sys.modules["mlx_lm.models.qwen3_next"]
    q3 = sys.modules["mlx_lm.models.qwen3"]
    rope_utils = sys.modules["mlx_lm.models.rope_utils"]
    cfg, w = hybrid_fixture_weights()
    f64 = lambda t: t.double().numpy()  # noqa: E731
    H, T = cfg.hidden_size, 12
    Hk, Hv, Dk, Dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, \
        cfg.linear_value_head_dim
    kd, vd = Hk * Dk, Hv * Dv
    C = 2 * kd + vd

    def lin(wt):
        m = nn.Linear(wt.shape[1], wt.shape[0], bias=False)
        m.weight = f64(wt)
        return m

    def norm(wt, eps=cfg.rms_norm_eps):
        m = nn.RMSNorm(wt.shape[0], eps=eps)
        m.weight = f64(wt)
        return m

    def mlp(lw):
        m = q3.MLP(H, cfg.intermediate_size)
        m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight = f64(lw["gate_proj"]), f64(lw["up_proj"]), \
            f64(lw["down_proj"])
        return m

    rng = np.random.default_rng(7)
    out: dict[str, np.ndarray] = {}
    # gated-delta layer 0
    lw = w["layers"][0]
    conv = nn.Conv1d(C, C, 4, groups=C)
    conv.weight = f64(lw["conv1d"])[:, :, None]
    gnorm = qn.Qwen3NextRMSNormGated(Dv, eps=cfg.rms_norm_eps)
    gnorm.weight = f64(lw["norm"])
    linear = SimpleNamespace(in_proj_qkv=lin(lw["in_proj_qkv"]), in_proj_z=lin(lw["in_proj_z"]),
                             in_proj_b=lin(lw["in_proj_b"]), in_proj_a=lin(lw["in_proj_a"]), conv1d=conv,
                             norm=gnorm, out_proj=lin(lw["out_proj"]), num_v_heads=Hv, num_k_heads=Hk,
                             head_v_dim=Dv, head_k_dim=Dk, key_dim=kd, value_dim=vd, conv_kernel_size=4,
                             A_log=f64(lw["A_log"]), dt_bias=f64(lw["dt_bias"]), training=False)
    layer = SimpleNamespace(linear_attn=linear, input_layernorm=norm(lw["input_layernorm"]),
                            post_attention_layernorm=norm(lw["post_attention_layernorm"]), mlp=mlp(lw))
    out["gdn_in"] = rng.standard_normal((1, T, H))
    out["gdn_conv0"] = rng.standard_normal((1, 3, C)) * 0.5
    out["gdn_state0"] = rng.standard_normal((1, Hv, Dv, Dk)) * 0.1
    res = cq.forward_linear_layer_explicit_with_record(layer, out["gdn_in"], None, out["gdn_conv0"],
                                                       out["gdn_state0"])
    out["gdn_out"], out["gdn_conv1"], out["gdn_state1"] = (np.asarray(x) for x in res[:3])
    # gated full-attention layer 3 against 20 cached (post-RoPE) keys
    lw = w["layers"][3]
    hd, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    attn = SimpleNamespace(q_proj=lin(lw["q_proj"]), k_proj=lin(lw["k_proj"]), v_proj=lin(lw["v_proj"]),
                           o_proj=lin(lw["o_proj"]), q_norm=norm(lw["q_norm"]), k_norm=norm(lw["k_norm"]),
                           num_attention_heads=Hq, num_key_value_heads=Hkv, scale=hd ** -0.5,
                           rope=rope_utils.initialize_rope(cfg.rope_dim, base=cfg.rope_theta, traditional=False))
    layer = SimpleNamespace(self_attn=attn, input_layernorm=norm(lw["input_layernorm"]),
                            post_attention_layernorm=norm(lw["post_attention_layernorm"]), mlp=mlp(lw))
    offset = 20
    out["attn_in"] = rng.standard_normal((1, T, H))
    out["attn_k0"] = rng.standard_normal((1, Hkv, offset, hd))
    out["attn_v0"] = rng.standard_normal((1, Hkv, offset, hd))
    h, nk, nv = cq.forward_full_attention_layer_explicit(layer, out["attn_in"], out["attn_k0"], out["attn_v0"], offset)
    out["attn_out"], out["attn_k1"], out["attn_v1"] = np.asarray(h), np.asarray(nk), np.asarray(nv)
    out["meta"] = np.array([7, T, offset])
    return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DFLASH_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <reference tree> (or set DFLASH_REFERENCE_ROOT)")
    fx = make_runtime_fixture(ref_root)
    with open(os.path.join(HERE, "runtime_loop.json"), "w") as f:
        json.dump(fx, f)
    np.savez_compressed(os.path.join(HERE, "gdr_rollback.npz"), **make_gdr_fixture(ref_root))
    np.savez_compressed(os.path.join(HERE, "draft_forward.npz"), **make_draft_fixture(ref_root))
    np.savez_compressed(os.path.join(HERE, "hybrid_layers.npz"), **make_hybrid_layer_fixture(ref_root))
    print("wrote runtime_loop.json, gdr_rollback.npz, draft_forward.npz, hybrid_layers.npz")


if __name__ == "__main__":
    main()
