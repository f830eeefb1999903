"""Parity at the benchmark configurations' full depth and width.

The yardstick is the oracle's own rounding sensitivity. Residual values reach |h| ~ 40 at
Qwen3-4B depth (a bf16 ulp of 0.25) and logits reach 5-6 (an ulp of 0.03), so an absolute
bound of 2e-2 is below bf16 resolution there; what a correct bf16 kernel must meet is
"no further from the oracle than the oracle's bf16 arithmetic is from its own fp32
arithmetic on the same inputs" (d_gpu = |gpu - oracle|, d_ref = |oracle_fp32 - oracle|:
mean d_gpu <= mean d_ref, and every element's d_gpu <= 1.5 max d_ref or within one bf16
ulp of the larger of the two values).

* Qwen3-4B (config 3), all 36 layers, teacher forced: every GPU layer is fed the oracle's
  input (a 48-row prefill, then a 16-row verify block over the cached prefix); then the
  lm_head on the oracle's final hidden states; then the free-running 36-layer forward
  end to end (greedy tokens agree with the oracle's on >= 90 % of rows).
* Qwen3.5-27B width (config 5), per gated-delta layer fed the oracle's input: the
  recurrence on the oracle's own q, k, v, g, beta is within 1e-3 relative on the fp32
  state (north_star's bound); the whole layer (bf16 projections in front of it) meets
  the sensitivity yardstick on its output and its state.
"""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp(x: torch.Tensor) -> torch.Tensor:
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.pow(2.0, e - 7)


def _within(got: torch.Tensor, ref: torch.Tensor, ulps: int, tol: float = 2e-2) -> tuple[bool, float, float]:
    d = (got.float() - ref.float()).abs()
    ok = bool(((d <= tol) | (d <= ulps * _ulp(ref))).all())
    return ok, d.max().item(), d.mean().item()


def _cpu_weights(cfg, seed):
    """Seeded weights drawn on the GPU (fast at billions of parameters) and copied to the
    host for the oracle; the GPU models are built from the same host tensors."""
    from dflash_b200.weights import random_target_weights
    w = random_target_weights(cfg, seed, device=DEV)
    out = {k: v.cpu() for k, v in w.items() if k != "layers"}
    out["layers"] = [{k: v.cpu() for k, v in lw.items()} for lw in w["layers"]]
    del w
    torch.cuda.empty_cache()
    return out


def _vs_sensitivity(got: torch.Tensor, ref: torch.Tensor, ref32: torch.Tensor):
    """(ok, max d_gpu, mean d_gpu, max d_ref, mean d_ref): the yardstick of the module
    docstring."""
    d = (got.float() - ref.float()).abs()
    r = (ref32.float() - ref.float()).abs()
    # one ulp in the larger binade of the two values (a rounding that crosses a power of two)
    ulp = _ulp(torch.maximum(got.float().abs(), ref.float().abs()))
    ok = bool(d.mean() <= r.mean()) and bool((d <= torch.clamp(ulp, min=1.5 * r.max())).all())
    return bool(ok), d.max().item(), d.mean().item(), r.max().item(), r.mean().item()


def _oracle_layer_inputs(ot, prompt, block):
    """Runs the oracle layer by layer over the prefill and then the block (one KV cache
    per layer); returns, for both passes, the residual stream entering every layer (and
    leaving the last) and the logits."""
    from oracle import dflash_oracle as O
    c = ot.cfg
    cache = ot.make_cache(len(prompt) + len(block) + 8)
    outs = []
    for toks, start in ((prompt, 0), (block, len(prompt))):
        pos = torch.arange(start, start + len(toks))
        h = ot.embed_tokens(toks)
        hs = [h]
        for l in range(c.num_hidden_layers):
            h = ot.layer(l, h, pos, cache[l])
            hs.append(h)
        logits = ot.lm_head_logits(O.rms_norm(h, ot.w["norm"], c.rms_norm_eps))
        outs.append((hs, logits))
    return outs


def test_qwen3_4b_36_layers_teacher_forced_and_end_to_end(monkeypatch):
    from oracle import dflash_oracle as O
    from dflash_b200.config import qwen3_4b_pair
    from dflash_b200.model import TargetModel
    tcfg, _ = qwen3_4b_pair()
    tw = _cpu_weights(tcfg, 2)
    g = torch.Generator().manual_seed(2)
    P, T = 48, 16
    prompt = torch.randint(0, tcfg.vocab_size, (P,), generator=g).tolist()
    block = torch.randint(0, tcfg.vocab_size, (T,), generator=g).tolist()
    ot = O.OracleTarget(tcfg, tw)
    (hs_p, lg_p), (hs_b, lg_b) = _oracle_layer_inputs(ot, prompt, block)
    H = tcfg.hidden_size
    i32 = dict(dtype=torch.int32, device=DEV)

    # the fp32 oracle on the same (bf16) layer inputs: the oracle's own rounding sensitivity
    with monkeypatch.context() as mp:
        mp.setattr(O, "bf16", lambda x: x.float())
        c32 = ot.make_cache(P + T + 8)
        out32 = [(ot.layer(l, hs_p[l], torch.arange(P), c32[l]), ot.layer(l, hs_b[l], torch.arange(P, P + T), c32[l]))
                 for l in range(tcfg.num_hidden_layers)]
        fin = torch.cat([hs_p[-1], hs_b[-1]], 0)
        lm32 = ot.lm_head_logits(O.rms_norm(fin, ot.w["norm"], tcfg.rms_norm_eps))

    # --- teacher-forced per layer ---------------------------------------------------
    one = dataclasses.replace(tcfg, num_hidden_layers=1, vocab_size=P + T)
    bad = []
    for l in range(tcfg.num_hidden_layers):
        rows = torch.cat([hs_p[l], hs_b[l]], 0).to(torch.bfloat16)
        m = TargetModel(one, {"embed": rows, "norm": tw["norm"], "layers": [tw["layers"][l]]}, DEV)
        cache = m.make_cache(1, P + T)
        tp = torch.empty((P, H), dtype=torch.bfloat16, device=DEV)
        tb = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
        m.forward(torch.arange(P, **i32), torch.arange(P, **i32), cache, max_kv=P, layer_ids=[0], taps_out=tp,
                  head="hidden")
        m.forward(torch.arange(P, P + T, **i32), torch.arange(P, P + T, **i32), cache, max_kv=P + T,
                  layer_ids=[0], taps_out=tb, head="hidden")
        for what, got, ref, r32 in (("prefill", tp, hs_p[l + 1], out32[l][0]), ("block", tb, hs_b[l + 1], out32[l][1])):
            ok, mx, mean, rmx, rmean = _vs_sensitivity(got.cpu(), ref, r32)
            if l % 6 == 0 or not ok:
                print(f"layer {l} {what}: gpu vs oracle max {mx:.4f} mean {mean:.2e}; oracle fp32 vs bf16 max "
                      f"{rmx:.4f} mean {rmean:.2e}")
            if not ok:
                bad.append((l, what, mx, mean, rmx, rmean))
        del m, cache

    # --- lm_head on the oracle's final hidden states --------------------------------
    zero = dataclasses.replace(tcfg, num_hidden_layers=0, tie_word_embeddings=False)
    m0 = TargetModel(zero, {"embed": fin.to(torch.bfloat16), "lm_head": tw["embed"], "norm": tw["norm"],
                            "layers": []}, DEV)
    lg = m0.forward(torch.arange(P + T, **i32), torch.arange(P + T, **i32), m0.make_cache(1, P + T),
                    max_kv=P + T, head="logits").float().cpu()
    ok, mx, mean, rmx, rmean = _vs_sensitivity(lg, torch.cat([lg_p, lg_b], 0), lm32)
    print(f"lm_head teacher-forced: max err {mx:.4f} mean {mean:.2e} (oracle fp32 vs bf16 max {rmx:.4f} "
          f"mean {rmean:.2e})")
    if not ok:
        bad.append(("lm_head", mx, mean, rmx, rmean))
    del m0

    # --- end to end, free running ---------------------------------------------------
    target = TargetModel(tcfg, tw, DEV)
    cache = target.make_cache(1, P + T)
    got_p = target.forward(torch.tensor(prompt, **i32), torch.arange(P, **i32), cache, max_kv=P,
                           head="logits").float().cpu()
    got_b = target.forward(torch.tensor(block, **i32), torch.arange(P, P + T, **i32), cache, max_kv=P + T,
                           head="logits").float().cpu()
    del target, cache
    got, ref = torch.cat([got_p, got_b], 0), torch.cat([lg_p, lg_b], 0)
    with monkeypatch.context() as mp:
        mp.setattr(O, "bf16", lambda x: x.float())
        (_, f_p), (_, f_b) = _oracle_layer_inputs(O.OracleTarget(tcfg, tw), prompt, block)
    ref32 = torch.cat([f_p, f_b], 0)
    d_gpu = (got - ref).abs()
    d_ora = (ref32 - ref).abs()
    agree = (got.argmax(-1) == ref.argmax(-1)).float().mean().item()
    agree32 = (ref32.argmax(-1) == ref.argmax(-1)).float().mean().item()
    print(f"36 layers end to end: gpu vs oracle max {d_gpu.max().item():.4f} mean {d_gpu.mean().item():.2e}, "
          f"greedy agreement {agree:.3f}; oracle fp32 vs oracle bf16 max {d_ora.max().item():.4f} "
          f"mean {d_ora.mean().item():.2e} agreement {agree32:.3f}")
    assert not bad, bad
    assert d_gpu.max().item() <= 1.5 * d_ora.max().item()
    assert d_gpu.mean().item() <= d_ora.mean().item()
    assert agree >= 0.9


def test_qwen35_27b_width_gdn_state_teacher_forced(monkeypatch):
    """Per gated-delta layer of a 27B-width hybrid (layers 0-2 of 4), fed the oracle's
    input: prefill of 40 rows, a 16-row verify block, rollback to 6 accepted rows."""
    from oracle import dflash_oracle as O
    from dflash_b200.config import qwen35_27b_pair
    from dflash_b200 import ops
    from dflash_b200.hybrid import HybridTargetModel
    tcfg, _ = qwen35_27b_pair(4)
    tw = _cpu_weights(tcfg, 4)
    g = torch.Generator().manual_seed(4)
    P, T, acc = 40, 16, 6
    prompt = torch.randint(0, tcfg.vocab_size, (P,), generator=g).tolist()
    block = torch.randint(0, tcfg.vocab_size, (T,), generator=g).tolist()
    ot = O.OracleHybridTarget(tcfg, tw)
    oc = ot.make_cache(P + T + 8)
    ins = {}
    for name, toks, start in (("prefill", prompt, 0), ("block", block, P)):
        pos = torch.arange(start, start + len(toks))
        h = ot.embed_tokens(toks)
        for l in range(tcfg.num_hidden_layers):
            lw = tw["layers"][l]
            ins[(name, l)] = h
            h = ot.gdn_layer(lw, h, oc[l]) if tcfg.is_linear_layer(l) else ot.attn_layer(lw, h, pos, oc[l])
            ins[(name, l + 1)] = h
    ot.rollback_linear(oc, acc)
    H = tcfg.hidden_size
    i32 = dict(dtype=torch.int32, device=DEV)
    one = dataclasses.replace(tcfg, num_hidden_layers=1, vocab_size=P + T)
    assert one.is_linear_layer(0)
    for l in range(tcfg.num_hidden_layers):
        if not tcfg.is_linear_layer(l):
            continue
        rows = torch.cat([ins[("prefill", l)], ins[("block", l)]], 0).to(torch.bfloat16)
        m = HybridTargetModel(one, {"embed": rows, "norm": tw["norm"], "layers": [tw["layers"][l]]}, DEV)
        hc = m.make_cache(1, P + T + 8, block=T)
        seq = slice(0, 1)
        tp = torch.empty((P, H), dtype=torch.bfloat16, device=DEV)
        m.forward(torch.arange(P, **i32), torch.arange(P, **i32), hc, max_kv=P, layer_ids=[0], taps_out=tp,
                  seqs=seq, verify=False, T=P, head="hidden")
        m.commit_prefill(hc, seq, torch.full((1,), P, **i32), P)
        tb = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
        m.forward(torch.arange(P, P + T, **i32), torch.arange(P, P + T, **i32), hc, max_kv=P + T, layer_ids=[0],
                  taps_out=tb, seqs=seq, verify=True, T=T, head="hidden")
        m.rollback(hc, torch.full((1,), acc, **i32), 1, T)
        lw = tw["layers"][l]
        state, ref_state = hc.state[0][0].cpu(), oc[l].state
        rel = ((state - ref_state).abs().max() / ref_state.abs().max()).item()
        # the recurrence itself on the oracle's own q, k, v, g, beta of this layer (identical
        # inputs): prefill, then the block with snapshots, state after `acc` tokens
        conv = torch.zeros((3, ot.C))
        st = torch.zeros((1, ot.Hv, ot.Dv, ot.Dk), device=DEV)
        for name, n in (("prefill", P), ("block", T)):
            x = O.rms_norm(ins[(name, l)], lw["input_layernorm"], tcfg.rms_norm_eps)
            qkv = O.linear(x, lw["in_proj_qkv"])
            window = torch.cat([conv, qkv], 0)
            q, k, v = O.gdn_conv_qkv(window, lw["conv1d"], ot.Hk, ot.Hv, ot.Dk, ot.Dv)
            gg, bb = O.gdn_gates(O.linear(x, lw["in_proj_a"]), O.linear(x, lw["in_proj_b"]), lw["A_log"],
                                 lw["dt_bias"])
            conv = window[-3:]
            args = [t[None].contiguous().to(DEV) for t in (q.bfloat16(), k.bfloat16(), v.bfloat16(), gg, bb)]
            if name == "prefill":
                ops.gdr_recurrence(*args, st, state_out=st)
            else:
                snaps = torch.empty((1, n, ot.Hv, ot.Dv, ot.Dk), device=DEV)
                ops.gdr_recurrence(*args, st, snapshots=snaps)
                st = snaps[:, acc - 1]
        op_rel = ((st[0].cpu() - ref_state).abs().max() / ref_state.abs().max()).item()
        # the fp32 oracle layer on the same inputs (its own rounding sensitivity)
        with monkeypatch.context() as mp:
            mp.setattr(O, "bf16", lambda x: x.float())
            c32 = O.GDNCache(ot.C, ot.Hv, ot.Dv, ot.Dk)
            o32_p = ot.gdn_layer(lw, ins[("prefill", l)], c32)
            o32_b = ot.gdn_layer(lw, ins[("block", l)], c32)
            c32.state = c32.record[1][acc - 1]
        rel32 = ((c32.state - ref_state).abs().max() / ref_state.abs().max()).item()
        ok_p, mx_p, _, rmx_p, _ = _vs_sensitivity(tp.cpu(), ins[("prefill", l + 1)], o32_p)
        ok_b, mx_b, _, rmx_b, _ = _vs_sensitivity(tb.cpu(), ins[("block", l + 1)], o32_b)
        ok_c, conv_d, _ = _within(hc.conv[0][0].cpu(), oc[l].conv, ulps=1)
        print(f"gdn layer {l}: recurrence on identical inputs: state rel err {op_rel:.2e}; whole layer: state rel "
              f"err {rel:.2e} (oracle fp32 vs bf16 {rel32:.2e}), output max err prefill {mx_p:.4f} (oracle "
              f"{rmx_p:.4f}) block {mx_b:.4f} (oracle {rmx_b:.4f}), conv state max err {conv_d:.2e}")
        # north_star's 1e-3 on the fp32 state holds for the recurrence on identical inputs; the
        # whole layer's q, k, v are bf16 projections whose roundings can differ by one ulp from
        # the oracle's (fp32 sums in another order), which moves the state by ~2^-9 relative:
        # the layer's state must then stay within the oracle's own bf16-vs-fp32 spread
        assert op_rel <= 1e-3, (l, op_rel)
        assert rel <= max(1e-3, 1.5 * rel32), (l, rel, rel32)
        assert ok_p and ok_b, (l, mx_p, mx_b)
        assert ok_c, (l, conv_d)  # the conv state holds bf16 projection rows
        del m, hc
