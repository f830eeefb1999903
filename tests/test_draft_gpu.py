"""The CUDA DFlash draft against the CPU oracle draft (itself pinned to the reference's
``DFlashDraftModel`` by tests/golden/draft_forward.npz).

What is checked, per cached call (draft.py:109-223, runtime.py:408-423):
  * ``hidden_norm(fc(taps))`` of the context rows and their K/V for every layer
    (k_norm, RoPE at ``offset .. offset + ctx``) appended to the draft cache;
  * the block rows (embedding of ``[last, mask x (bs-1)]``) with RoPE at
    ``offset + ctx + i``, attending to the cache plus the block, mask none or causal;
  * the final-normed hidden states, the lm_head logits of rows 1.. and the proposals
    (their argmax), then the trim of the block's keys (``trim_draft_cache``).
Three calls in a row: the prompt's context, then two accepted prefixes, so the cache
offsets and the block trim are exercised as in the decode loop.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp(x: torch.Tensor) -> torch.Tensor:
    """bf16 spacing at |x| (one unit in the last place of the value a bf16 holds)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.pow(2.0, e - 7)


def _draft_calls(tcfg, dcfg, tw, dw, mask_mode, ctx_rows, seed, monkeypatch):
    """Runs the GPU draft, the oracle draft and the oracle draft in fp32 arithmetic (its
    own rounding sensitivity) over the same calls; returns per call (gpu hidden, oracle
    hidden, fp32 oracle hidden, gpu logits of rows 1.., oracle logits, fp32 oracle logits)."""
    from oracle import dflash_oracle as O
    from dflash_b200.model import DraftModel, TargetModel
    target = TargetModel(tcfg, tw, DEV)
    draft = DraftModel(dcfg, dw, target, mask_mode=mask_mode)
    ot = O.OracleTarget(tcfg, tw)
    od = O.OracleDraft(dcfg, dw, ot, mask_mode=mask_mode)
    bs, H = dcfg.block_size, dcfg.hidden_size
    ntaps = len(dcfg.target_layer_ids)
    cap = sum(ctx_rows) + 2 * bs
    cache = draft.make_cache(1, cap)
    ocache = od.make_cache(cap)
    ocache32 = od.make_cache(cap)
    g = torch.Generator().manual_seed(seed)
    # taps: residual-stream-like rows (bf16, unit scale)
    taps_all = torch.randn(sum(ctx_rows), ntaps * H, generator=g).to(torch.bfloat16)
    lasts = torch.randint(0, tcfg.vocab_size, (len(ctx_rows),), generator=g).tolist()
    off = 0
    out = []
    for Tc, last in zip(ctx_rows, lasts):
        ctx = taps_all[off:off + Tc]
        block = [last] + [dcfg.mask_token_id] * (bs - 1)
        pos_ctx = torch.arange(off, off + Tc, dtype=torch.int32, device=DEV)
        pos_blk = torch.arange(off + Tc, off + Tc + bs, dtype=torch.int32, device=DEV)
        kv_len = torch.tensor([off + Tc + bs], dtype=torch.int32, device=DEV)
        toks = torch.tensor(block, dtype=torch.int32, device=DEV)
        draft.ingest_context(ctx.to(DEV), pos_ctx, cache)
        hid = draft.forward_block(toks, pos_blk, cache, kv_len, cap, head="hidden").float().cpu()
        # the same call again (the block's keys land in the same slots): logits of the proposals
        lg = draft.forward_block(toks, pos_blk, cache, kv_len, cap, head="logits")[1:].float().cpu()
        dh = od(ot.embed_tokens(block), ctx.float(), ocache)
        olg = ot.lm_head_logits(dh[1:])
        with monkeypatch.context() as mp:
            mp.setattr(O, "bf16", lambda x: x.float())
            dh32 = od(ot.embed_tokens(block), ctx.float(), ocache32)
            olg32 = ot.lm_head_logits(dh32[1:])
        for c in ocache + ocache32:
            c.trim(bs)  # trim_draft_cache (runtime.py:32-34, 420)
        out.append((hid, dh, dh32, lg, olg, olg32))
        off += Tc
    return out


def _check(calls, what, tol=2e-2):
    """Within the oracle's own rounding sensitivity: mean |gpu - oracle| <= mean
    |oracle_fp32 - oracle|, and every element within 1.5 x the latter's max or within one
    bf16 ulp of the oracle's value; proposals equal except at near-ties (top-two oracle
    logits within 2 x tol)."""
    bad = []
    for i, (hid, ref_h, h32, lg, ref_lg, l32) in enumerate(calls):
        prop, ref_prop = lg.argmax(-1), ref_lg.argmax(-1)
        top2 = ref_lg.topk(2, dim=-1).values
        gap = top2[:, 0] - top2[:, 1]
        mism = prop != ref_prop
        for name, got, ref, r32 in (("hidden", hid, ref_h, h32), ("logits", lg, ref_lg, l32)):
            d, r = (got - ref).abs(), (r32 - ref).abs()
            ok = bool(d.mean() <= r.mean()) and bool((d <= torch.clamp(_ulp(ref), min=1.5 * r.max())).all())
            print(f"{what} call {i} {name}: gpu vs oracle max {d.max().item():.4f} mean {d.mean().item():.2e}; "
                  f"oracle fp32 vs bf16 max {r.max().item():.4f} mean {r.mean().item():.2e}")
            if not ok:
                bad.append((i, name))
        print(f"{what} call {i}: proposals equal {int((~mism).sum())}/{len(prop)}")
        if not bool((gap[mism] <= 2 * tol).all()):
            bad.append((i, "proposals", gap[mism].tolist()))
    assert not bad, (what, bad)


@pytest.mark.parametrize("mask_mode", ["none", "causal"])
def test_tiny_draft_matches_oracle(mask_mode, monkeypatch):
    from dflash_b200.config import tiny_pair
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    tw, dw = random_target_weights(tcfg, 0), random_draft_weights(dcfg, 0)
    _check(_draft_calls(tcfg, dcfg, tw, dw, mask_mode, [64, 5, 8], seed=11, monkeypatch=monkeypatch),
           f"tiny/{mask_mode}")


@pytest.mark.parametrize("mask_mode", ["none", "causal"])
def test_qwen3_4b_width_draft_matches_oracle(mask_mode, monkeypatch):
    """The config-3 draft: 5 layers at Qwen3-4B width, 5 taps (12800 -> 2560 fc), block 16,
    lm_head over the 151936-token vocabulary."""
    import dataclasses
    from dflash_b200.config import qwen3_4b_pair
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = qwen3_4b_pair()
    tcfg = dataclasses.replace(tcfg, num_hidden_layers=1)  # the draft uses the target's embedding only
    tw, dw = random_target_weights(tcfg, 2), random_draft_weights(dcfg, 2)
    _check(_draft_calls(tcfg, dcfg, tw, dw, mask_mode, [40, 7, 16], seed=12, monkeypatch=monkeypatch),
           f"qwen3-4b/{mask_mode}")


def test_tiny_real_draft_acceptance_matches_oracle_loop():
    """Config 1 with the real draft (no injection): the GPU decode loop's acceptance
    lengths equal the oracle loop's (O.spec_generate, pinned to the reference runtime) step
    for step up to the first step where a bf16 near-tie changes a token, and the committed
    tokens equal the oracle's over that span."""
    from oracle import dflash_oracle as O
    from dflash_b200.config import tiny_pair
    from dflash_b200.model import DraftModel, TargetModel
    from dflash_b200.runtime import SpecSession, S_FINISHED
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    tw, dw = random_target_weights(tcfg, 0), random_draft_weights(dcfg, 0)
    target = TargetModel(tcfg, tw, DEV)
    draft = DraftModel(dcfg, dw, target)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, tcfg.vocab_size, (64,), generator=g).tolist()
    sess = SpecSession(target, draft, 1, 64 + 128, dcfg.block_size, set(), use_graph=True)
    sess.prefill([prompt], 128)
    for _ in range(129):
        if int(sess.state[0, S_FINISHED].item()):
            break
        sess.step()
    outs, accs, _ = sess.outputs()
    ot = O.OracleTarget(tcfg, tw)
    ref_out, ref_accs = O.spec_generate(ot, O.OracleDraft(dcfg, dw, ot), prompt, 128, dcfg.block_size)
    n_same = 0
    for a, b in zip(accs[0], ref_accs):
        if a != b:
            break
        n_same += 1
    committed = 64 + 1 + sum(ref_accs[:n_same])
    print(f"acceptance lengths equal for {n_same}/{len(ref_accs)} steps; gpu {accs[0][:12]} oracle {ref_accs[:12]}")
    assert n_same >= 4
    assert outs[0][:committed] == ref_out[:committed]
