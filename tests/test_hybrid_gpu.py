"""Qwen3.5 hybrid target on the GPU: adapter-level forward / verify / rollback against
the CPU oracle (tiny and 27B-width layers), and the lossless property of the fused
speculative step with gated-delta snapshot rollback (single and batched)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp(x):
    return torch.pow(2.0, torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126))) - 7)


def _logit_check(got, ref, ref32, what, agree_min=0.9):
    """Within the oracle's own rounding sensitivity on the same inputs (ref32 = the oracle
    in fp32 arithmetic): mean |gpu - oracle| <= mean |ref32 - oracle|, every element within
    1.5 x the latter's max or one bf16 ulp; greedy agreement at least agree_min (and at
    least the oracle's own bf16-vs-fp32 agreement minus one row)."""
    got = got.float().cpu().reshape(ref.shape)
    d, r = (got - ref).abs(), (ref32 - ref).abs()
    agree = (got.argmax(-1) == ref.argmax(-1)).float().mean().item()
    agree32 = (ref32.argmax(-1) == ref.argmax(-1)).float().mean().item()
    print(f"{what}: max|ref| {ref.abs().max().item():.3f} gpu vs oracle max {d.max().item():.4f} mean "
          f"{d.mean().item():.2e} agreement {agree:.3f}; oracle fp32 vs bf16 max {r.max().item():.4f} mean "
          f"{r.mean().item():.2e} agreement {agree32:.3f}")
    assert d.mean().item() <= r.mean().item(), what
    assert bool((d <= torch.clamp(_ulp(ref), min=1.5 * r.max().item())).all()), what
    assert agree >= min(agree_min, agree32 - 1.0 / ref.shape[0]), what


def _adapter_sequence(cfg, w, prompt, blocks, accepts, layer_ids, monkeypatch, cap=512):
    """Prefill, then for each block: verify with records, roll back to `accepted`, rewind
    the KV by block - accepted. Returns, per forward, the GPU logits, the oracle's and the
    oracle's in fp32 arithmetic (its rounding sensitivity), and the caches."""
    from oracle import dflash_oracle as O
    from dflash_b200.adapters import load_target_model
    lt = load_target_model((cfg, w), device="cuda")
    cache = lt.make_cache(cap)
    ot = O.OracleHybridTarget(cfg, w)
    oc, oc32 = ot.make_cache(cap), ot.make_cache(cap)

    def fp32(fn, *args):
        with monkeypatch.context() as mp:
            mp.setattr(O, "bf16", lambda x: x.float())
            return fn(*args)

    def rollback(c, n_trim, acc):
        for x in c:
            if isinstance(x, O.KV):
                x.trim(n_trim)
        ot.rollback_linear(c, acc)

    pairs = []
    lg, taps = lt.forward_with_hidden_states(torch.tensor(prompt), cache, layer_ids)
    rl, rt = ot.forward_with_hidden_states(prompt, oc, layer_ids)
    r32, _ = fp32(ot.forward_with_hidden_states, prompt, oc32, layer_ids)
    pairs.append(("prefill", lg[0], rl, r32, taps[0], rt))
    for i, (blk, acc) in enumerate(zip(blocks, accepts)):
        lg, taps, rec = lt.forward_with_hidden_states(torch.tensor(blk), cache, layer_ids,
                                                      return_rollback_records=True)
        rl, rt = ot.forward_with_hidden_states(blk, oc, layer_ids)
        r32, _ = fp32(ot.forward_with_hidden_states, blk, oc32, layer_ids)
        pairs.append((f"block{i}", lg[0], rl, r32, taps[0], rt))
        if acc < len(blk):
            lt.rewind_kv_caches(cache, len(blk) - acc)
            lt.rollback_linear_caches(cache, rec, acc)
            rollback(oc, len(blk) - acc, acc)
            fp32(rollback, oc32, len(blk) - acc, acc)
    return lt, cache, ot, oc, oc32, pairs


def test_tiny_hybrid_verify_rollback_matches_oracle(monkeypatch):
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.weights import random_target_weights
    tcfg, dcfg = tiny_hybrid_pair()
    w = random_target_weights(tcfg, 0, std=0.05)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, tcfg.vocab_size, (150,), generator=g).tolist()  # two prefill chunks
    blocks = torch.randint(0, tcfg.vocab_size, (3, 8), generator=g).tolist()
    lt, cache, ot, oc, oc32, pairs = _adapter_sequence(tcfg, w, prompt, blocks, [3, 8, 1], [1, 3], monkeypatch)
    for name, lg, rl, r32, tp, rt in pairs:
        _logit_check(lg, rl, r32, name)
        assert (tp.float().cpu() - rt).abs().max().item() <= 3e-2 * rt.abs().max().item()
    # recurrent state of every gated-delta layer after the last rollback: within the
    # oracle's own bf16-vs-fp32 spread of that state (or 1e-3)
    hc = cache.kv
    for l, gi in lt.model.gdn_index.items():
        got, ref, ref32 = hc.state[gi][0].cpu(), oc[l].state, oc32[l].state
        rel = ((got - ref).abs().max() / ref.abs().max()).item()
        rel32 = ((ref32 - ref).abs().max() / ref.abs().max()).item()
        print(f"layer {l} state rel err {rel:.2e} (oracle fp32 vs bf16 {rel32:.2e})")
        assert rel <= max(1e-3, 1.5 * rel32)
        # the conv state holds bf16 projection rows: within the oracle's own spread too
        d = (hc.conv[gi][0].float().cpu() - oc[l].conv).abs()
        r = (oc32[l].conv - oc[l].conv).abs()
        assert d.mean().item() <= r.mean().item()
        assert bool((d <= torch.clamp(_ulp(oc[l].conv), min=1.5 * r.max().item())).all())


def test_qwen35_27b_layer_logits_parity(monkeypatch):
    """27B-width hybrid layers (3 gated-delta + 1 gated attention): prefill and a verify
    block with rollback, logits against the oracle, measured against the oracle's own
    bf16-vs-fp32 spread on the same inputs (0.22 max, mean 0.028 on the prefill logits
    of max |logit| 7.3)."""
    from dflash_b200.config import qwen35_27b_pair
    from dflash_b200.weights import random_target_weights
    tcfg, _ = qwen35_27b_pair(4)
    w = random_target_weights(tcfg, 4)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, tcfg.vocab_size, (40,), generator=g).tolist()
    blocks = torch.randint(0, tcfg.vocab_size, (2, 16), generator=g).tolist()
    _, _, _, _, _, pairs = _adapter_sequence(tcfg, w, prompt, blocks, [5, 16], [1, 3], monkeypatch, cap=128)
    for name, lg, rl, r32, tp, rt in pairs:
        _logit_check(lg, rl, r32, name, agree_min=0.9 if name == "prefill" else 0.8)


def _tiny_models():
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.hybrid import HybridTargetModel
    from dflash_b200.model import DraftModel
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_hybrid_pair()
    tw, dw = random_target_weights(tcfg, 0, std=0.05), random_draft_weights(dcfg, 0)
    target = HybridTargetModel(tcfg, tw, "cuda")
    return tcfg, dcfg, target, DraftModel(dcfg, dw, target, mask_mode="causal")


def _run(target, draft, prompts, max_new, bs, graph=False, inject=None):
    from dflash_b200.runtime import SpecSession, S_FINISHED
    B = len(prompts)
    sess = SpecSession(target, draft, B, max(len(p) for p in prompts) + max_new, bs, set(), use_graph=graph)
    if inject is not None:
        sess.set_injection(*inject)
    sess.prefill(prompts, max_new)
    for _ in range(max_new + 1):
        if bool(sess.state[:, S_FINISHED].all().item()):
            break
        sess.step()
    outs, accs, _ = sess.outputs()
    return outs, accs


@pytest.mark.parametrize("graph", [False, True])
def test_tiny_hybrid_spec_equals_plain_greedy(graph):
    tcfg, dcfg, target, draft = _tiny_models()
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, tcfg.vocab_size, (40,), generator=g).tolist()
    bs, max_new = dcfg.block_size, 64
    plain, _ = _run(target, None, [prompt], max_new + 3 * bs, 1)
    # injected drafts: the plain trace for a random prefix, noise after it
    steps = max_new + 1
    lengths = torch.randint(0, bs, (steps,), generator=g)
    noise = torch.randint(0, tcfg.vocab_size, (steps, bs), generator=g)
    tr = torch.tensor(plain[0], dtype=torch.int32)
    spec, accs = _run(target, draft, [prompt], max_new, bs, graph=graph, inject=(tr, lengths, noise))
    assert spec[0] == plain[0][:len(spec[0])]
    assert len(spec[0]) == len(prompt) + max_new
    assert any(1 < a < bs for a in accs[0])
    spec_real, _ = _run(target, draft, [prompt], max_new, bs, graph=graph)
    assert spec_real[0] == plain[0][:len(spec_real[0])]


def test_tiny_hybrid_batched_rollback_is_per_sequence():
    """Three sequences of different lengths and acceptance patterns in one batched
    step: each equals its own single-sequence plain greedy decode."""
    tcfg, dcfg, target, draft = _tiny_models()
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in (30, 57, 12)]
    bs, max_new = dcfg.block_size, 40
    plains = [_run(target, None, [p], max_new + 3 * bs, 1)[0][0] for p in prompts]
    L = max(len(p) for p in plains)
    steps = max_new + 1
    B = len(prompts)
    trace = torch.zeros((B, L), dtype=torch.int32)
    for b, p in enumerate(plains):
        trace[b, :len(p)] = torch.tensor(p, dtype=torch.int32)
    lengths = torch.randint(0, bs, (B, steps), generator=g, dtype=torch.int32)
    lengths[1] = bs - 1  # one sequence accepts whole blocks while the others roll back
    noise = torch.randint(0, tcfg.vocab_size, (B, steps * bs), generator=g, dtype=torch.int32)
    outs, accs = _run(target, draft, prompts, max_new, bs, graph=True, inject=(trace, lengths, noise))
    for b, p in enumerate(prompts):
        assert outs[b] == plains[b][:len(outs[b])], b
        assert len(outs[b]) == len(p) + max_new
    assert max(accs[1]) == bs
    assert any(1 < a < bs for a in accs[0] + accs[2])
