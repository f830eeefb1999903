"""Temperature sampling (sample_tokens, runtime.py:22-29, temperature >= 1e-5) on the
GPU: the Gumbel-max kernel draws from softmax(logits / T), its noise is the host
restatement's, and a speculative sampled decode equals the plain sampled decode with
the same seed (noise keyed by absolute position), for Qwen3 and the Qwen3.5 hybrid."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _host_noise(key: int, V: int) -> np.ndarray:
    """Host restatement of gumbel_noise: u from the top 24 bits of mix64(key ^ col * c)."""
    from dflash_b200 import ops
    out = np.empty(V)
    for c in range(V):
        x = ops.mix64(key ^ ((c * 0xD1B54A32D192ED03) & ops._M64))
        u = ((x >> 40) + 0.5) / 16777216.0
        out[c] = -math.log(-math.log(u))
    return out


def test_sample_partials_match_host_noise():
    from dflash_b200 import ops
    g = torch.Generator().manual_seed(0)
    M, V, T = 64, 1000, 0.7
    logits = (torch.randn((M, V), generator=g) * 2).bfloat16()
    keys = [ops.sample_key(11, ops.SAMPLE_TAG_TARGET, 0, p) for p in range(M)]
    part = ops.sample_partials(logits.cuda(), ops.keys_tensor(keys, "cuda"), T)
    got = ops.argmax_reduce(part).cpu().numpy()
    lf = logits.float().numpy().astype(np.float64) / T
    for m in range(M):
        s = lf[m] + _host_noise(keys[m], V)
        top = np.sort(s)[-2:]
        if top[1] - top[0] > 1e-4:  # not a float32 near-tie
            assert got[m] == int(np.argmax(s)), m


def test_sample_keys_kernel_matches_host():
    from dflash_b200 import ops
    from dflash_b200.runtime import S_START, STATE_INTS
    B, bs = 3, 5
    st = torch.zeros((B, STATE_INTS), dtype=torch.int32)
    st[:, S_START] = torch.tensor([7, 100, 4096])
    st = st.cuda()
    keys = torch.empty(B * bs, dtype=torch.int64, device="cuda")
    for tag, off in ((ops.SAMPLE_TAG_DRAFT, 0), (ops.SAMPLE_TAG_TARGET, 1)):
        ops.sample_keys(st, B, bs, 2 ** 63 + 5, tag, off, keys)
        want = [ops.sample_key(2 ** 63 + 5, tag, b, int(st[b, S_START]) + i + off) for b in range(B)
                for i in range(bs)]
        assert keys.cpu().tolist() == ops.keys_tensor(want, "cpu").tolist()


def test_sample_distribution_is_softmax():
    """Frequencies over 65536 keys against softmax(logits / T): chi-square test."""
    from dflash_b200 import ops
    V, T, N = 40, 0.8, 65536
    g = torch.Generator().manual_seed(1)
    row = (torch.randn(V, generator=g) * 1.5).bfloat16()
    logits = row.expand(N, V).contiguous().cuda()
    keys = ops.keys_tensor([ops.sample_key(5, 0, 0, r) for r in range(N)], "cuda")
    got = ops.argmax_reduce(ops.sample_partials(logits, keys, T)).long().cpu()
    counts = torch.bincount(got, minlength=V).double()
    p = torch.softmax(row.double() / T, dim=0)
    exp = p * N
    chi2 = float(((counts - exp) ** 2 / exp).sum())
    # 39 degrees of freedom: P(chi2 > 80) < 1e-4
    assert chi2 < 80.0, chi2
    # and the runtime's sample_tokens at temperature 0 is the argmax
    from dflash_b200.runtime import sample_tokens
    assert int(sample_tokens(logits[:1], 0.0)[0]) == int(torch.argmax(row.float()))


def _session(target, draft, prompts, max_new, bs, T, seed, graph=False, inject=None):
    from dflash_b200.runtime import S_FINISHED, SpecSession
    B = len(prompts)
    sess = SpecSession(target, draft, B, max(len(p) for p in prompts) + max_new, bs, set(), use_graph=graph,
                       temperature=T, seed=seed)
    if inject is not None:
        sess.set_injection(*inject)
    sess.prefill(prompts, max_new)
    for _ in range(max_new + 1):
        if bool(sess.state[:, S_FINISHED].all().item()):
            break
        sess.step()
    outs, accs, _ = sess.outputs()
    return outs, accs


def _injected(trace_rows, bs, steps, V, g):
    B = len(trace_rows)
    L = max(len(t) for t in trace_rows)
    trace = torch.zeros((B, L), dtype=torch.int32)
    for b, t in enumerate(trace_rows):
        trace[b, :len(t)] = torch.tensor(t, dtype=torch.int32)
    lengths = torch.randint(0, bs, (B, steps), generator=g, dtype=torch.int32)
    noise = torch.randint(0, V, (B, steps * bs), generator=g, dtype=torch.int32)
    return trace, lengths, noise


def _check_lossless(target, draft, V, bs, prompts, max_new, graph):
    g = torch.Generator().manual_seed(9)
    T, seed = 0.8, 1234
    plains = [_session(target, None, [p], max_new + 3 * bs, 1, T, seed)[0][0] for p in prompts]
    # the plain decode of sequence b in a batch keys its noise by b: run the batch plainly too
    plain_batch = _session(target, None, prompts, max_new + 3 * bs, 1, T, seed)[0]
    assert plain_batch[0] == plains[0]
    other = _session(target, None, [prompts[0]], max_new, 1, T, seed + 1)[0][0]
    assert other != plains[0][:len(other)]  # the seed changes the draws
    inj = _injected(plain_batch, bs, max_new + 1, V, g)
    outs, accs = _session(target, draft, prompts, max_new, bs, T, seed, graph=graph, inject=inj)
    for b, p in enumerate(prompts):
        assert outs[b] == plain_batch[b][:len(outs[b])], b
        assert len(outs[b]) == len(p) + max_new
    assert any(1 < a < bs for row in accs for a in row)
    real, _ = _session(target, draft, prompts, max_new, bs, T, seed, graph=graph)
    for b in range(len(prompts)):
        assert real[b] == plain_batch[b][:len(real[b])], b


@pytest.mark.parametrize("graph", [False, True])
def test_qwen3_sampled_spec_equals_plain(graph):
    from dflash_b200.config import tiny_pair
    from dflash_b200.model import DraftModel, TargetModel
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    target = TargetModel(tcfg, random_target_weights(tcfg, 0), "cuda")
    draft = DraftModel(dcfg, random_draft_weights(dcfg, 0), target)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in (48, 21)]
    _check_lossless(target, draft, tcfg.vocab_size, dcfg.block_size, prompts, 48, graph)


def test_hybrid_sampled_spec_equals_plain():
    from dflash_b200.config import tiny_hybrid_pair
    from dflash_b200.hybrid import HybridTargetModel
    from dflash_b200.model import DraftModel
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_hybrid_pair()
    target = HybridTargetModel(tcfg, random_target_weights(tcfg, 0, std=0.05), "cuda")
    draft = DraftModel(dcfg, random_draft_weights(dcfg, 0), target, mask_mode="causal")
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in (33, 17)]
    _check_lossless(target, draft, tcfg.vocab_size, dcfg.block_size, prompts, 40, True)
