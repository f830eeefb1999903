"""The step-level C ABI (dfl_ctx_create / dfl_draft_step / dfl_verify_step / dfl_rollback)
driven by a C-style loop reproduces the Python runtime's SpecSession bit for bit:
config 1 with the real draft, single and batched (3 sequences; 6 sequences take the
batched kernel forms), with and without recorded graphs, plus oracle-injected drafts."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _tiny():
    from dflash_b200.config import tiny_pair
    from dflash_b200.model import DraftModel, TargetModel
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    target = TargetModel(tcfg, random_target_weights(tcfg, 0), "cuda")
    return tcfg, dcfg, target, DraftModel(dcfg, random_draft_weights(dcfg, 0), target)


def _session(target, draft, prompts, max_new, bs, inject=None):
    from dflash_b200.runtime import SpecSession, S_FINISHED
    sess = SpecSession(target, draft, len(prompts), max(len(p) for p in prompts) + max_new, bs, set(),
                       use_graph=True)
    if inject is not None:
        sess.set_injection(*inject)
    sess.prefill(prompts, max_new)
    for _ in range(max_new + 1):
        if bool(sess.state[:, S_FINISHED].all().item()):
            break
        sess.step()
    return sess.outputs()[0]


def _c_loop(target, draft, prompts, max_new, bs, graph, inject=None):
    from dflash_b200.engine import StepContext
    ctx = StepContext(target, draft, len(prompts), max(len(p) for p in prompts) + max_new, bs, use_graph=graph)
    if inject is not None:
        ctx.set_injection(*[t.to("cuda", torch.int32).contiguous() for t in inject])
    for b, p in enumerate(prompts):
        ctx.prefill(b, p, max_new)
    for _ in range(max_new + 1):
        st, _ = ctx.read()
        if bool((st[:, 5] != 0).all()):
            break
        ctx.step()
    out = ctx.outputs()
    ctx.close()
    return out


@pytest.mark.parametrize("n_seq", [1, 3, 6])
@pytest.mark.parametrize("graph", [False, True])
def test_c_step_loop_equals_spec_session(n_seq, graph):
    tcfg, dcfg, target, draft = _tiny()
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in (64, 30, 57, 12, 41, 9)[:n_seq]]
    ref = _session(target, draft, prompts, 48, dcfg.block_size)
    got = _c_loop(target, draft, prompts, 48, dcfg.block_size, graph)
    assert got == ref


def test_c_step_loop_injected_and_plain():
    """Oracle-injected drafts through dfl_ctx_set_injection, and block size 1 (no draft:
    plain greedy through the same driver) against the session."""
    tcfg, dcfg, target, draft = _tiny()
    g = torch.Generator().manual_seed(22)
    prompt = torch.randint(0, tcfg.vocab_size, (40,), generator=g).tolist()
    bs, max_new = dcfg.block_size, 64
    plain = _session(target, None, [prompt], max_new + 3 * bs, 1)
    assert _c_loop(target, None, [prompt], max_new + 3 * bs, 1, True) == plain
    steps = max_new + 1
    lengths = torch.randint(0, bs, (1, steps), generator=g, dtype=torch.int32)
    noise = torch.randint(0, tcfg.vocab_size, (1, steps * bs), generator=g, dtype=torch.int32)
    trace = torch.tensor(plain[0], dtype=torch.int32)[None]
    ref = _session(target, draft, [prompt], max_new, bs, inject=(trace, lengths, noise))
    got = _c_loop(target, draft, [prompt], max_new, bs, True, inject=(trace, lengths, noise))
    assert got == ref
    assert got[0] == plain[0][:len(got[0])]
