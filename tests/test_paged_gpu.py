"""Paged K/V: the paged append and attention equal the contiguous ones bit for bit, with
pages handed out in a scrambled order; a paged session equals a contiguous one token for
token, and holds pages for each sequence's own length only."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("key_chunk,causal", [(128, True), (1024, True), (128, False), (64, True)])
def test_paged_append_and_attention_equal_contiguous(key_chunk, causal):
    from dflash_b200 import ops
    g = torch.Generator().manual_seed(5)
    B, bs, Hq, Hkv, hd, PS = 3, 16, 32, 8, 128, 64
    lens = [700, 130, 1500]  # cached context per sequence
    cap = max(lens) + bs + 64
    n_pages_each = [(n + bs + PS - 1) // PS for n in lens]
    total = sum(n_pages_each)
    perm = torch.randperm(total, generator=g)
    table = torch.full((B, (cap + PS - 1) // PS), total, dtype=torch.int32)
    o = 0
    for b, n in enumerate(n_pages_each):
        table[b, :n] = perm[o:o + n].to(torch.int32)
        o += n
    table = table.to(DEV)
    kc = torch.zeros((B, Hkv, cap, hd), dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    kp = torch.zeros((total + 1, Hkv, PS, hd), dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    # the cached contexts: written through both layouts by the append of random rows
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16().to(DEV)
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16().to(DEV)
    inv = (1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))).float().to(DEV)
    for b, n in enumerate(lens):
        rows = torch.randn(n, (Hq + 2 * Hkv) * hd, generator=g).bfloat16().to(DEV)
        pos = torch.arange(n, dtype=torch.int32, device=DEV)
        seq = torch.full((n,), b, dtype=torch.int32, device=DEV)
        ops.qkv_rope_append(rows, pos, qn, kn, inv, kc, vc, Hq, Hkv, hd, hd, 1e-6, row_seq=seq)
        ops.qkv_rope_append(rows, pos, qn, kn, inv, kp, vp, Hq, Hkv, hd, hd, 1e-6, row_seq=seq, page_table=table,
                            page_size=PS)
    # a verify block per sequence
    blk = torch.randn(B * bs, (Hq + 2 * Hkv) * hd, generator=g).bfloat16().to(DEV)
    pos = torch.tensor([n + i for n in lens for i in range(bs)], dtype=torch.int32, device=DEV)
    seq = (torch.arange(B * bs, device=DEV) // bs).to(torch.int32)
    q1 = ops.qkv_rope_append(blk, pos, qn, kn, inv, kc, vc, Hq, Hkv, hd, hd, 1e-6, row_seq=seq)
    q2 = ops.qkv_rope_append(blk, pos, qn, kn, inv, kp, vp, Hq, Hkv, hd, hd, 1e-6, row_seq=seq, page_table=table,
                             page_size=PS)
    assert torch.equal(q1, q2)
    for b, n in enumerate(lens):  # every cached row landed in its page
        for p in (0, n // 2, n + bs - 1):
            pg, r = int(table[b, p // PS]), p % PS
            assert torch.equal(kp[pg, :, r], kc[b, :, p]) and torch.equal(vp[pg, :, r], vc[b, :, p])
    kv_len = torch.tensor([n + bs for n in lens], dtype=torch.int32, device=DEV)
    a1 = ops.attention(q1, kc, vc, pos, causal, max_kv=cap, kv_len=kv_len, row_seq=seq, seq_rows=bs,
                       key_chunk=key_chunk)
    a2 = ops.attention(q2, kp, vp, pos, causal, max_kv=cap, kv_len=kv_len, row_seq=seq, seq_rows=bs,
                       key_chunk=key_chunk, page_table=table, page_size=PS)
    assert torch.equal(a1, a2)


def test_paged_session_equals_contiguous_session_and_saves_memory():
    from dflash_b200.config import tiny_pair
    from dflash_b200.model import DraftModel, TargetModel
    from dflash_b200.runtime import SpecSession, S_FINISHED
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg, dcfg = tiny_pair()
    target = TargetModel(tcfg, random_target_weights(tcfg, 0), DEV)
    draft = DraftModel(dcfg, random_draft_weights(dcfg, 0), target)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in (300, 20, 41, 9, 150)]
    outs, sizes = [], []
    for paged in (False, True):
        sess = SpecSession(target, draft, len(prompts), 300 + 40, dcfg.block_size, set(), use_graph=True,
                           paged=paged)
        sess.prefill(prompts, 40)
        for _ in range(41):
            if bool(sess.state[:, S_FINISHED].all().item()):
                break
            sess.step()
        outs.append(sess.outputs()[0])
        sizes.append(sess.tcache.k.numel() + sess.dcache.k.numel())
    assert outs[0] == outs[1]
    print(f"K/V elements contiguous {sizes[0]} paged {sizes[1]}")
    assert sizes[1] < 0.75 * sizes[0]
