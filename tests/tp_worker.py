"""Worker for tests/test_tp_gpu.py, launched with torch.distributed.run (one rank per
GPU). Checks the tensor-parallel Qwen3.5 hybrid against the single-GPU model:
prefill + verify logits (tiny and 27B width), every rank holding the same tokens,
and the lossless property (speculative decode == plain greedy) under TP.
All single-GPU reference work is done before the tensor-parallel phase so that the
ranks issue their all-sum calls together."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "dflash-mlx_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def forward_logits(model, toks, cache, layer_ids, T):
    dev = model.device
    t = torch.tensor(toks, dtype=torch.int32, device=dev)
    pos = torch.arange(cache.kv_offset, cache.kv_offset + len(toks), dtype=torch.int32, device=dev)
    taps = torch.empty((len(toks), len(layer_ids) * model.cfg.hidden_size), dtype=torch.bfloat16, device=dev)
    out = model.forward(t, pos, cache.hc, max_kv=cache.kv_offset + len(toks), layer_ids=layer_ids, taps_out=taps,
                        head="logits", seqs=slice(0, 1), verify=T is not None, T=len(toks)).float().clone()
    if T is None:
        model.commit_prefill(cache.hc, slice(0, 1), torch.full((1,), len(toks), dtype=torch.int32, device=dev),
                             len(toks))
    else:
        model.rollback(cache.hc, torch.full((1,), T, dtype=torch.int32, device=dev), 1, len(toks))
    cache.kv_offset += len(toks)
    return out, taps.float().clone()


class Cache:
    def __init__(self, model, cap):
        self.hc = model.make_cache(1, cap, block=16)
        self.kv_offset = 0


def check_logits(name, got, ref, max_bound):
    d = (got - ref).abs()
    agree = (got.argmax(-1) == ref.argmax(-1)).float().mean().item()
    print(f"[{name}] max err {d.max().item():.4f} mean err {d.mean().item():.2e} agreement {agree:.3f}", flush=True)
    assert d.mean().item() <= 2e-2 and d.max().item() <= max_bound and agree >= 0.9, name


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    from dflash_b200.config import qwen35_27b_pair, tiny_hybrid_pair
    from dflash_b200.hybrid import HybridTargetModel
    from dflash_b200.model import DraftModel
    from dflash_b200.runtime import SpecSession, S_FINISHED
    from dflash_b200.tp import TPComm, shard_config, shard_weights
    from dflash_b200.weights import random_draft_weights, random_target_weights
    from dflash_b200 import ops

    # the TP path sums fp32 partials (one bf16 rounding per projection, as on one GPU):
    # it differs from the single-GPU model by the order of the K sums only
    cases = [("tiny", *tiny_hybrid_pair(), 0.05, 0.08), ("27b-width", *qwen35_27b_pair(4), 0.02, 0.15)]
    g = torch.Generator().manual_seed(11)
    results = {}
    # ---- phase 1: single-GPU references (every rank computes them; no TP calls) ----
    for name, tcfg, dcfg, std, _ in cases:
        w = random_target_weights(tcfg, 4, std=std, device="cuda")
        prompt = torch.randint(0, tcfg.vocab_size, (40,), generator=g).tolist()
        block = torch.randint(0, tcfg.vocab_size, (16,), generator=g).tolist()
        ref = HybridTargetModel(tcfg, w, dev)
        c = Cache(ref, 128)
        l0, _ = forward_logits(ref, prompt, c, [1, 3], None)
        l1, _ = forward_logits(ref, block, c, [1, 3], 5)
        results[name] = (tcfg, w, prompt, block, l0, l1)
        del ref, c
    torch.cuda.synchronize()
    dist.barrier()
    # ---- phase 2: the same through the tensor-parallel model ----
    for name, tcfg, dcfg, std, bound in cases:
        tcfg, w, prompt, block, l0, l1 = results[name]
        comm = TPComm(rank, world, dev, max_rows=128, hidden=tcfg.hidden_size)
        m = HybridTargetModel(shard_config(tcfg, world), shard_weights(tcfg, w, rank, world), dev, tp=comm)
        c = Cache(m, 128)
        t0, _ = forward_logits(m, prompt, c, [1, 3], None)
        t1, _ = forward_logits(m, block, c, [1, 3], 5)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        check_logits(f"{name} prefill rank {rank}", t0, l0, bound)
        check_logits(f"{name} verify rank {rank}", t1, l1, bound)
        both = [torch.zeros_like(t1) for _ in range(world)]
        dist.all_gather(both, t1)
        assert all(torch.equal(both[0], x) for x in both), "ranks disagree"
        del m, c
        comm.close()
    # ---- phase 3: lossless speculative decode under TP (tiny) ----
    tcfg, dcfg = tiny_hybrid_pair()
    w = random_target_weights(tcfg, 0, std=0.05, device="cuda")
    dw = random_draft_weights(dcfg, 0, device="cuda")
    comm = TPComm(rank, world, dev, max_rows=128, hidden=tcfg.hidden_size)
    m = HybridTargetModel(shard_config(tcfg, world), shard_weights(tcfg, w, rank, world), dev, tp=comm)
    draft = DraftModel(dcfg, dw, m, mask_mode="causal")
    prompt = torch.randint(0, tcfg.vocab_size, (30,), generator=torch.Generator().manual_seed(5)).tolist()
    bs, max_new = dcfg.block_size, 48

    def run(dr, b, inject=None, graph=True):
        sess = SpecSession(m, dr, 1, len(prompt) + max_new + 4 * bs, b, set(), use_graph=graph)
        if inject is not None:
            sess.set_injection(*inject)
        sess.prefill([prompt], max_new + (3 * bs if dr is None else 0))
        for _ in range(max_new + 3 * bs + 1):
            if bool(sess.state[:, S_FINISHED].all().item()):
                break
            sess.step()
        return sess.outputs()[0][0], sess.outputs()[1][0]

    plain, _ = run(None, 1)
    gi = torch.Generator().manual_seed(6)
    lengths = torch.randint(0, bs, (max_new + 2,), generator=gi)
    noise = torch.randint(0, tcfg.vocab_size, (max_new + 2, bs), generator=gi)
    spec, accs = run(draft, bs, inject=(torch.tensor(plain, dtype=torch.int32), lengths, noise))
    assert spec == plain[:len(spec)], "spec != plain under TP"
    assert any(1 < a < bs for a in accs)
    toks = torch.tensor(spec, dtype=torch.int64, device=dev)
    gathered = [torch.zeros_like(toks) for _ in range(world)]
    dist.all_gather(gathered, toks)
    assert all(torch.equal(gathered[0], x) for x in gathered)
    assert ops.device_error() == 0
    comm.close()
    dist.barrier()
    if rank == 0:
        print("TP_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
