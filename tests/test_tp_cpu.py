"""Tensor-parallel sharding of the Qwen3.5 hybrid (the reference's Model.shard,
custom_qwen35_model.py:1286-1402), checked on the CPU: the sum over ranks of each
rank's row-parallel branch output (computed by the oracle on that rank's shard)
equals the unsharded branch, layer by layer; plus the host-side exchange of the
peer-buffer handles over a world-size-2 gloo group."""
import os

import pytest
import torch

from oracle import dflash_oracle as O


@pytest.mark.parametrize("size", [2, 4])
def test_sharded_hybrid_sums_to_full(monkeypatch, size):
    from dflash_b200.config import TargetConfig
    from dflash_b200.tp import shard_config, shard_weights
    from dflash_b200.weights import random_target_weights
    monkeypatch.setattr(O, "bf16", lambda x: x.float())  # fp32: the comparison is of the sharding algebra
    # 4 layers (3 GDN + gated attention), 8 q / 2 kv heads of 64 (kv repeated when size > 2)
    cfg = TargetConfig(model_type="qwen3_5", hidden_size=256, num_hidden_layers=4, num_attention_heads=8,
                       num_key_value_heads=2, head_dim=64, partial_rotary_factor=0.25, intermediate_size=1024,
                       vocab_size=512, linear_num_key_heads=4, linear_num_value_heads=8, linear_key_head_dim=32,
                       linear_value_head_dim=32)
    w = random_target_weights(cfg, 5, std=0.05)
    full = O.OracleHybridTarget(cfg, w)
    ranks = [O.OracleHybridTarget(shard_config(cfg, size), shard_weights(cfg, w, r, size)) for r in range(size)]
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
    pos = torch.arange(12)
    fc = full.make_cache(64)
    rc = [r.make_cache(64) for r in ranks]
    h = full.embed_tokens(toks)
    for l in range(cfg.num_hidden_layers):
        lw = w["layers"][l]
        if cfg.is_linear_layer(l):
            ref = full.gdn_mixer(lw, h, fc[l])
            parts = [r.gdn_mixer(r.w["layers"][l], h, rc[i][l]) for i, r in enumerate(ranks)]
        else:
            ref = full.attn_mixer(lw, h, pos, fc[l])
            parts = [r.attn_mixer(r.w["layers"][l], h, pos, rc[i][l]) for i, r in enumerate(ranks)]
        torch.testing.assert_close(sum(parts), ref, rtol=1e-4, atol=1e-5)
        h = h + ref
        ref = full.mlp_out(lw, h)
        parts = [r.mlp_out(r.w["layers"][l], h) for r in ranks]
        torch.testing.assert_close(sum(parts), ref, rtol=1e-4, atol=1e-5)
        h = h + ref
    # recurrent state of each rank = its heads of the full state
    Hv = cfg.linear_num_value_heads // size
    for l in range(cfg.num_hidden_layers):
        if cfg.is_linear_layer(l):
            for i in range(size):
                torch.testing.assert_close(rc[i][l].state, fc[l].state[i * Hv:(i + 1) * Hv], rtol=1e-4, atol=1e-6)


def _gather_worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    handle = bytes([rank]) * 64
    got = [None] * world
    dist.all_gather_object(got, handle)
    out[rank] = [g[0] for g in got]
    dist.destroy_process_group()


def test_handle_exchange_gloo():
    """TPComm exchanges 64-byte IPC handles with all_gather_object: every rank sees
    every rank's handle in rank order (world size 2, gloo, CPU)."""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = mp.Manager().dict()
    mp.spawn(_gather_worker, args=(2, port, out), nprocs=2, join=True)
    assert out[0] == [0, 1] and out[1] == [0, 1]


def test_shard_config_rejects_indivisible():
    from dflash_b200.config import qwen35_27b_pair
    from dflash_b200.tp import shard_config
    cfg, _ = qwen35_27b_pair(4)
    for n in (2, 4, 8):
        c = shard_config(cfg, n)
        assert c.num_attention_heads * n == 24 and c.linear_num_value_heads * n == 48
        assert c.num_key_value_heads == max(1, 4 // n)
    with pytest.raises(ValueError):
        shard_config(cfg, 5)
