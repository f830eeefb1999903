"""Kernel parity tests: every C-ABI kernel against the CPU oracle (or a torch fp32
reference for plain contractions), plus the row-invariance the lossless
spec == plain-greedy property depends on."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ops():
    from dflash_b200 import ops
    return ops


def _rand(shape, std=1.0, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(dtype)


@pytest.mark.parametrize("M,N,K", [(16, 6144, 2560), (1, 2560, 4096), (5, 2560, 9728), (40, 512, 256),
                                   (16, 151936, 2560), (128, 1536, 2560), (16, 10240, 2560), (2, 2560, 12800)])
def test_gemm_store_matches_fp32(M, N, K):
    ops = _ops()
    x = _rand((M, K), 1.0, 1)
    w = _rand((N, K), 0.02, 2)
    y = ops.gemm(x.to(DEV), w.to(DEV)).float().cpu()
    ref = (x.float() @ w.float().T)
    err = (y - ref).abs().max().item()
    tol = 1e-2 * ref.abs().max().item() + 1e-3
    assert err <= tol, (err, tol)


def test_gemm_residual_and_tap():
    ops = _ops()
    M, N, K = 16, 2560, 4096
    x, w, r = _rand((M, K), 1.0, 3), _rand((N, K), 0.02, 4), _rand((M, N), 1.0, 5)
    rd = r.to(DEV)
    tap = torch.zeros((M, 3 * N), dtype=torch.bfloat16, device=DEV)
    out = ops.gemm(x.to(DEV), w.to(DEV), ops.EPI_RESIDUAL, residual=rd, out=rd, out2=tap[:, N:2 * N])
    ref = (r.float() + (x.float() @ w.float().T).bfloat16().float())
    assert (out.float().cpu() - ref).abs().max().item() < 0.05
    assert torch.equal(tap[:, N:2 * N], out)
    assert tap[:, :N].abs().sum().item() == 0


def test_gemm_silu_mul():
    from dflash_b200.weights import pack_gate_up
    ops = _ops()
    M, F, K = 16, 9728, 2560
    x, wg, wu = _rand((M, K), 1.0, 6), _rand((F, K), 0.02, 7), _rand((F, K), 0.02, 8)
    out = ops.gemm(x.to(DEV), pack_gate_up(wg, wu).to(DEV), ops.EPI_SILU_MUL).float().cpu()
    g = (x.float() @ wg.float().T).bfloat16().float()
    u = (x.float() @ wu.float().T).bfloat16().float()
    ref = (torch.nn.functional.silu(g).bfloat16().float() * u)
    assert (out - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 1e-3


def test_gemm_argmax_matches_logits():
    ops = _ops()
    M, N, K = 16, 151936, 2560
    x, w = _rand((M, K), 1.0, 9), _rand((N, K), 0.02, 10)
    xd, wd = x.to(DEV), w.to(DEV)
    part = ops.gemm(xd, wd, ops.EPI_ARGMAX)
    tok = ops.argmax_reduce(part).cpu()
    logits = ops.gemm(xd, wd).cpu()  # bf16 logits of the same kernel family
    ref = torch.argmax(logits.float(), dim=-1).to(torch.int32)
    assert torch.equal(tok, ref)


def test_gemm_row_invariance():
    """A row's output is bit-identical whatever M is (plain decode M=1 vs verify M=16)."""
    ops = _ops()
    K, N = 2560, 6144
    x, w = _rand((16, K), 1.0, 11).to(DEV), _rand((N, K), 0.02, 12).to(DEV)
    full = ops.gemm(x, w)
    for r in (0, 7, 15):
        one = ops.gemm(x[r:r + 1].contiguous(), w)
        assert torch.equal(one[0], full[r])


def test_rmsnorm():
    from oracle import dflash_oracle as O
    ops = _ops()
    x, w = _rand((33, 2560), 1.0, 13), _rand((2560,), 1.0, 14)
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6).float().cpu()
    ref = O.rms_norm(x.float(), w, 1e-6)
    assert (y - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item()


def test_qkv_rope_append():
    from oracle import dflash_oracle as O
    from dflash_b200.weights import rope_inv_freq
    ops = _ops()
    Hq, Hkv, hd, M = 32, 8, 128, 16
    qkv = _rand((M, (Hq + 2 * Hkv) * hd), 1.0, 15)
    qn, kn = _rand((hd,), 1.0, 16), _rand((hd,), 1.0, 17)
    pos = torch.arange(1000, 1000 + M, dtype=torch.int32)
    pos[3] = -1  # skipped row
    kc = torch.zeros((1, Hkv, 1100, hd), dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    inv = rope_inv_freq(hd, 1e6)
    q = ops.qkv_rope_append(qkv.to(DEV), pos.to(DEV), qn.to(DEV), kn.to(DEV), inv.to(DEV), kc, vc, Hq, Hkv, hd, hd,
                            1e-6).float().cpu()
    valid = pos >= 0
    p = pos[valid].long()
    qr = O.rope(O.rms_norm(qkv[valid, :Hq * hd].float().reshape(-1, Hq, hd), qn, 1e-6), p, inv, hd)
    kr = O.rope(O.rms_norm(qkv[valid, Hq * hd:(Hq + Hkv) * hd].float().reshape(-1, Hkv, hd), kn, 1e-6), p, inv, hd)
    vr = qkv[valid, (Hq + Hkv) * hd:].float().reshape(-1, Hkv, hd)
    assert (q[valid] - qr).abs().max().item() < 3e-2
    kgot = kc[0].float().cpu()[:, p].transpose(0, 1)
    vgot = vc[0].float().cpu()[:, p].transpose(0, 1)
    assert (kgot - kr).abs().max().item() < 3e-2
    assert torch.equal(vgot, vr)
    assert kc[0, :, 1003].abs().sum().item() == 0  # the skipped row wrote nothing


@pytest.mark.parametrize("hd,Hq,Hkv,causal,L", [(128, 32, 8, True, 700), (128, 32, 8, False, 300),
                                                (64, 4, 2, True, 90), (64, 4, 2, False, 1)])
def test_attention_matches_oracle(hd, Hq, Hkv, causal, L):
    from oracle import dflash_oracle as O
    ops = _ops()
    M = 16
    cap = 1024
    q = _rand((M, Hq, hd), 1.0, 20)
    kc = _rand((1, Hkv, cap, hd), 1.0, 21)
    vc = _rand((1, Hkv, cap, hd), 1.0, 22)
    start = max(0, L - M) if causal else 0
    pos = torch.arange(start, start + M, dtype=torch.int32)
    kv_len = torch.tensor([L], dtype=torch.int32)
    out = ops.attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos.to(DEV), causal, max_kv=cap,
                        kv_len=kv_len.to(DEV)).float().cpu()
    lims = [int(p) + 1 for p in pos] if causal else [L] * M
    ref = O.attention(q.float(), kc[0].float(), vc[0].float(), lims, 1 / math.sqrt(hd))
    assert (out - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("key_chunk", [0, 1024])
def test_attention_row_invariance(key_chunk):
    """A query row attends identically in a 16-row causal block and alone (plain decode),
    with many key splits and with one split covering every key."""
    ops = _ops()
    Hq, Hkv, hd, cap = 32, 8, 128, 1024
    kc = _rand((1, Hkv, cap, hd), 1.0, 23).to(DEV)
    vc = _rand((1, Hkv, cap, hd), 1.0, 24).to(DEV)
    q = _rand((16, Hq, hd), 1.0, 25).to(DEV)
    pos = torch.arange(500, 516, dtype=torch.int32, device=DEV)
    full = ops.attention(q, kc, vc, pos, True, max_kv=cap, key_chunk=key_chunk)
    for r in (0, 9, 15):
        one = ops.attention(q[r:r + 1].contiguous(), kc, vc, pos[r:r + 1].contiguous(), True, max_kv=r + 501,
                            key_chunk=key_chunk)
        assert torch.equal(one[0], full[r])


@pytest.mark.parametrize("T,with_snap,B,Hk,Hv,D", [(16, True, 1, 16, 32, 128), (100, False, 1, 16, 32, 128),
                                                   (16, True, 3, 2, 4, 64), (37, False, 2, 2, 4, 64)])
def test_gdr_recurrence_matches_oracle(T, with_snap, B, Hk, Hv, D):
    from oracle import dflash_oracle as O
    ops = _ops()
    g = torch.Generator().manual_seed(1)
    q = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, Hv, D, generator=g).bfloat16()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, Hv, generator=g)))
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g))
    S0 = torch.randn(B, Hv, D, D, generator=g) * 0.1
    o_ref, snaps_ref, S_ref = O.gdr_recurrence(q, k, v, alpha, beta, S0)
    sd = S0.to(DEV)
    out = torch.empty((B, Hv, D, D), device=DEV)
    snaps = torch.empty((B, T, Hv, D, D), device=DEV) if with_snap else None
    o = torch.empty((B, T, Hv, D), dtype=torch.bfloat16, device=DEV)
    ops.gdr_recurrence(q.to(DEV), k.to(DEV), v.to(DEV), alpha.to(DEV), beta.to(DEV), sd, state_out=out,
                       snapshots=snaps, o=o)
    rel = (out.cpu() - S_ref).abs().max() / S_ref.abs().max()
    assert rel.item() < 1e-3
    assert (o.float().cpu() - o_ref).abs().max().item() < 2e-2 * o_ref.abs().max().item() + 1e-3
    if with_snap:
        rels = (snaps.cpu() - snaps_ref).abs().max() / snaps_ref.abs().max()
        assert rels.item() < 1e-3
        assert torch.equal(snaps[:, -1], out)


def _config2_inputs(T: int):
    """Benchmark config 2's draws (seed 1, in this order): q, k ~ bf16 N(0,1) then
    L2-normalised, v ~ bf16 N(0,1), g = -softplus(N(0,1)) used as alpha = exp(g),
    beta = sigmoid(N(0,1)), S0 ~ fp32 N(0, 0.01) of shape [32, 128(Dv), 128(Dk)];
    16 QK heads, 32 V heads, batch 1."""
    B, Hk, Hv, D = 1, 16, 32, 128
    g = torch.Generator().manual_seed(1)
    q = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    k = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    v = torch.randn(B, T, Hv, D, generator=g).bfloat16()
    q = torch.nn.functional.normalize(q.float(), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(k.float(), dim=-1).bfloat16()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, Hv, generator=g)))
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g))
    S0 = torch.randn(B, Hv, D, D, generator=g) * 0.01
    return q, k, v, alpha, beta, S0


@pytest.mark.parametrize("T", [16, 4096])
def test_gdr_recurrence_config2(T):
    """Config 2 exactly: the T=16 verify block with per-token snapshots, and the T=4096
    chunked-prefill length (final state and outputs); fp32 state within 1e-3 relative."""
    from oracle import dflash_oracle as O
    ops = _ops()
    q, k, v, alpha, beta, S0 = _config2_inputs(T)
    snap = T == 16
    o_ref, snaps_ref, S_ref = O.gdr_recurrence(q, k, v, alpha, beta, S0, keep_snapshots=snap)
    B, _, Hk, D = q.shape
    Hv = v.shape[2]
    out = torch.empty((B, Hv, D, D), device=DEV)
    snaps = torch.empty((B, T, Hv, D, D), device=DEV) if snap else None
    o = torch.empty((B, T, Hv, D), dtype=torch.bfloat16, device=DEV)
    ops.gdr_recurrence(q.to(DEV), k.to(DEV), v.to(DEV), alpha.to(DEV), beta.to(DEV), S0.to(DEV), state_out=out,
                       snapshots=snaps, o=o)
    rel = ((out.cpu() - S_ref).abs().max() / S_ref.abs().max()).item()
    o_err = (o.float().cpu() - o_ref).abs().max().item()
    print(f"config 2 T={T}: final state rel err {rel:.2e}, output max err {o_err:.2e} (max|o| "
          f"{o_ref.abs().max().item():.3f})")
    assert rel < 1e-3
    # o is stored as bf16: within one bf16 rounding of the fp32 reference
    assert o_err <= 2 ** -8 * o_ref.abs().max().item() + 1e-4
    if snap:
        rels = ((snaps.cpu() - snaps_ref).abs().max() / snaps_ref.abs().max()).item()
        assert rels < 1e-3
        assert torch.equal(snaps[:, -1], out)


@pytest.mark.parametrize("M,N,K", [(16, 6144, 2560), (3, 19456, 2560), (16, 151936, 2560)])
def test_gemm_fused_rmsnorm_prologue(M, N, K):
    """embed -> sumsq partials -> GEMM with the fused RMSNorm equals linear(rms_norm(x))."""
    from oracle import dflash_oracle as O
    ops = _ops()
    V = 1000
    table = _rand((V, K), 0.5, 30)
    tok = torch.randint(0, V, (M,), generator=torch.Generator().manual_seed(31), dtype=torch.int32)
    nw = (1.0 + 0.1 * _rand((K,), 1.0, 32).float()).bfloat16()
    w = _rand((N, K), 0.02, 33)
    x = torch.empty((M, K), dtype=torch.bfloat16, device=DEV)
    ss = torch.empty((M, K // 32), dtype=torch.float32, device=DEV)
    ops.embed(tok.to(DEV), table.to(DEV), out=x, sumsq_out=ss)
    assert torch.equal(x.cpu(), table[tok.long()])
    ref_ss = (table[tok.long()].float() ** 2).reshape(M, K // 32, 32).sum(-1)
    assert torch.allclose(ss.cpu(), ref_ss, rtol=1e-5)
    y = ops.gemm(x, w.to(DEV), norm_w=nw.to(DEV), sumsq_in=ss).float().cpu()
    ref = O.linear(O.rms_norm(table[tok.long()].float(), nw, 1e-6), w)
    assert (y - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-3


def test_gemm_sumsq_out_chain():
    """sumsq_out of a residual epilogue feeds the next GEMM's fused norm."""
    from oracle import dflash_oracle as O
    ops = _ops()
    M, H, K = 16, 2560, 4096
    x, w1, r, w2 = _rand((M, K), 1.0, 34), _rand((H, K), 0.02, 35), _rand((M, H), 1.0, 36), _rand((512, H), 0.02, 37)
    nw = torch.ones(H, dtype=torch.bfloat16)
    h = r.to(DEV).clone()
    ss = torch.empty((M, H // 32), dtype=torch.float32, device=DEV)
    ops.gemm(x.to(DEV), w1.to(DEV), ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss)
    ref_h = (r.float() + (x.float() @ w1.float().T).bfloat16().float()).bfloat16().float()
    assert torch.allclose(ss.cpu(), (h.float().cpu() ** 2).reshape(M, -1, 32).sum(-1), rtol=1e-4)
    y = ops.gemm(h, w2.to(DEV), norm_w=nw.to(DEV), sumsq_in=ss).float().cpu()
    ref = O.linear(O.rms_norm(ref_h, nw, 1e-6), w2)
    assert (y - ref).abs().max().item() <= 3e-2 * ref.abs().max().item() + 1e-3


def test_no_bounded_wait_gave_up():
    """After the kernels above no bounded device wait has expired."""
    assert _ops().device_error() == 0


# ---------------------------------------------------------------------------
# Qwen3.5 hybrid kernels
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("B,T,Hk,Hv,D", [(1, 16, 16, 48, 128), (3, 5, 2, 4, 64), (1, 128, 16, 48, 128)])
def test_gdn_prep_matches_oracle(B, T, Hk, Hv, D):
    from oracle import dflash_oracle as O
    ops = _ops()
    C = 2 * Hk * D + Hv * D
    vd = Hv * D
    ld = C + vd + 2 * Hv + 7  # row stride wider than the packed columns
    proj = _rand((B * T, ld), 1.0, 30)
    conv_w = _rand((C, 4), 0.3, 31)
    A_log = torch.log(torch.linspace(1.0, 16.0, Hv))
    dt_bias = torch.rand(Hv, generator=torch.Generator().manual_seed(32)) + 0.5
    conv_state = _rand((B, 3, C), 1.0, 33)
    window = torch.zeros((B, 3 + T + 4, C), dtype=torch.bfloat16, device=DEV)
    got = ops.gdn_prep(proj.to(DEV), conv_w.to(DEV), A_log.to(DEV), dt_bias.to(DEV), conv_state.to(DEV), B, T, Hk,
                       Hv, D, D, window=window)
    for b in range(B):
        rows = proj[b * T:(b + 1) * T]
        win = torch.cat([conv_state[b], rows[:, :C]], 0).float()
        q, k, v = O.gdn_conv_qkv(win, conv_w, Hk, Hv, D, D)
        g, beta = O.gdn_gates(rows[:, C + vd + Hv:C + vd + 2 * Hv], rows[:, C + vd:C + vd + Hv], A_log, dt_bias)
        sl = slice(b * T, (b + 1) * T)
        # one bf16 ulp where the conv sum lands on a rounding boundary
        for name, ref in (("q", q), ("k", k), ("v", v)):
            d = (got[name][sl].float().cpu() - ref).abs()
            assert d.max().item() <= 2 ** -7 * ref.abs().max().item(), name
            assert (d > 0).float().mean().item() < 0.01, name
        torch.testing.assert_close(got["g"][sl].cpu(), g, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(got["beta"][sl].cpu(), beta, rtol=1e-5, atol=1e-6)
        assert torch.equal(window[b, :3 + T].cpu(), win.bfloat16())


def test_gdn_rollback_copies_snapshot_and_conv_rows():
    ops = _ops()
    B, T, Hv, D, C = 3, 16, 4, 32, 96
    S = Hv * D * D
    snaps = torch.randn(B, T, Hv, D, D, device=DEV)
    state = torch.zeros(B, Hv, D, D, device=DEV)
    conv = torch.zeros(B, 3, C, dtype=torch.bfloat16, device=DEV)
    window = _rand((B, 3 + T + 2, C), 1.0, 34).to(DEV)
    acc_host = torch.tensor([[1] + [0] * 15, [7] + [0] * 15, [16] + [0] * 15], dtype=torch.int32)
    ops.gdn_rollback(state, snaps, conv, window, acc_host.to(DEV), 16, B, T, Hv, D, D, C)
    for b, a in enumerate((1, 7, 16)):
        assert torch.equal(state[b], snaps[b, a - 1])
        assert torch.equal(conv[b], window[b, a:a + 3])
    assert S == state[0].numel()


@pytest.mark.parametrize("M,H,D", [(16, 48, 128), (5, 4, 64)])
def test_gated_rmsnorm_matches_oracle(M, H, D):
    from oracle import dflash_oracle as O
    ops = _ops()
    o = _rand((M, H * D), 1.0, 35)
    z = _rand((M, H * D + 64), 1.0, 36)[:, 32:32 + H * D]  # strided view
    w = _rand((D,), 1.0, 37)
    got = ops.gated_rmsnorm(o.to(DEV), z.to(DEV), w.to(DEV), H, D, 1e-6).float().cpu()
    ref = O.gated_rms_norm(o.float().reshape(M, H, D), z.float().reshape(M, H, D), w, 1e-6).reshape(M, H * D)
    d = (got - ref).abs()
    assert d.max().item() <= 2 ** -7 * ref.abs().max().item()
    assert (d > 0).float().mean().item() < 0.01


@pytest.mark.parametrize("L,key_chunk", [(40, 0), (1000, 0), (1000, 2048), (1000, 256)])
def test_attention_hd256_gated_matches_oracle(L, key_chunk):
    """Qwen3.5 full attention: head_dim 256, output gate sigmoid(gate) applied in the
    combine, gate read from the interleaved [q | gate] q_proj rows."""
    from oracle import dflash_oracle as O
    ops = _ops()
    M, Hq, Hkv, hd, cap = 16, 24, 4, 256, 1024
    qg = _rand((M, Hq, 2 * hd), 1.0, 38)
    q = qg[:, :, :hd].contiguous()
    kc = _rand((1, Hkv, cap, hd), 1.0, 39)
    vc = _rand((1, Hkv, cap, hd), 1.0, 40)
    pos = torch.arange(L - M, L, dtype=torch.int32)
    qg_d = qg.reshape(M, Hq * 2 * hd).to(DEV)
    out = ops.attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos.to(DEV), True, max_kv=cap, gate=qg_d[:, hd:],
                        gate_head_stride=2 * hd, key_chunk=key_chunk).float().cpu()
    ref = O.attention(q.float(), kc[0].float(), vc[0].float(), [int(p) + 1 for p in pos], 1 / math.sqrt(hd))
    ref = O.bf16(ref * O.bf16(torch.sigmoid(qg[:, :, hd:].reshape(M, Hq * hd).float())))
    assert (out - ref).abs().max().item() < 2e-2
    plain = ops.attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos.to(DEV), True, max_kv=cap).float().cpu()
    ref_plain = O.attention(q.float(), kc[0].float(), vc[0].float(), [int(p) + 1 for p in pos], 1 / math.sqrt(hd))
    assert (plain - ref_plain).abs().max().item() < 2e-2


@pytest.mark.parametrize("rows,seq_rows_arg,key_chunk", [(8, 8, 0), (5, 5, 0), (3, 0, 0), (16, 16, 0), (1, 1, 0),
                                                        (16, 16, 1024), (5, 5, 192), (8, 8, 64)])
def test_attention_batched_sequences_share_tiles(rows, seq_rows_arg, key_chunk):
    """Several sequences' verify rows inside one 16-row tile each read their own cache."""
    from oracle import dflash_oracle as O
    ops = _ops()
    B, Hq, Hkv, hd, cap = 7, 8, 2, 128, 256
    q = _rand((B * rows, Hq, hd), 1.0, 41)
    kc = _rand((B, Hkv, cap, hd), 1.0, 42)
    vc = _rand((B, Hkv, cap, hd), 1.0, 43)
    starts = [17 + 29 * b for b in range(B)]
    pos = torch.tensor([starts[b] + i for b in range(B) for i in range(rows)], dtype=torch.int32)
    row_seq = torch.arange(B * rows, dtype=torch.int32) // rows
    out = ops.attention(q.to(DEV), kc.to(DEV), vc.to(DEV), pos.to(DEV), True, max_kv=cap, row_seq=row_seq.to(DEV),
                        seq_rows=seq_rows_arg, key_chunk=key_chunk).float().cpu()
    for b in range(B):
        sl = slice(b * rows, (b + 1) * rows)
        ref = O.attention(q[sl].float(), kc[b].float(), vc[b].float(), [int(p) + 1 for p in pos[sl]],
                          1 / math.sqrt(hd))
        assert (out[sl] - ref).abs().max().item() < 2e-2, b
    assert ops.device_error() == 0


# ---------------------------------------------------------------------------
# Wide GEMM (whole-K tiles for many rows)
# ---------------------------------------------------------------------------
def _wide_ws(split: int = 1):
    from dflash_b200 import ops
    return ops.Workspace(torch.device(DEV), wide=True, wide_split=split)


@pytest.mark.parametrize("M,N,K", [(1024, 6144, 2560), (1024, 2560, 9728), (300, 512, 256), (16, 1536, 2560),
                                   (1000, 2560, 4096)])
def test_wide_gemm_store_matches_fp32(M, N, K):
    ops = _ops()
    x = _rand((M, K), 1.0, 50)
    w = _rand((N, K), 0.02, 51)
    y = ops.gemm(x.to(DEV), w.to(DEV), ws=_wide_ws()).float().cpu()
    ref = x.float() @ w.float().T
    err = (y - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("M,split", [(512, 1), (128, 4)])
def test_wide_gemm_epilogues_and_norm(M, split):
    """Residual + tap + sum-of-squares, SiLU·up and argmax epilogues, and the RMSNorm
    prologue, in the wide form (whole-K tiles, and fixed split-K ranges) against the
    weight-streaming form's definitions."""
    from oracle import dflash_oracle as O
    from dflash_b200.weights import pack_gate_up
    ops = _ops()
    ws = _wide_ws(split)
    H, I = 2560, 9728
    x = _rand((M, H), 1.0, 52).to(DEV)
    res = _rand((M, H), 1.0, 53).to(DEV)
    w = _rand((H, H), 0.02, 54).to(DEV)
    tap = torch.empty((M, H), dtype=torch.bfloat16, device=DEV)
    ss = torch.empty((M, H // 32), dtype=torch.float32, device=DEV)
    y = ops.gemm(x, w, ops.EPI_RESIDUAL, residual=res, out2=tap, ws=ws, sumsq_out=ss)
    ref = O.bf16(res.float().cpu() + O.bf16(x.float().cpu() @ w.float().cpu().T))
    assert (y.float().cpu() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    assert torch.equal(tap, y)
    yf = y.float()
    torch.testing.assert_close(ss, (yf * yf).reshape(M, H // 32, 32).sum(-1), rtol=1e-4, atol=1e-3)
    # RMSNorm prologue from the sum-of-squares partials, into a SiLU·up projection
    nw = _rand((H,), 1.0, 55).to(DEV)
    g, u = _rand((I, H), 0.02, 56).to(DEV), _rand((I, H), 0.02, 57).to(DEV)
    act = ops.gemm(y, pack_gate_up(g, u), ops.EPI_SILU_MUL, ws=ws, norm_w=nw, sumsq_in=ss, eps=1e-6)
    xn = O.rms_norm(yf.cpu(), nw.cpu(), 1e-6)
    gr, ur = O.bf16(xn @ g.float().cpu().T), O.bf16(xn @ u.float().cpu().T)
    ref_act = O.silu_mul(gr, ur)
    assert (act.float().cpu() - ref_act).abs().max().item() <= 3e-2 * ref_act.abs().max().item()
    # argmax
    V = 151936
    wl = _rand((V, H), 0.02, 58).to(DEV)
    part = ops.gemm(y[:64].contiguous(), wl, ops.EPI_ARGMAX, ws=ws)
    got = ops.argmax_reduce(part).cpu()
    logits = ops.gemm(y[:64].contiguous(), wl, ws=ws).float()
    assert torch.equal(got, logits.argmax(-1).int().cpu())


@pytest.mark.parametrize("split,N", [(1, 6144), (4, 2560)])
def test_wide_gemm_row_invariance(split, N):
    """A row's wide-GEMM result is the same bits whatever M (and tile width) is, for a
    given split of K."""
    ops = _ops()
    ws = _wide_ws(split)
    x = _rand((1024, 2560), 1.0, 59).to(DEV)
    w = ops.pack_weight(_rand((N, 2560), 0.02, 60).to(DEV))
    full = ops.gemm(x, w, ws=ws)
    ref = x.float() @ _rand((N, 2560), 0.02, 60).to(DEV).float().T
    assert (full.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    for M in (8, 16, 64, 200, 256):
        part = ops.gemm(x[:M].contiguous(), w, ws=ws)
        assert torch.equal(part, full[:M]), M
    assert ops.device_error() == 0


@pytest.mark.parametrize("wide", [False, True])
def test_gemm_fp32_store(wide):
    """DFL_EPI_STORE_F32 (tensor-parallel partials): the fp32 accumulator, whose bf16
    rounding is the bf16 store's output."""
    ops = _ops()
    ws = ops.Workspace(torch.device(DEV), wide=wide)
    M, N, K = 300 if wide else 16, 2560, 4096
    x = _rand((M, K), 1.0, 61).to(DEV)
    w = ops.pack_weight(_rand((N, K), 0.02, 62).to(DEV))
    yf = ops.gemm(x, w, ops.EPI_STORE_F32, ws=ws)
    yb = ops.gemm(x, w, ws=ws)
    assert yf.dtype == torch.float32
    assert torch.equal(yf.bfloat16(), yb)
    ref = x.float() @ _rand((N, K), 0.02, 62).to(DEV).float().T
    assert (yf - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_wide_gemm_partials_slabs():
    """DFL_EPI_PARTIALS leaves the K-range partials unsummed; summed in slab order they
    are the split GEMM's fp32 result bit for bit."""
    ops = _ops()
    ws = _wide_ws(4)
    M, N, K = 128, 2560, 9728
    x = _rand((M, K), 1.0, 63).to(DEV)
    w = ops.pack_weight(_rand((N, K), 0.02, 64).to(DEV))
    S = ops.wide_split(N, K, ws)
    assert S == 4
    slabs = ops.gemm(x, w, ops.EPI_PARTIALS, ws=ws)
    assert slabs.shape == (S, M, N)
    full = ops.gemm(x, w, ops.EPI_STORE_F32, ws=ws)
    acc = torch.zeros_like(full)
    for s in range(S):
        acc += slabs[s]
    assert torch.equal(acc, full)


def test_gdr_replay_of_accepted_prefix_equals_snapshot():
    """Rollback by replay (tokens = each sequence's accepted length, read on the
    device) leaves exactly the state the per-token snapshot of that token holds."""
    ops = _ops()
    B, T, Hk, Hv, D = 3, 16, 2, 4, 128
    g = torch.Generator().manual_seed(7)
    q = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).bfloat16().to(DEV)
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=g), dim=-1).bfloat16().to(DEV)
    v = torch.randn(B, T, Hv, D, generator=g).bfloat16().to(DEV)
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, Hv, generator=g))).to(DEV)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g)).to(DEV)
    S0 = (torch.randn(B, Hv, D, D, generator=g) * 0.1).to(DEV)
    snaps = torch.empty((B, T, Hv, D, D), device=DEV)
    o_full = torch.empty((B, T, Hv, D), dtype=torch.bfloat16, device=DEV)
    ops.gdr_recurrence(q, k, v, alpha, beta, S0, snapshots=snaps, o=o_full)
    state = S0.clone()
    acc = torch.tensor([[5, 0, 0], [16, 0, 0], [0, 0, 0]], dtype=torch.int32, device=DEV)  # stride 3
    ops.gdr_recurrence(None, k, v, alpha, beta, state, state_out=state, tokens=acc, tokens_stride=3)
    assert torch.equal(state[0], snaps[0, 4])
    assert torch.equal(state[1], snaps[1, 15])
    assert torch.equal(state[2], S0[2])  # no accepted token: untouched
    # outputs of a verify pass without state writes equal those of the snapshot pass
    o2 = torch.empty_like(o_full)
    ops.gdr_recurrence(q, k, v, alpha, beta, S0, o=o2)
    assert torch.equal(o2, o_full)


@pytest.mark.parametrize("case", ["single_straddle", "batched16", "rows4", "finished_rows"])
def test_attention_qkv_fused_matches_append_then_attention(case):
    """dfl_attention_qkv (norm + RoPE + append inside the attention launch, mma.sync form)
    against dfl_qkv_rope_append followed by dfl_attention: both caches bit for bit; the
    outputs within one bf16 rounding when dfl_attention takes its tensor-core form (a
    different summation order), bit for bit otherwise."""
    from dflash_b200 import ops
    from dflash_b200.model import rope_inv_freq
    g = torch.Generator(device="cuda").manual_seed(11)
    Hq, Hkv, hd, eps = 32, 8, 128, 1e-6
    row_seq = None
    if case == "single_straddle":
        B, rows, starts, kc = 1, 16, [1016], 128
    elif case == "batched16":
        B, rows, starts, kc = 6, 16, [5, 700, 1023, 2048, 130, 3000], 1024
    else:
        B, rows, starts, kc = 8, 4, [9, 64, 127, 500, 1, 1999, 250, 1000], 128
    M = B * rows
    cap = max(starts) + rows + 8
    if B > 1:
        row_seq = torch.arange(M, device="cuda", dtype=torch.int32) // rows
    pos = torch.tensor([s + i for s in starts for i in range(rows)], dtype=torch.int32, device="cuda")
    if case == "finished_rows":
        pos[4:8] = -1  # a finished sequence: no append, no output
    qkv = (torch.randn((M, (Hq + 2 * Hkv) * hd), device="cuda", generator=g) * 2).bfloat16()
    q_norm = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).bfloat16()
    k_norm = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).bfloat16()
    inv_freq = rope_inv_freq(hd, 1e6, "cuda")
    kc0 = torch.randn((B, Hkv, cap, hd), device="cuda", generator=g).bfloat16()
    vc0 = torch.randn((B, Hkv, cap, hd), device="cuda", generator=g).bfloat16()
    max_kv = max(starts) + rows
    ws = ops.Workspace(torch.device("cuda"))
    k1, v1 = kc0.clone(), vc0.clone()
    q = ops.qkv_rope_append(qkv, pos, q_norm, k_norm, inv_freq, k1, v1, Hq, Hkv, hd, hd, eps, row_seq=row_seq)
    o1 = ops.attention(q, k1, v1, pos, True, max_kv=max_kv, row_seq=row_seq, ws=ws, seq_rows=rows if B > 1 else 0,
                       key_chunk=kc)
    k2, v2 = kc0.clone(), vc0.clone()
    assert ops.fused_attention_ok(M, row_seq, rows if B > 1 else 0, hd, hd)
    o2 = ops.attention_qkv(qkv, pos, q_norm, k_norm, inv_freq, k2, v2, Hq, eps, max_kv, row_seq=row_seq, ws=ws,
                           seq_rows=rows if B > 1 else 0, key_chunk=kc)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    live = pos >= 0
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    d = (o1[live].float() - o2[live].float()).abs()
    scale = o1[live].float().abs().max().item()
    assert d.max().item() <= 2 ** -7 * scale, d.max().item()


@pytest.mark.parametrize("M", [1, 16])
def test_gemm_chain_matches_separate_launches(M):
    """One dfl_gemm_chain launch of a layer's projections at the Qwen3-4B shape (o_proj with
    residual, gate/up with the fused RMSNorm and SiLU, down with residual + tap, the next
    qkv with RMSNorm, the lm_head argmax) against the same ops as separate dfl_gemm_bf16
    launches: outputs within one bf16 rounding (the two forms split K differently), argmax
    equal except at near-ties, and three launches in a row give identical bits (the
    kernel leaves its counters ready for the next launch)."""
    ops = _ops()
    H, F, Nq, V = 2560, 9728, 6144, 151936
    g = torch.Generator().manual_seed(40 + M)
    w_o = ops.pack_weight(_rand((H, 4096), 0.02, 41).to(DEV))
    w_gu = ops.pack_weight(_rand((2 * F, H), 0.02, 42).to(DEV))
    w_dn = ops.pack_weight(_rand((H, F), 0.02, 43).to(DEV))
    w_q = ops.pack_weight(_rand((Nq, H), 0.02, 44).to(DEV))
    w_lm = ops.pack_weight(_rand((V, H), 0.02, 45).to(DEV))
    nw1 = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16().to(DEV)
    nw2 = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16().to(DEV)
    nw3 = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16().to(DEV)
    attn = torch.randn(M, 4096, generator=g).bfloat16().to(DEV)
    h0 = torch.randn(M, H, generator=g).bfloat16().to(DEV)

    def run(chain):
        h = h0.clone()
        ss = torch.zeros(M, H // 32, device=DEV)
        act = torch.empty(M, F, dtype=torch.bfloat16, device=DEV)
        qkv = torch.empty(M, Nq, dtype=torch.bfloat16, device=DEV)
        tap = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
        part = torch.empty(M, ops.argmax_tiles(V), 2, device=DEV)
        specs = [dict(x=attn, w=w_o, epilogue=ops.EPI_RESIDUAL, residual=h, out=h, sumsq_out=ss),
                 dict(x=h, w=w_gu, epilogue=ops.EPI_SILU_MUL, out=act, norm_w=nw1, sumsq_in=ss),
                 dict(x=act, w=w_dn, epilogue=ops.EPI_RESIDUAL, residual=h, out=h, out2=tap, sumsq_out=ss),
                 dict(x=h, w=w_q, out=qkv, norm_w=nw2, sumsq_in=ss),
                 dict(x=h, w=w_lm, epilogue=ops.EPI_ARGMAX, argmax_partials=part, norm_w=nw3, sumsq_in=ss)]
        if chain:
            ops.gemm_chain([ops.chain_op(**sp) for sp in specs])
        else:
            for sp in specs:
                sp = dict(sp)
                x, w = sp.pop("x"), sp.pop("w")
                ops.gemm(x, w, **sp)
        torch.cuda.synchronize()
        return h.float().cpu(), act.float().cpu(), qkv.float().cpu(), tap.float().cpu(), ops.argmax_reduce(part).cpu()

    ref = run(False)
    got = run(True)
    for name, a, b in zip(("h", "act", "qkv", "tap"), got[:4], ref[:4]):
        d = (a - b).abs()
        # rounding-order differences only: most values identical, the rest within a few ulps
        # of the row's scale (a residual sum can cancel, so not of the element itself)
        scale = torch.pow(2.0, torch.floor(torch.log2(b.abs().amax(1, keepdim=True).clamp_min(2.0 ** -126))) - 7)
        eq = (d == 0).float().mean().item()
        print(f"chain vs separate, M={M}, {name}: max diff {d.max().item():.4f}, equal {eq:.3f}")
        assert bool((d <= 4 * scale).all()) and eq >= 0.8, name
    assert (got[4] == ref[4]).float().mean().item() >= 0.9
    again = [run(True) for _ in range(2)]
    for r in again:
        for a, b in zip(r, got):
            assert torch.equal(a, b)
    assert ops.device_error() == 0


@pytest.mark.parametrize("N,K", [(256, 256), (1536, 256), (256, 768), (4096, 256)])
def test_gemm_chain_ops_with_fewer_units_than_ctas(N, K):
    """Ops whose 128 x 64 weight units are fewer than the chain's CTAs (the tiny
    configuration's projections) run on the first CTAs only; three chain launches in a row
    give the separate launch's values within one rounding and identical bits to each other."""
    ops = _ops()
    g = torch.Generator().manual_seed(N + K)
    x = torch.randn(16, K, generator=g).bfloat16().to(DEV)
    w = ops.pack_weight((torch.randn(N, K, generator=g) * 0.02).bfloat16().to(DEV))
    y1 = ops.gemm(x, w)
    outs = []
    for _ in range(3):
        y2 = torch.zeros_like(y1)
        ops.gemm_chain([ops.chain_op(x, w, out=y2)])
        outs.append(y2)
    torch.cuda.synchronize()
    d = (y1.float() - outs[0].float()).abs()
    assert d.max().item() <= 2 ** -7 * y1.float().abs().max().item(), d.max().item()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    assert ops.device_error() == 0


@pytest.mark.parametrize("case", ["qwen3_4b", "qwen3_4b_paged", "two_seqs", "rows_20", "hd64"])
def test_gemm_qkv_rope_matches_separate_calls(case):
    """dfl_gemm_qkv_rope (the QKV projection with the q/k head norm + RoPE + cache append
    after its split-K reduction, in the GEMM launch) against dfl_gemm_bf16 followed by
    dfl_qkv_rope_append on the same inputs: projection rows, q and both caches bit for
    bit. At the Qwen3-4B verify shape the append kernel must not run (the fused form);
    20 rows (two row tiles) and head_dim 64 take the two-kernel form inside the call."""
    from dflash_b200.weights import rope_inv_freq
    ops = _ops()
    H, Hq, Hkv, hd, M = 2560, 32, 8, 128, 16
    if case == "rows_20":
        M = 20
    if case == "hd64":
        H, Hq, Hkv, hd = 256, 4, 2, 64
    n_seq = 2 if case == "two_seqs" else 1
    N = (Hq + 2 * Hkv) * hd
    x = _rand((M, H), 1.0, 60).to(DEV)
    w = ops.PackedWeight(_rand((N, H), 0.02, 61).to(DEV))
    in_norm = (1.0 + 0.1 * _rand((H,), 1.0, 62).float()).bfloat16().to(DEV)
    qn, kn = _rand((hd,), 1.0, 63).to(DEV), _rand((hd,), 1.0, 64).to(DEV)
    ss = (x.float() ** 2).reshape(M, H // 32, 32).sum(-1).contiguous()
    inv = rope_inv_freq(hd, 1e6).to(DEV)
    if n_seq == 2:
        pos = torch.tensor(list(range(300, 308)) + list(range(811, 819)), dtype=torch.int32, device=DEV)
        row_seq = torch.tensor([0] * 8 + [1] * 8, dtype=torch.int32, device=DEV)
    else:
        pos = torch.arange(1000, 1000 + M, dtype=torch.int32, device=DEV)
        pos[3] = -1  # a skipped row
        row_seq = None
    cap = 1152
    paged = case == "qwen3_4b_paged"
    pg = {}
    if paged:
        n_pages = cap // 64
        perm = torch.randperm(n_pages, generator=torch.Generator().manual_seed(65)).to(torch.int32).to(DEV)
        pg = {"page_table": perm.view(1, -1), "page_size": 64}

    def caches():
        shape = (cap // 64, Hkv, 64, hd) if paged else (n_seq, Hkv, cap, hd)
        return torch.zeros(shape, dtype=torch.bfloat16, device=DEV), torch.zeros(shape, dtype=torch.bfloat16,
                                                                                   device=DEV)

    kc0, vc0 = caches()
    qkv0 = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out=qkv0, norm_w=in_norm, sumsq_in=ss)
    q0 = ops.qkv_rope_append(qkv0, pos, qn, kn, inv, kc0, vc0, Hq, Hkv, hd, hd, 1e-6, row_seq=row_seq, **pg)
    kc1, vc1 = caches()
    qkv1 = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    q1 = torch.zeros((M, Hq, hd), dtype=torch.bfloat16, device=DEV)
    q1[3] = q0[3]  # the skipped row is left as it was
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        ops.gemm_qkv_rope(x, w, qkv1, pos, qn, kn, inv, kc1, vc1, q1, Hq, Hkv, hd, 1e-6, norm_w=in_norm, sumsq_in=ss,
                          row_seq=row_seq, **pg)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert ops.device_error() == 0
    assert torch.equal(qkv1, qkv0)
    assert torch.equal(q1, q0)
    assert torch.equal(kc1, kc0) and torch.equal(vc1, vc0)
    assert kc1.abs().sum().item() > 0
    appended = any("qkv_rope_append" in n for n in names)
    print(case, "kernels:", sorted(set(n[:40] for n in names)))
    if names:
        assert appended == (case in ("rows_20", "hd64")), names


@pytest.mark.parametrize("case", ["draft_4b", "draft_4b_paged", "rows_20"])
def test_gemm_kv_append_layers_matches_separate_calls(case):
    """dfl_gemm_kv_append_layers (the draft's stacked context K/V projection with every
    layer's k_norm + RoPE + append after the split-K reduction, in the GEMM launch) against
    dfl_gemm_bf16 followed by one dfl_qkv_rope_append per layer: projection rows and every
    layer's caches bit for bit. 20 rows take the per-layer append launches inside the call."""
    from dflash_b200.weights import rope_inv_freq
    ops = _ops()
    L, H, Hkv, hd = 5, 2560, 8, 128
    M = 20 if case == "rows_20" else 16
    per = 2 * Hkv * hd
    N = L * per
    x = _rand((M, H), 1.0, 70).to(DEV)
    w = ops.PackedWeight(_rand((N, H), 0.02, 71).to(DEV))
    hn = (1.0 + 0.1 * _rand((H,), 1.0, 72).float()).bfloat16().to(DEV)
    kns = [_rand((hd,), 1.0, 73 + l).to(DEV) for l in range(L)]
    ss = (x.float() ** 2).reshape(M, H // 32, 32).sum(-1).contiguous()
    inv = rope_inv_freq(hd, 1e6).to(DEV)
    pos = torch.arange(700, 700 + M, dtype=torch.int32, device=DEV)
    pos[5] = -1
    cap = 1024
    paged = case == "draft_4b_paged"
    pg = {}
    if paged:
        perm = torch.randperm(cap // 64, generator=torch.Generator().manual_seed(79)).to(torch.int32).to(DEV)
        pg = {"page_table": perm.view(1, -1), "page_size": 64}
    shape = (L, cap // 64, Hkv, 64, hd) if paged else (L, 1, Hkv, cap, hd)
    kc0, vc0 = torch.zeros(shape, dtype=torch.bfloat16, device=DEV), torch.zeros(shape, dtype=torch.bfloat16, device=DEV)
    kv0 = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out=kv0, norm_w=hn, sumsq_in=ss)
    for l in range(L):
        ops.qkv_rope_append(kv0[:, l * per:(l + 1) * per], pos, kns[l], kns[l], inv, kc0[l], vc0[l], 0, Hkv, hd, hd,
                            1e-6, do_q=False, **pg)
    kc1, vc1 = torch.zeros_like(kc0), torch.zeros_like(vc0)
    kv1 = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        ops.gemm_kv_append_layers(x, w, kv1, pos, kns, inv, kc1, vc1, Hkv, hd, 1e-6, norm_w=hn, sumsq_in=ss, **pg)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert ops.device_error() == 0
    assert torch.equal(kv1, kv0)
    assert torch.equal(kc1, kc0) and torch.equal(vc1, vc0)
    assert kc1.abs().sum().item() > 0
    n_append = sum("qkv_rope_append" in n for n in names)
    print(case, "append launches:", n_append)
    if names:
        assert n_append == (L if case == "rows_20" else 0), names
