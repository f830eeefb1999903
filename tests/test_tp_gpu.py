"""Tensor-parallel Qwen3.5 hybrid on 2+ GPUs (config 5's TP path): runs
tests/tp_worker.py under torch.distributed.run, one rank per GPU. Skipped on a
single-GPU box."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("world", [2])
def test_tp_hybrid_matches_single_gpu(lib, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--nproc-per-node", str(world),
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0 and "TP_OK" in r.stdout


def test_tp_all_sum_wait_gives_up_and_reports(lib):
    """The all-sum's bounded wait on one GPU: call it as rank 0 of 2 ranks where rank 1's
    flag is never published (its "peer" buffers are plain local memory that no other
    kernel writes). The kernel must give up after its wait limit (about 2 s), record
    device error 401, leave h untouched and return; the context stays usable: after the
    error is read and cleared, a 1-rank call sums normally."""
    import ctypes
    import time
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = "cuda"
    M, H = 4, 512
    g = torch.Generator().manual_seed(0)
    part0 = torch.randn(M, H, generator=g).to(dev)
    part1 = torch.randn(M, H, generator=g).to(dev)
    h0 = torch.randn(M, H, generator=g).to(torch.bfloat16).to(dev)
    h = h0.clone()
    flags = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(2)]
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    code = ctypes.c_int(0)
    assert lib.dfl_device_error(ctypes.byref(code), 1, stream) == 0

    def call(n_ranks):
        parts = (ctypes.c_void_p * 2)(part0.data_ptr(), part1.data_ptr())
        fl = (ctypes.c_void_p * 2)(flags[0].data_ptr(), flags[1].data_ptr())
        st = lib.dfl_tp_reduce_residual(parts, fl, epoch.data_ptr(), done.data_ptr(), 0, n_ranks, 1, 0,
                                        h.data_ptr(), H, None, 0, None, M, H, stream)
        assert st == 0, lib.dfl_last_error()

    t0 = time.perf_counter()
    call(2)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert lib.dfl_device_error(ctypes.byref(code), 1, stream) == 0
    print(f"wait gave up after {waited:.2f} s with device error {code.value}")
    assert code.value == 401
    assert torch.equal(h, h0)
    assert 0.2 < waited < 30
    # cleared, and the next (single-rank) call completes and sums
    assert lib.dfl_device_error(ctypes.byref(code), 0, stream) == 0 and code.value == 0
    call(1)
    torch.cuda.synchronize()
    assert lib.dfl_device_error(ctypes.byref(code), 1, stream) == 0 and code.value == 0
    ref = (h0.float() + part0.to(torch.bfloat16).float()).to(torch.bfloat16)
    assert torch.equal(h, ref)


@pytest.mark.parametrize("M", [128, 16])
def test_tp_all_sum_norm_rows_equal_the_projection_norm(lib, M):
    """One GPU, one rank: dfl_tp_reduce_residual_norm gives the same h, tap and sums of
    squares as dfl_tp_reduce_residual, and its normed rows fed to a projection without a
    norm give the same bits as that projection norming h itself (wide form at 128 rows,
    weight-streaming form at 16), the claim that lets the tensor-parallel forward skip the
    projection's norm pass."""
    from dflash_b200 import ops
    from dflash_b200.tp import TPComm
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda")
    H, N = 5120, 2048
    g = torch.Generator(device=dev).manual_seed(5)
    h0 = torch.randn((M, H), generator=g, device=dev).bfloat16()
    part = torch.randn((M, H), generator=g, device=dev) * 0.5
    nw = (1.0 + 0.1 * torch.randn((H,), generator=g, device=dev)).bfloat16()
    w = ops.PackedWeight((torch.randn((N, H), generator=g, device=dev) * 0.02).bfloat16())
    comm = TPComm(0, 1, dev, max_rows=M, hidden=H)
    try:
        outs = []
        for with_norm in (False, True):
            h = h0.clone()
            tap = torch.empty_like(h)
            ss = torch.empty((M, H // 32), dtype=torch.float32, device=dev)
            xn = torch.empty_like(h)
            comm.partial(0, M).copy_(part)
            if with_norm:
                comm.reduce_residual(0, h, tap, ss, M, norm_w=nw, eps=1e-6, xn=xn)
            else:
                comm.reduce_residual(0, h, tap, ss, M)
            torch.cuda.synchronize()
            outs.append((h, tap, ss, xn))
        assert ops.device_error() == 0
        (h_a, tap_a, ss_a, _), (h_b, tap_b, ss_b, xn_b) = outs
        assert torch.equal(h_a, h_b) and torch.equal(tap_a, tap_b) and torch.equal(ss_a, ss_b)
        ws = ops.Workspace(dev, wide=M > 16)
        y_norm = ops.gemm(h_a, w, ws=ws, norm_w=nw, sumsq_in=ss_a, eps=1e-6)
        y_rows = ops.gemm(xn_b, w, ws=ws)
        assert torch.equal(y_norm, y_rows)
    finally:
        comm.close()
