"""dfl_gemm_bf16_noalloc: the GEMM entry point for callers that cannot allocate device
memory (host callbacks, plugins whose host application owns all allocations, engines
that forbid cudaMalloc after start-up). Its split-K scratch is an array built into the
library. Called through the C ABI; output must match dfl_gemm_bf16 (which takes a
caller workspace) on two calls in a row. Collected last on purpose."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _rand(shape, std, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K,epi", [(16, 2560, 4096, 1), (5, 6144, 2560, 0), (16, 151936, 2560, 3)])
def test_noalloc_matches_workspace_gemm(M, N, K, epi):
    from dflash_b200 import _lib, ops
    lib = _lib.load()
    dev = "cuda"
    x = _rand((M, K), 1.0, 1).to(dev)
    w = ops.pack_weight(_rand((N, K), 0.02, 2).to(dev))
    r = _rand((M, N), 1.0, 3).to(dev)
    stream = torch.cuda.current_stream().cuda_stream
    argmax = epi == ops.EPI_ARGMAX

    def run(noalloc):
        y = r.clone() if epi == ops.EPI_RESIDUAL else torch.zeros((M, N), dtype=torch.bfloat16, device=dev)
        part = torch.zeros((M, N // 32, 2), dtype=torch.float32, device=dev) if argmax else None
        res = y if epi == ops.EPI_RESIDUAL else None
        args = [x.data_ptr(), K, w.data_ptr(), M, N, K, epi, res.data_ptr() if res is not None else None,
                N if res is not None else 0, None if argmax else y.data_ptr(), 0 if argmax else N, None, 0,
                part.data_ptr() if argmax else None, None, None, 0, 1e-6, None]
        if noalloc:
            status = lib.dfl_gemm_bf16_noalloc(*args, stream)
        else:
            ws = ops.workspace(torch.device(dev))
            need = int(lib.dfl_gemm_workspace_bytes(M, N, K, epi))
            ws.ensure_gemm(need)
            status = lib.dfl_gemm_bf16(*args, ws.gemm.data_ptr(), ws.gemm.numel(), stream)
        assert status == 0, lib.dfl_last_error()
        torch.cuda.synchronize()
        return (ops.argmax_reduce(part) if argmax else y).cpu()

    ref = run(False)
    for _ in range(2):  # two calls in a row share (and must reset) the built-in scratch
        got = run(True)
        # the same kernel with the same split points and reduction order: identical bits
        assert torch.equal(got, ref)
    code = ctypes.c_int(0)
    assert lib.dfl_device_error(ctypes.byref(code), 1, stream) == 0 and code.value == 0


def test_noalloc_rejects_oversize():
    from dflash_b200 import _lib
    lib = _lib.load()
    st = lib.dfl_gemm_bf16_noalloc(1, 2560, 1, 17, 2560, 2560, 0, None, 0, 1, 2560, None, 0, None, None, None, 0,
                                   1e-6, None, None)
    assert st == 2 and b"scratch limit" in lib.dfl_last_error()
    assert lib.dfl_gemm_noalloc_scratch_bytes() < 8 << 20
    st = lib.dfl_gemm_bf16_noalloc(1, 2560, 1, -1, 2560, 2560, 0, None, 0, 1, 2560, None, 0, None, None, None, 0,
                                   1e-6, None, None)
    assert st == 1 and b"negative size" in lib.dfl_last_error()
