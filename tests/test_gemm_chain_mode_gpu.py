"""The GEMM-chain mode of the forwards, which is opt-in (DFLASH_B200_GEMM_CHAIN=1, read
once per process): the lossless, oracle-parity, paged and C-level-driver tests rerun in a
child process with it switched on."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_model_suite_with_gemm_chains(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ, DFLASH_B200_GEMM_CHAIN="1")
    files = ["test_spec_gpu.py", "test_draft_gpu.py", "test_paged_gpu.py", "test_step_abi_gpu.py"]
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider"] + [os.path.join(HERE, f) for f in files]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    print(r.stdout[-3000:], r.stderr[-2000:])
    assert r.returncode == 0
