"""The tensor-core (tcgen05 / TMEM / TMA) attention form, which is opt-in
(DFLASH_B200_ATTN_TC=1, read once per process): the attention and paged-cache tests of
this suite rerun in a child process with it switched on -- oracle parity, row invariance,
batched tiles, paged caches and the fused-append comparison."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_attention_suite_with_tensor_core_form(lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ, DFLASH_B200_ATTN_TC="1")
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-k", "attention or paged",
           os.path.join(HERE, "test_kernels_gpu.py"), os.path.join(HERE, "test_paged_gpu.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-2000:])
    assert r.returncode == 0
