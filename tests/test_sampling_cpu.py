"""Host side of temperature sampling (no GPU): the key mixer is splitmix64's published
finaliser, keys are distinct per (seed, tag, sequence, position), temperature 0 is the
argmax (runtime.py:22-29), and sampling without a CUDA device fails loudly."""
import pytest
import torch


def test_mix64_is_splitmix64():
    """splitmix64 seeded with 0 yields 0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F
    (the state advances by the golden gamma; mix64 adds it before mixing)."""
    from dflash_b200 import ops
    gamma = 0x9E3779B97F4A7C15
    want = [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]
    assert [ops.mix64((i * gamma) & ops._M64) for i in range(3)] == want


def test_sample_keys_are_distinct():
    from dflash_b200 import ops
    keys = {ops.sample_key(s, t, b, p) for s in (0, 1) for t in (ops.SAMPLE_TAG_DRAFT, ops.SAMPLE_TAG_TARGET)
            for b in range(8) for p in range(512)}
    assert len(keys) == 2 * 2 * 8 * 512
    assert all(0 <= k < 1 << 64 for k in keys)
    # the int64 view the device reads is the same 64 bits
    k = ops.sample_key(3, 2, 1, 99)
    assert ops.keys_tensor([k], "cpu").item() & ops._M64 == k


def test_temperature_zero_is_argmax():
    from dflash_b200.runtime import sample_tokens
    g = torch.Generator().manual_seed(0)
    logits = torch.randn((3, 5, 97), generator=g)
    got = sample_tokens(logits, 0.0)
    assert got.shape == (3, 5)
    assert torch.equal(got.long(), logits.argmax(-1))


def test_sampling_needs_cuda():
    from dflash_b200.runtime import sample_tokens
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(Exception):
        sample_tokens(torch.randn(2, 64), 0.8, seed=1)
