"""Host-side rules of the device paths (no GPU): when the fused append + attention launch
applies, and the argument checks of the batched stream."""
import pytest

from dflash_b200 import ops


def test_fused_attention_applies_only_when_sequences_sit_in_one_tile():
    assert ops.fused_attention_ok(16, None, 0, 128, 128)       # one sequence, one tile
    assert not ops.fused_attention_ok(17, None, 0, 128, 128)   # one sequence over two tiles
    assert not ops.fused_attention_ok(128, None, 0, 128, 128)  # a prefill chunk
    rs = object()  # any row_seq
    for rows in (1, 2, 4, 8, 16):
        assert ops.fused_attention_ok(64, rs, rows, 128, 128)
    for rows in (0, 3, 5, 12, 32):
        assert not ops.fused_attention_ok(64, rs, rows, 128, 128)
    assert not ops.fused_attention_ok(16, None, 0, 256, 64)    # Qwen3.5 gated heads (partial rotary)
    assert not ops.fused_attention_ok(16, None, 0, 128, 64)


def test_batch_stream_checks_arguments():
    from dflash_b200.runtime import dflash_generate_batch_stream
    assert list(dflash_generate_batch_stream(None, None, [], [], 0.0, set())) == []
    with pytest.raises(ValueError):
        list(dflash_generate_batch_stream(None, None, [[1, 2]], [4, 5], 0.0, set()))
