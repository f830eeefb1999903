"""Host-side API pieces that need no GPU: the reference-shaped ``load_draft_model``
return and the draft quantization round trip (draft.py:224-252, api.py:62-66)."""
import pytest
import torch


def test_load_draft_model_returns_draft_and_path():
    from dflash_b200.api import DraftCheckpoint, load_draft_model
    draft, path = load_draft_model("random:tiny", seed=0)
    assert isinstance(draft, DraftCheckpoint)
    assert path == "random:tiny"
    assert draft.block_size == 8 and draft.target_layer_ids == [1, 3] and draft.mask_token_id == 4095


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("group", [32, 64])
def test_quantize_dequantize_affine(bits, group):
    from dflash_b200.api import quantize_dequantize
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(64, 256, generator=g) * 0.02).to(torch.bfloat16)
    wq = quantize_dequantize(w, bits, group)
    assert wq.dtype == torch.bfloat16 and wq.shape == w.shape
    x = w.float().reshape(64, -1, group)
    step = (x.amax(-1) - x.amin(-1)) / ((1 << bits) - 1)
    err = (wq.float() - w.float()).reshape(64, -1, group).abs().amax(-1)
    # within half a quantization step, plus the bf16 roundings of scale, bias and result
    # (each relative 2^-9, the scale's multiplied by up to 2^bits - 1)
    assert bool((err <= 0.5 * step + 2 ** -7 * x.abs().amax(-1)).all())
    # each group holds at most 2^bits distinct values
    for r in range(4):
        assert wq[r, :group].unique().numel() <= (1 << bits)


def test_quantize_draft_rejects_bad_settings():
    from dflash_b200.api import load_draft_model, maybe_quantize_draft_model
    d, _ = load_draft_model("random:tiny")
    assert maybe_quantize_draft_model(d, None, 64) is None
    with pytest.raises(ValueError):
        maybe_quantize_draft_model(d, 7, 64)
    with pytest.raises(ValueError):
        maybe_quantize_draft_model(d, 4, 48)
    rec = maybe_quantize_draft_model(d, 4, 64)
    assert rec == {"group_size": 64, "bits": 4}
    assert d.weights["layers"][0]["q_proj"][0, :64].unique().numel() <= 16
