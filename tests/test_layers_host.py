"""Host logic of the Reflex layer mirrors (no GPU): argument checks and the
attention-mask to (source validity, suffix blocks) conversion."""
import pytest
import torch

from reflex_b200.layers import StreamingAttention


def test_constructor_and_slot_checks():
    with pytest.raises(ValueError, match="quantize_kv_cache"):
        StreamingAttention(1 / 16)
    with pytest.raises(ValueError, match="kv_scheme"):
        StreamingAttention(1 / 16, quantize_kv_cache=True, kv_scheme="fp8")
    a = StreamingAttention(1 / 16, quantize_kv_cache=True)
    with pytest.raises(ValueError, match="cache_slot"):
        a.prefill_source(torch.zeros(1, 1, 4, 256), torch.zeros(1, 1, 4, 256), cache_slot="other")
    assert a.merged_k_cache is None and a.source_length == 0


def _block_mask(blocks, n_src, B=2):
    b = torch.tensor(blocks)
    suf = b[None, :] <= b[:, None]
    m = torch.cat([torch.ones(len(blocks), n_src, dtype=torch.bool), suf], dim=1)
    return m[None, None].expand(B, 1, -1, -1).clone()


@pytest.mark.parametrize("blocks", [[0] * 5, [0, 1, 1, 1, 1], [0, 0, 1, 2, 2]])
def test_mask_to_structure_block_causal(blocks):
    n_src = 7
    valid, block = StreamingAttention._mask_to_structure(_block_mask(blocks, n_src), 2, len(blocks), n_src, 0)
    assert block.tolist() == blocks
    assert valid.shape == (2, n_src) and bool(valid.all())


def test_mask_to_structure_additive_and_source_holes():
    blocks, n_src = [0, 1, 1], 4
    m = _block_mask(blocks, n_src)
    m[:, :, :, 1] = False  # a padded source token
    add = torch.where(m, 0.0, torch.finfo(torch.float32).min)
    valid, block = StreamingAttention._mask_to_structure(add, 2, 3, n_src, 3)
    assert block.tolist() == blocks
    assert valid.shape == (2, 3 + n_src)
    assert valid[0].tolist() == [0, 0, 0, 1, 0, 1, 1]


def test_mask_to_structure_rejects_general_masks():
    m = _block_mask([0, 0, 0], 2)
    m[:, :, 0, 2] = False  # row 0 loses a suffix key of its own block
    with pytest.raises(ValueError, match="block-causal"):
        StreamingAttention._mask_to_structure(m, 2, 3, 2, 0)
    m = _block_mask([0, 0, 0], 2)
    m[:, :, 1, 0] = False  # source visibility differs between rows
    with pytest.raises(ValueError, match="same source"):
        StreamingAttention._mask_to_structure(m, 2, 3, 2, 0)
