"""Host logic of the Reflex layer mirrors (no GPU): argument checks and the
attention-mask to (source validity, suffix blocks) conversion."""
import pytest
import torch

from reflex_b200.layers import StreamingAttention


def test_constructor_and_slot_checks():
    # the reference's default (no quantization requested) keeps the source as int8
    assert StreamingAttention(1 / 16).kv_scheme == "i8_sym"
    assert StreamingAttention(1 / 16, quantize_kv_cache=True).kv_scheme == "u8_ref"
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


def test_fused_linears_are_modules_with_reference_parameters():
    """QKVLinear / MergedColumnLinear carry the reference's parameters
    (reflex/layers/linear.py:29-148), so the fusion init of
    modeling_pi05.py:843-866 / 883-917 (construct, .to(device, dtype), copy
    the projection weights into slices under no_grad) runs on them."""
    from torch import nn

    from reflex_b200.layers import MergedColumnLinear, QKVLinear

    qkv = QKVLinear(64, 16, 4, 1, bias=True)
    assert isinstance(qkv, nn.Module)
    assert dict(qkv.named_parameters()).keys() == {"weight", "bias"}
    assert qkv.weight.shape == ((4 + 2) * 16, 64) and qkv.bias.shape == (96,)
    qkv.to(device="cpu", dtype=torch.bfloat16)
    assert qkv.weight.dtype == torch.bfloat16
    q_w, k_w, v_w = torch.randn(64, 64), torch.randn(16, 64), torch.randn(16, 64)
    with torch.no_grad():
        qkv.weight[:64].copy_(q_w)
        qkv.weight[64:80].copy_(k_w)
        qkv.weight[80:].copy_(v_w)
    assert torch.equal(qkv.weight[64:80].float(), k_w.bfloat16().float())
    assert set(qkv.state_dict()) == {"weight", "bias"}
    mc = MergedColumnLinear(64, [128, 128])
    assert mc.bias is None and mc.weight.shape == (256, 64)
    assert list(dict(mc.named_parameters())) == ["weight"]
    with pytest.raises(ValueError, match="3D"):
        qkv(torch.zeros(2, 64))
    with pytest.raises(ValueError, match="CUDA"):
        qkv(torch.zeros(1, 2, 64, dtype=torch.bfloat16))


def test_eviction_moves_the_ring_head():
    a = StreamingAttention(1 / 16, max_cache_size=8)
    a.source_length, a.ring = 6, type("R", (), {"capacity": 8})()
    a.evict_source_prefix(5)
    assert a.source_length == 1 and a._head == 5
    assert a.source_slots(0, 1).tolist() == [5]
    a.source_length = 5  # as after appending four more tokens: they wrap
    assert a.source_slots(0, 5).tolist() == [5, 6, 7, 0, 1]


def test_policy_entry_points_keep_reference_signatures():
    """Parameter names and order of the reference's entry points:
    PI05Model.denoise_step / sample_actions (reflex/policies/pi05/
    modeling_pi05.py:1181,1244), PI05Policy.predict_action_chunk /
    select_action (:1649,1681), PI0Model.sample_actions (reflex/policies/pi0/
    modeling_pi0.py:785) and PI0Policy.predict_action_chunk (:1010)."""
    import inspect

    from reflex_b200.policy import PI0Model, PI0Policy, PI05Model, PI05Policy

    def names(f):
        return list(inspect.signature(f).parameters)

    assert names(PI05Model.denoise_step) == ["self", "prefix_pad_masks", "prefix_att_masks", "state", "x_t",
                                             "timestep"]
    assert names(PI05Model.sample_actions) == ["self", "images", "img_masks", "tokens", "masks", "state", "noise",
                                               "num_steps", "incremental_input"]
    assert names(PI05Policy.predict_action_chunk) == ["self", "batch", "noise", "num_steps", "incremental_input"]
    assert names(PI05Policy.select_action) == ["self", "batch", "noise"]
    assert names(PI0Model.sample_actions) == ["self", "images", "img_masks", "tokens", "masks", "state", "noise",
                                              "num_steps"]
    assert names(PI0Policy.predict_action_chunk) == ["self", "batch", "noise"]
    assert names(PI05Policy.reset) == ["self"]
