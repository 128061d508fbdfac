"""CPU checks of the drop-in module contract (no GPU needed).

Mirrors the reference's own boundary tests: weight naming and strict state-dict copies
(tests/test_models.py:69-101 of the reference), packed-QKV order, and mask handling.
"""

import copy

import pytest
import torch

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200 import TransformerConfig, UserOptimizedTransformer, copy_model_weights
from tiktoktechjam2026track3_b200.cases import BASELINE_CONFIGS, config_from


class _RefLikeConfig:  # any object with the reference TransformerConfig's fields
    batch_size, seq_len, d_model, num_heads, ffn_dim, num_layers, causal = 1, 8, 16, 4, 32, 1, True


def test_seeded_construction_matches_reference_weights():
    cfg = TransformerConfig(1, 8, 64, 4, 96, 2, True)
    torch.manual_seed(7)
    model = UserOptimizedTransformer(cfg)
    expected = oracle.build_reference_state(cfg, 7)
    state = model.state_dict()
    assert list(state.keys()) == list(expected.keys())
    for k in expected:
        assert torch.equal(state[k], expected[k]), k


def test_strict_copy_from_reference_layout():
    cfg = TransformerConfig(1, 8, 16, 4, 32, 2, True)
    src = UserOptimizedTransformer(cfg)
    dst = UserOptimizedTransformer(cfg)
    with torch.no_grad():
        for p in src.parameters():
            p.uniform_(-1, 1)
    copy_model_weights(src, dst, strict=True)
    for (k, a), (_, b) in zip(src.state_dict().items(), dst.state_dict().items()):
        assert torch.equal(a, b), k
    dst.load_state_dict(oracle.build_reference_state(cfg, 0), strict=True)


def test_packed_qkv_order_and_refresh():
    cfg = TransformerConfig(1, 8, 16, 4, 32, 1, True)
    model = UserOptimizedTransformer(cfg)
    att = model.layers[0].attention
    packed = model.packed_weights()[0]
    d = cfg.d_model
    assert torch.equal(packed.w_qkv[:d], att.q_proj.weight)
    assert torch.equal(packed.w_qkv[d:2 * d], att.k_proj.weight)
    assert torch.equal(packed.w_qkv[2 * d:], att.v_proj.weight)
    assert torch.equal(packed.b_qkv[d:2 * d], att.k_proj.bias)
    with torch.no_grad():
        att.k_proj.weight.add_(1.0)
    packed2 = model.packed_weights()[0]
    assert torch.equal(packed2.w_qkv[d:2 * d], att.k_proj.weight)


def test_state_dict_round_trip():
    cfg = TransformerConfig(1, 8, 16, 4, 32, 1, True)
    model = UserOptimizedTransformer(cfg)
    saved = copy.deepcopy(model.state_dict())
    other = UserOptimizedTransformer(cfg)
    other.load_state_dict(saved, strict=True)
    for k, v in other.state_dict().items():
        assert torch.equal(v, saved[k])


def test_accepts_reference_style_config():
    model = UserOptimizedTransformer(_RefLikeConfig())
    assert model.config == config_from(_RefLikeConfig())


def test_config_validation_messages():
    with pytest.raises(ValueError, match="divisible"):
        TransformerConfig(1, 8, 10, 4, 32, 1, True).validate()
    with pytest.raises(ValueError, match="num_layers"):
        UserOptimizedTransformer(TransformerConfig(1, 8, 16, 4, 32, 0, True))


def test_no_cpu_fallback():
    model = UserOptimizedTransformer(TransformerConfig(1, 8, 256, 4, 32, 1, True))
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.randn(1, 8, 256))


def test_mask_to_lengths_prefix_and_elision():
    model = UserOptimizedTransformer(TransformerConfig(3, 6, 16, 4, 32, 1, False))
    assert model.mask_to_lengths(None, 3, 6) == (None, None)
    assert model.mask_to_lengths(torch.ones(3, 6, dtype=torch.bool), 3, 6) == (None, None)
    lengths = torch.tensor([6, 2, 4])
    mask = torch.arange(6)[None, :] < lengths[:, None]
    kv_len, row_mask = model.mask_to_lengths(mask, 3, 6)
    assert kv_len.dtype == torch.int32 and kv_len.tolist() == [6, 2, 4]
    assert row_mask.dtype == torch.uint8 and row_mask.tolist() == mask.reshape(-1).int().tolist()
    # cached result is reused while the mask is unchanged, refreshed after an in-place edit
    assert model.mask_to_lengths(mask, 3, 6)[0] is kv_len
    mask[1, 2] = True
    assert model.mask_to_lengths(mask, 3, 6)[0].tolist() == [6, 3, 4]


def test_non_prefix_mask_rejected():
    model = UserOptimizedTransformer(TransformerConfig(1, 4, 16, 4, 32, 1, False))
    with pytest.raises(NotImplementedError, match="prefix"):
        model.mask_to_lengths(torch.tensor([[True, False, True, True]]), 1, 4)
    with pytest.raises(ValueError, match="bool"):
        model.mask_to_lengths(torch.ones(1, 4, dtype=torch.int32), 1, 4)


def test_baseline_configs_are_valid():
    for w in BASELINE_CONFIGS.values():
        w.config.validate()
        assert w.config.head_dim in (64, 128)
    assert BASELINE_CONFIGS["c5"].config == TransformerConfig(32, 100000, 1024, 16, 1024, 2, True)


def test_package_generator_matches_oracle_generator():
    from tiktoktechjam2026track3_b200.cases import generate_random_case

    cfg = TransformerConfig(3, 40, 16, 4, 32, 1, False)
    for pad in (0.0, 0.5):
        a = generate_random_case(cfg, torch.device("cpu"), torch.float32, 9, pad)
        b = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 9, pad)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_layernorm_fusion_policy_depends_on_widths_only():
    """norm2 / norm1 run inside the residual GEMMs only where the library recommends it for d_model
    (nowhere in this build: measured slower), forced on where a plan exists, and the choice is the
    same for every token count (so batch shards reproduce the full batch)."""
    c2 = UserOptimizedTransformer(BASELINE_CONFIGS["c2"].config)  # d_model 768: 4 CTAs x 192
    assert not any(c2.layernorm_fused(t) for t in (1, 4096, 10**6))
    c2.fuse_layernorm = True
    assert all(c2.layernorm_fused(t) for t in (1, 4096, 10**6))
    c2.fuse_layernorm = False
    assert not c2.layernorm_fused(4096)
    c3 = UserOptimizedTransformer(BASELINE_CONFIGS["c3"].config)  # d_model 1024: 256-wide tiles
    c3.fuse_layernorm = True
    assert c3.layernorm_fused(4096)
    odd = UserOptimizedTransformer(TransformerConfig(1, 8, 2560, 20, 256, 1, True))  # no plan for 2560
    odd.fuse_layernorm = True
    assert not odd.layernorm_fused(8)
    assert UserOptimizedTransformer.launches_per_forward(12, True) == 62
    assert UserOptimizedTransformer.launches_per_forward(12) == 85


def test_mask_cache_keeps_its_mask_alive():
    """The cache entry holds the mask tensor, so a freed mask's storage cannot come back as a
    different mask of the same shape that the entry would still match (same address, same version)."""
    model = UserOptimizedTransformer(TransformerConfig(2, 8, 16, 4, 32, 1, False))
    mask = torch.arange(8)[None, :] < torch.tensor([[3], [8]])
    ptr = mask.data_ptr()
    assert model.mask_to_lengths(mask, 2, 8)[0].tolist() == [3, 8]
    del mask
    cached = model._mask_lengths._cache
    assert cached is not None and cached[1].data_ptr() == ptr  # still owned by the cache
    other = torch.arange(8)[None, :] < torch.tensor([[5], [2]])
    assert other.data_ptr() != ptr
    assert model.mask_to_lengths(other, 2, 8)[0].tolist() == [5, 2]


def test_inference_tensor_weights_are_refreshed_every_call():
    """Parameters created under inference mode carry no version counter: the packed q/k/v copies
    are refreshed in place on every call instead of trusting a cached version."""
    cfg = TransformerConfig(1, 8, 16, 4, 32, 1, True)
    with torch.inference_mode():
        model = UserOptimizedTransformer(cfg)
    att = model.layers[0].attention
    assert att.k_proj.weight.is_inference()
    assert model._weights_key() is None
    packed = model.packed_weights()[0]
    with torch.inference_mode():
        att.k_proj.weight.add_(1.0)
        att.q_proj.bias.mul_(2.0)
    again = model.packed_weights()[0]
    assert again is packed  # same storage: captured graphs stay valid
    d = cfg.d_model
    assert torch.equal(again.w_qkv[d:2 * d], att.k_proj.weight)
    assert torch.equal(again.b_qkv[:d], att.q_proj.bias)


def test_repacking_drops_graphs_of_every_shape():
    model = UserOptimizedTransformer(TransformerConfig(1, 8, 16, 4, 32, 1, True))
    model.packed_weights()
    model._graphs[("a",)] = object()
    model._graphs[("b",)] = object()
    with torch.no_grad():
        model.layers[0].ffn_in.bias.add_(1.0)
    model.packed_weights()
    assert model._graphs == {}
