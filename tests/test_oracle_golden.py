"""Pins the fp32 oracle (oracle/reference_fp32.py) to the reference itself.

The golden vectors were produced by tests/golden/make_golden.py, which imports and runs the
reference's own generate_random_case (transformer_benchmark/cases.py:60-98) and
BaselineTransformer (transformer_benchmark/models.py:895-919) on CPU in fp32.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200.cases import TransformerConfig

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())


def _case(name):
    m = MANIFEST[name]
    cfg = TransformerConfig(m["batch_size"], m["seq_len"], m["d_model"], m["num_heads"], m["ffn_dim"],
                            m["num_layers"], m["causal"])
    return cfg, m, np.load(GOLDEN / f"{name}.npz")


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_weight_construction_matches_reference(name):
    cfg, m, g = _case(name)
    state = oracle.build_reference_state(cfg, m["seed"])
    keys = [str(k) for k in g["param_keys"]]
    assert sorted(state.keys()) == keys
    sums = oracle.state_checksums(state)
    for key, (s, q) in zip(keys, g["param_sums"]):
        assert sums[key][0] == pytest.approx(s, rel=0, abs=1e-9 * max(1.0, abs(q)))
        assert sums[key][1] == pytest.approx(q, rel=1e-12)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_input_generator_matches_reference(name):
    cfg, m, g = _case(name)
    x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, m["seed"], m["padding_ratio"])
    assert torch.equal(mask, torch.from_numpy(g["mask"]))
    assert np.array_equal(x.reshape(-1)[:256].numpy(), g["x_head"])
    xd = x.double()
    assert float(xd.sum()) == pytest.approx(float(g["x_sums"][0]), rel=0, abs=1e-6)
    assert float((xd * xd).sum()) == pytest.approx(float(g["x_sums"][1]), rel=1e-12)


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_forward_matches_reference_fp32(name):
    cfg, m, g = _case(name)
    state = oracle.build_reference_state(cfg, m["seed"])
    x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, m["seed"], m["padding_ratio"])
    with torch.inference_mode():
        out = oracle.forward(state, cfg, x, mask, query_chunk=64)
    ref = torch.from_numpy(g["out_fp32"])
    assert torch.allclose(out, ref, rtol=0, atol=2e-5), float((out - ref).abs().max())


@pytest.mark.parametrize("name", sorted(MANIFEST))
def test_oracle_forward_matches_reference_on_bf16_values(name):
    """The parity target of the GPU path: fp32 math on bf16-rounded weights and inputs."""
    cfg, m, g = _case(name)
    state = oracle.round_state_to_bf16(oracle.build_reference_state(cfg, m["seed"]))
    x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, m["seed"], m["padding_ratio"])
    x = x.to(torch.bfloat16).float()
    with torch.inference_mode():
        out = oracle.forward(state, cfg, x, mask)
    ref = torch.from_numpy(g["out_bf16_inputs"])
    assert torch.allclose(out, ref, rtol=0, atol=2e-5), float((out - ref).abs().max())


def test_chunked_attention_equals_unchunked():
    torch.manual_seed(3)
    q, k, v = (torch.randn(2, 3, 70, 16) for _ in range(3))
    mask = torch.arange(70)[None, :] < torch.tensor([[70], [41]])
    for causal in (False, True):
        a = oracle.attention_core(q, k, v, mask, causal, 0.25, query_chunk=70)
        b = oracle.attention_core(q, k, v, mask, causal, 0.25, query_chunk=16)
        assert torch.allclose(a, b, atol=1e-6)


def test_flop_model():
    cfg = TransformerConfig(2, 128, 256, 4, 1024, 2, True)
    f = oracle.flops_per_forward(cfg)
    assert f["gemm"] == 2 * (8 * 256 * 256 * 256 + 4 * 256 * 256 * 1024)
    assert f["attention"] == 2 * 4 * 256 * 2 * (128 * 129 / 2)
