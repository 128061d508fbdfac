"""Schema-v2 result documents (report.py) and the official case matrix, on CPU."""

import json
from dataclasses import astuple

from tiktoktechjam2026track3_b200 import report
from tiktoktechjam2026track3_b200.cases import OFFICIAL_TEST_CASES, TransformerConfig
from tiktoktechjam2026track3_b200.correctness import baseline_gate, compare_outputs
from tiktoktechjam2026track3_b200.models import SUPPORTED_HEAD_DIMS

import torch


def test_official_cases_are_the_reference_matrix_and_supported():
    assert len(OFFICIAL_TEST_CASES) == 14
    # cases.py:42-57 of the reference: (B, S, D, H, F, L, causal)
    assert astuple(OFFICIAL_TEST_CASES[5]) == (10000, 128, 128, 4, 128, 4, True)
    assert astuple(OFFICIAL_TEST_CASES[13]) == (32, 100000, 1024, 16, 1024, 2, True)
    for cfg in OFFICIAL_TEST_CASES:
        cfg.validate()
        assert cfg.head_dim in SUPPORTED_HEAD_DIMS


def test_timing_block_matches_reference_fields():
    t = report.timing_block([3.0, 1.0, 2.0, 4.0], tokens_per_call=1000)
    assert set(t) == {"samples_ms", "median_ms", "mean_ms", "p90_ms", "min_ms", "tokens_per_second"}
    assert t["median_ms"] == 2.5 and t["min_ms"] == 1.0 and t["p90_ms"] == 4.0
    assert t["tokens_per_second"] == 1000 * 1000.0 / 2.5


def test_matrix_document_status_logic(tmp_path):
    cfg = TransformerConfig(2, 16, 64, 1, 64, 1, True)
    y = torch.ones(2, 16, 64)
    acc = compare_outputs(y, y, rtol=0.02, atol=0.002)
    perf = report.performance_block([2.0, 2.0], [1.0, 1.0], cfg, 1, 2, 1)
    assert perf["speedup"] == 2.0
    ok = report.official_case_result(1, cfg, acc, perf, gate=baseline_gate(y, y))
    bad_acc = compare_outputs(y, y * 2, rtol=0.02, atol=0.002)
    bad = report.official_case_result(2, cfg, bad_acc, None)
    failed = report.execution_failed_result(3, cfg, "out_of_memory", RuntimeError("CUDA out of memory"))
    env = {"device": "cpu"}
    doc = report.matrix_document([1], [ok], env, {})
    assert doc["schema_version"] == 2 and doc["mode"] == "official_matrix"
    assert doc["complete"] and doc["all_cases_executed"] and doc["correctness_passed"] is True
    doc = report.matrix_document([1, 2], [ok, bad], env, {})
    assert doc["correctness_passed"] is False and doc["failure_category"] == "correctness"
    doc = report.matrix_document([1, 2, 3], [ok, bad, failed], env, {})
    assert doc["correctness_passed"] is None and doc["failure_category"] == "execution"
    doc = report.matrix_document([1, 2, 3], [ok], env, {})
    assert not doc["complete"] and doc["failure_category"] is None
    path = tmp_path / "m.json"
    report.write_json_document(path, doc)
    back = json.loads(path.read_text())
    assert back["cases"][0]["gate"]["passed"] is True
