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


# ----------------------------------------------------------------------------- schema-2 checks
def _validate_schema2(doc):
    """The checks benchmarkctl applies to a schema-2 result (orchestrator/crates/benchmarkctl/src/
    main.rs:1155-1240 of the reference), restated: mode, environment / settings objects, a
    non-empty integer requested_case_ids, `complete` agreeing with the number of cases,
    all_cases_executed implying complete, a passing result being complete and fully executed, and
    failure_category a string or null."""
    assert isinstance(doc.get("schema_version"), int) and doc["schema_version"] == 2
    assert doc.get("mode") == "official_matrix"
    assert isinstance(doc.get("environment"), dict) and isinstance(doc.get("settings"), dict)
    req = doc.get("requested_case_ids")
    assert isinstance(req, list) and req and all(isinstance(c, int) and c >= 0 for c in req)
    cases = doc.get("cases")
    assert isinstance(cases, list)
    assert isinstance(doc.get("complete"), bool) and isinstance(doc.get("all_cases_executed"), bool)
    assert doc["complete"] == (len(cases) == len(req))
    assert not (doc["all_cases_executed"] and not doc["complete"])
    assert "correctness_passed" in doc and doc["correctness_passed"] in (True, False, None)
    if doc["correctness_passed"] is True:
        assert doc["complete"] and doc["all_cases_executed"]
    assert "failure_category" in doc and (doc["failure_category"] is None or isinstance(doc["failure_category"], str))


def _reference_runner():
    import importlib
    import os
    import sys
    from pathlib import Path

    roots = [Path(p) for p in (os.environ.get("REFERENCE_ROOT"),) if p]
    roots.append(Path(__file__).resolve().parents[1] / "baseline" / "_ref")
    for root in roots:
        if (root / "transformer_benchmark" / "runner.py").is_file():
            if str(root) not in sys.path:
                sys.path.insert(0, str(root))
            return importlib.import_module("transformer_benchmark.runner")
    return None


def _scaled_case(case_id=1):
    cfg = TransformerConfig(2, 16, 64, 1, 64, 1, True)
    y = torch.ones(2, 16, 64)
    acc = compare_outputs(y, y, rtol=0.02, atol=0.002)
    perf = report.performance_block([2.0, 2.0], [1.0, 1.0], cfg, 1, 2, 1)
    gpus = [report.gpu_scaling_entry(n, ms, 32) for n, ms in ((2, 0.6), (1, 1.0), (8, 0.2))]
    roof = report.roofline_entry("gemm_tc_kernel", "tensor", 580.0, 1685.1, "TFLOP/s")
    cpu = report.cpu_baseline_entry(16, 85.0, 32, "port", "1 sequence through the fp32 CPU restatement")
    return cfg, acc, perf, report.official_case_result(case_id, cfg, acc, perf, gate=baseline_gate(y, y), gpus=gpus,
                                                       roofline=roof, cpu_baseline=cpu)


def test_gpu_roofline_and_cpu_fields():
    _, _, _, case = _scaled_case()
    assert [e["gpus"] for e in case["gpus"]] == [1, 2, 8]
    assert case["gpus"][0]["tokens_per_s"] == 32 * 1000.0 / 1.0 and case["gpus"][0]["ms_per_iter"] == 1.0
    assert abs(case["roofline"]["frac"] - 580.0 / 1685.1) < 1e-12 and case["roofline"]["bound"] == "tensor"
    assert case["cpu_baseline"]["cores"] == 16 and case["cpu_baseline"]["ms"] == 85.0
    doc = report.matrix_document([1], [case], {"device": "cuda"}, {})
    assert doc["gpus"] == 8
    _validate_schema2(doc)


def test_documents_pass_the_schema2_checks():
    _, _, _, ok = _scaled_case(1)
    cfg = TransformerConfig(2, 16, 64, 1, 64, 1, True)
    failed = report.execution_failed_result(2, cfg, "out_of_memory", RuntimeError("CUDA out of memory"))
    for ids, results in (([1], [ok]), ([1, 2], [ok, failed]), ([1, 2], [ok])):
        _validate_schema2(json.loads(json.dumps(report.matrix_document(ids, results, {"device": "cuda"}, {}))))


def test_case_and_document_keys_extend_the_reference_writer(tmp_path):
    """Everything the reference's own writer emits (runner.py:423-499) is in this build's documents
    with the same value for the same inputs; this build only adds keys."""
    import argparse

    runner = _reference_runner()
    if runner is None:
        import pytest

        pytest.skip("the reference package is not installed (baseline/install_reference.py)")
    cfg, acc, perf, ours = _scaled_case(1)
    ref_cfg = runner.TransformerConfig(**{k: getattr(cfg, k) for k in ("batch_size", "seq_len", "d_model", "num_heads",
                                                                         "ffn_dim", "num_layers", "causal")})
    ref_acc = runner.AccuracySummary(passed=True, rtol=0.02, atol=0.002, max_abs_error=0.0, max_relative_error=0.0,
                                     failed_elements=0, total_elements=2048, trials=[])
    ref_case = runner.official_case_result(1, ref_cfg, ref_acc, perf)
    ours = report.official_case_result(1, cfg, ref_acc, perf)
    for key, value in ref_case.items():
        assert key in ours, key
        assert json.dumps(ours[key], sort_keys=True) == json.dumps(value, sort_keys=True), key
    failed_ref = runner.execution_failed_result(2, ref_cfg, "out_of_memory", RuntimeError("CUDA out of memory"))
    failed_ours = report.execution_failed_result(2, cfg, "out_of_memory", RuntimeError("CUDA out of memory"))
    assert failed_ours == failed_ref
    args = argparse.Namespace(seed=0, padding_ratio=0.0, input_scale=1.0, accuracy_trials=1, rtol=0.02, atol=0.002,
                              warmup=1, repeats=2, benchmark_rounds=1, benchmark_on_failure=False,
                              matmul_precision="highest", allow_tf32=False, compile_baseline=False,
                              compile_user=False, profile_candidate=False)
    path = tmp_path / "ref.json"
    runner.write_matrix_result(path, args, torch.device("cpu"), torch.float32, [1, 2], [ref_case, failed_ref])
    ref_doc = json.loads(path.read_text())
    our_doc = report.matrix_document([1, 2], [ours, failed_ours], ref_doc["environment"], ref_doc["settings"])
    for key, value in ref_doc.items():
        assert key in our_doc, key
        if key == "cases":  # per case, the reference's keys with the same values (ours adds keys)
            for ref_c, our_c in zip(value, json.loads(json.dumps(our_doc["cases"]))):
                assert {k: our_c.get(k) for k in ref_c} == ref_c
            continue
        assert json.dumps(our_doc[key], sort_keys=True) == json.dumps(value, sort_keys=True), key
    _validate_schema2(ref_doc)
    _validate_schema2(our_doc)
