"""The reference's official case matrix (transformer_benchmark/cases.py:42-57) through the module,
with the result document in the reference runner's schema version 2 (runner.py:463-499).

Per case, as the reference runner does (runner.py:304-402): weights under seed 1234, inputs from
the reference generator (seed 1234 for accuracy, 1234 + 100000 for timing), padding ratio 0.
  * gate (this build's acceptance rule): max|y - r| <= 2^-7 max|r|, no NaN/Inf, r = the fp32
    oracle on the same bf16 weights and inputs; it decides `correctness_passed`;
  * accuracy (the reference's strict elementwise rule, rtol 0.02 / atol 0.002): against the
    oracle evaluated in bf16, which stands in for the reference's baseline module on the GPU;
  * performance: CUDA-event medians of this module and of that bf16 baseline.
Case 14 (32 x 100000 tokens) runs here on 2 sequences of 8192 tokens; its full length is checked in
test_gpu_model.py::test_model_full_length_against_oracle and measured by `bench.py --workload c5`.
The document is written to $B2_MATRIX_JSON when set, else under pytest's tmp_path.
"""

import os
import statistics
from dataclasses import asdict, replace
from pathlib import Path

import pytest
import torch

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200 import UserOptimizedTransformer, baseline_gate, report
from tiktoktechjam2026track3_b200.cases import OFFICIAL_TEST_CASES
from tiktoktechjam2026track3_b200.correctness import compare_outputs

pytestmark = pytest.mark.gpu

SEED = 1234
REDUCED = {14: dict(batch_size=2, seq_len=8192)}
WARMUP, REPEATS, BASELINE_REPEATS = 3, 10, 3
_RESULTS = {}


def _time(fn, warmup, repeats):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    samples = []
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        samples.append(start.elapsed_time(end))
    return samples


@pytest.mark.parametrize("case_id", range(1, len(OFFICIAL_TEST_CASES) + 1))
def test_official_case(cuda_device, case_id):
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = OFFICIAL_TEST_CASES[case_id - 1]
    if case_id in REDUCED:
        cfg = replace(cfg, **REDUCED[case_id])
    state = oracle.round_state_to_bf16(oracle.build_reference_state(cfg, SEED))
    model = UserOptimizedTransformer(cfg)
    model.load_state_dict(state, strict=True)
    model = model.to(device="cuda", dtype=torch.bfloat16).eval()
    dev = torch.device("cuda")
    x, mask = oracle.generate_random_case(cfg, dev, torch.float32, SEED, 0.0)
    xb = x.bfloat16()
    st32 = {k: v.to(dev, torch.float32) for k, v in state.items()}
    st16 = {k: v.to(dev, torch.bfloat16) for k, v in state.items()}
    with torch.inference_mode():
        y = model(xb, mask)
        ref32 = oracle.forward(st32, cfg, xb.float(), mask, query_chunk=512)
        ref16 = oracle.forward(st16, cfg, xb, mask, query_chunk=512, dtype=torch.bfloat16)
        gate = baseline_gate(y, ref32)
        accuracy = compare_outputs(ref16, y, rtol=0.02, atol=0.002)
        xt, mt = oracle.generate_random_case(cfg, dev, torch.bfloat16, SEED + 100000, 0.0)
        ours = _time(lambda: model(xt, mt), WARMUP, REPEATS)
        base = _time(lambda: oracle.forward(st16, cfg, xt, mt, query_chunk=512, dtype=torch.bfloat16), 1,
                     BASELINE_REPEATS)
    perf = report.performance_block(base, ours, cfg, WARMUP, REPEATS, 1)
    acc = asdict(accuracy)
    acc.update(rtol=0.02, atol=0.002, rule="strict_less_than_or", against="oracle in bf16 (reference baseline)")
    gpus = [report.gpu_scaling_entry(1, perf["optimized"]["median_ms"], cfg.batch_size * cfg.seq_len)]
    result = report.official_case_result(case_id, cfg, acc, perf, gate=gate, gpus=gpus)
    result["correctness_passed"] = gate.passed  # acceptance: the 2^-7 gate against fp32
    result["status"] = "succeeded" if gate.passed else "correctness_failed"
    result["failure_category"] = None if gate.passed else "correctness"
    if case_id in REDUCED:
        result["reduced"] = REDUCED[case_id]
    _RESULTS[case_id] = result
    assert gate.passed, (case_id, gate)
    assert torch.isfinite(y).all()


def test_official_matrix_document(cuda_device, tmp_path):
    if len(_RESULTS) != len(OFFICIAL_TEST_CASES):
        pytest.skip("needs every official case to have run in this session")
    ids = sorted(_RESULTS)
    settings = {"seed": SEED, "padding_ratio": 0.0, "input_scale": 1.0, "accuracy_trials": 1, "rtol": 0.02,
                "atol": 0.002, "accuracy_rule": "strict_less_than_or", "gate": "max|y-r| <= 2^-7 max|r|",
                "warmup": WARMUP, "repeats": REPEATS, "benchmark_rounds": 1, "allow_tf32": False}
    doc = report.matrix_document(ids, [_RESULTS[i] for i in ids], report.environment_metadata(
        torch.device("cuda"), torch.bfloat16), settings)
    path = Path(os.environ.get("B2_MATRIX_JSON", tmp_path / "official_matrix.json"))
    report.write_json_document(path, doc)
    assert doc["schema_version"] == 2 and doc["complete"] and doc["all_cases_executed"]
    assert doc["correctness_passed"] is True
    speedups = [r["performance"]["speedup"] for r in doc["cases"]]
    assert all(s is not None and s > 0 for s in speedups)
    print("official matrix:", {r["case_id"]: round(r["performance"]["optimized"]["median_ms"], 3) for r in doc["cases"]},
          "median speedup vs bf16 baseline", statistics.median(speedups))
