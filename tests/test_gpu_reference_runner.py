"""The reference's own benchmark CLI drives UserOptimizedTransformer as its candidate.

transformer_benchmark.runner (the reference, installed under baseline/_ref by
baseline/install_reference.py, or found through $REFERENCE_ROOT) builds the candidate from its
module-global slot (runner.py:20-24, 321), copies the baseline's weights into it, runs its accuracy
trials and its timing loop, and returns 0 when the accuracy phase passed (runner.py:551-559).
These tests rebind the slot exactly as tiktoktechjam2026track3_b200.reference_runner does (and
as INTEGRATION.md shows) and assert the runner's exit status and JSON result, on the first two
benchmark configurations:
  * with the B200 gate (2^-7 normwise against the fp32 evaluation of the reference model);
  * with the runner's own strict elementwise rule at the tolerances STRICT_RULE_TOLERANCES states.
Skipped when the reference package is not present.
"""

import json

import pytest
import torch

from tiktoktechjam2026track3_b200 import reference_runner

pytestmark = pytest.mark.gpu

SHAPES = {
    "c1": ["--batch-size", "2", "--seq-len", "128", "--d-model", "256", "--heads", "4", "--ffn-dim", "1024",
           "--layers", "2", "--causal"],
    "c2": ["--batch-size", "8", "--seq-len", "512", "--d-model", "768", "--heads", "12", "--ffn-dim", "3072",
           "--layers", "12", "--padding-ratio", "0.5"],
}
COMMON = ["--no-official-matrix", "--device", "cuda", "--dtype", "bfloat16", "--accuracy-trials", "3",
          "--warmup", "3", "--repeats", "10", "--benchmark-rounds", "1"]


@pytest.fixture(scope="module")
def runner(cuda_device):
    try:
        return reference_runner.import_runner()
    except ImportError as exc:
        pytest.skip(str(exc))


def _run(tmp_path, name, extra, gate):
    out = tmp_path / f"{name}.json"
    argv = (["--b200-gate"] if gate else []) + ["--"] + COMMON + SHAPES[name] + extra + ["--json-output", str(out)]
    status = reference_runner.main(argv)
    doc = json.loads(out.read_text())
    return status, doc


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_reference_runner_with_b200_gate(runner, tmp_path, name):
    status, doc = _run(tmp_path, name, [], gate=True)
    assert status == 0, doc["accuracy"]
    assert doc["correctness_passed"] is True
    perf = doc["performance"]
    assert perf["optimized"]["median_ms"] > 0 and perf["speedup"] > 1.0
    assert runner.UserOptimizedTransformer.__module__ == "tiktoktechjam2026track3_b200.models"


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_reference_runner_strict_rule_at_stated_tolerances(runner, tmp_path, name):
    atol, rtol = reference_runner.STRICT_RULE_TOLERANCES[name]
    status, doc = _run(tmp_path, name, ["--atol", str(atol), "--rtol", str(rtol)], gate=False)
    acc = doc["accuracy"]
    assert status == 0, {k: acc[k] for k in ("max_abs_error", "max_relative_error", "failed_elements")}
    assert doc["settings"]["atol"] == atol and doc["settings"]["rtol"] == rtol
    assert torch.cuda.is_available()
