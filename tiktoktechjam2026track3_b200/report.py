"""Result documents in the reference runner's JSON schema (version 2, official-matrix mode).

Mirrors transformer_benchmark/runner.py: `official_case_result` (:423-441),
`execution_failed_result` (:445-460), the matrix document of `write_matrix_result` (:463-499),
`environment_metadata` (:210-220) and the timing block of `benchmark_models`
(transformer_benchmark/timing.py:101-195), so that tools reading the reference's result files
(e.g. its `benchmarkctl` validators) read this build's files too. Added keys are additive only:
`"gate"` (the acceptance tolerance, max|y - r| <= 2^-7 max|r|) next to `"accuracy"`, per-case
`"implementation"` naming what produced the numbers, and the multi-GPU / roofline / CPU-baseline
records of this build: per case `"gpus"` (one entry per GPU count: `gpus`, `tokens_per_s`,
`ms_per_iter`, `scaling`), `"roofline"` (the dominant kernel: `kernel`, `bound`, `achieved`,
`peak`, `unit`, `frac`) and `"cpu_baseline"` (`cores`, `ms`, `tokens_per_s`, `kind`, `sample`);
per document `"gpus"` (the largest GPU count of any case). The reference's readers ignore keys
they do not know (its validator, orchestrator/crates/benchmarkctl/src/main.rs:1155-1240, checks only
the keys it needs), so every document stays a valid schema-2 result.
"""

from __future__ import annotations

import json
import math
import os
import platform
import statistics
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import torch

from .cases import TransformerConfig

SCHEMA_VERSION = 2
CASE_SET = "competition_appendix_3_7"


def timing_block(samples_ms: Sequence[float], tokens_per_call: int) -> Dict[str, object]:
    """The per-model timing record of timing.py:178-193 (median-based tokens/s)."""
    samples = [float(s) for s in samples_ms]
    if not samples:
        raise ValueError("no timing samples")
    ordered = sorted(samples)
    median = statistics.median(ordered)
    p90 = ordered[min(len(ordered) - 1, max(0, math.ceil(0.9 * len(ordered)) - 1))]
    return {
        "samples_ms": samples,
        "median_ms": median,
        "mean_ms": statistics.fmean(samples),
        "p90_ms": p90,
        "min_ms": ordered[0],
        "tokens_per_second": tokens_per_call * 1000.0 / median,
    }


def performance_block(baseline_ms: Optional[Sequence[float]], optimized_ms: Sequence[float], config: TransformerConfig,
                      warmup: int, repeats: int, rounds: int) -> Dict[str, object]:
    tokens = config.batch_size * config.seq_len
    optimized = timing_block(optimized_ms, tokens)
    baseline = timing_block(baseline_ms, tokens) if baseline_ms else None
    return {
        "baseline": baseline,
        "optimized": optimized,
        "speedup": (baseline["median_ms"] / optimized["median_ms"]) if baseline else None,
        "warmup": warmup,
        "repeats": repeats,
        "rounds": rounds,
    }


def gpu_scaling_entry(gpus: int, ms_per_iter: float, tokens_per_call: int, scaling: str = "strong") -> Dict[str, object]:
    """One GPU count's throughput record: the configuration's B*S tokens per call over the
    multi-GPU step time (max over ranks)."""
    if gpus < 1 or not ms_per_iter > 0:
        raise ValueError("gpus must be >= 1 and ms_per_iter positive")
    if scaling not in ("strong", "weak"):
        raise ValueError("scaling is 'strong' (fixed global batch) or 'weak' (fixed per-GPU batch)")
    return {"gpus": int(gpus), "tokens_per_s": tokens_per_call * 1000.0 / ms_per_iter, "ms_per_iter": float(ms_per_iter),
            "scaling": scaling}


def roofline_entry(kernel: str, bound: str, achieved: float, peak: float, unit: str) -> Dict[str, object]:
    """The dominant kernel against its roofline (tensor: TFLOP/s against the bf16 peak; hbm: GB/s
    against the copy bandwidth)."""
    if bound not in ("tensor", "hbm"):
        raise ValueError("bound is 'tensor' or 'hbm'")
    return {"kernel": kernel, "bound": bound, "achieved": float(achieved), "peak": float(peak), "unit": unit,
            "frac": float(achieved) / float(peak)}


def cpu_baseline_entry(cores: int, ms: float, tokens_per_call: int, kind: str, sample: str) -> Dict[str, object]:
    """The reference computation timed on the host CPU (kind "reference" or "port")."""
    return {"cores": int(cores), "ms": float(ms), "tokens_per_s": tokens_per_call * 1000.0 / ms, "kind": kind,
            "sample": sample}


def _plain(obj):
    return asdict(obj) if is_dataclass(obj) else obj


def official_case_result(case_id: int, config: TransformerConfig, accuracy, performance: Optional[Dict[str, object]],
                         gate=None, implementation: str = "tiktoktechjam2026track3_b200",
                         gpus: Optional[List[Dict[str, object]]] = None, roofline: Optional[Dict[str, object]] = None,
                         cpu_baseline: Optional[Dict[str, object]] = None) -> Dict[str, object]:
    acc = _plain(accuracy)
    passed = bool(acc["passed"])
    result: Dict[str, object] = {
        "case_id": case_id,
        "config": asdict(config),
        "status": "succeeded" if passed else "correctness_failed",
        "failure_category": None if passed else "correctness",
        "correctness_passed": passed,
        "accuracy": acc,
        "performance": performance,
        "implementation": implementation,
    }
    if gate is not None:
        result["gate"] = _plain(gate)
    if gpus is not None:
        result["gpus"] = sorted(gpus, key=lambda e: e["gpus"])
    if roofline is not None:
        result["roofline"] = roofline
    if cpu_baseline is not None:
        result["cpu_baseline"] = cpu_baseline
    return result


def execution_failed_result(case_id: int, config: TransformerConfig, failure_category: str,
                            error: BaseException) -> Dict[str, object]:
    return {
        "case_id": case_id,
        "config": asdict(config),
        "status": "execution_failed",
        "failure_category": failure_category,
        "correctness_passed": None,
        "accuracy": None,
        "performance": None,
        "error": str(error),
    }


def environment_metadata(device: torch.device, dtype: torch.dtype) -> Dict[str, object]:
    return {
        "python_version": platform.python_version(),
        "platform": platform.platform(),
        "device": str(device),
        "dtype": str(dtype),
        "torch_version": torch.__version__,
        "cuda_version": torch.version.cuda,
        "gpu": torch.cuda.get_device_name(device) if device.type == "cuda" else None,
        "pytorch_cuda_alloc_conf": os.environ.get("PYTORCH_CUDA_ALLOC_CONF"),
    }


def matrix_document(requested_case_ids: List[int], case_results: List[Dict[str, object]],
                    environment: Dict[str, object], settings: Dict[str, object]) -> Dict[str, object]:
    """The official-matrix document of runner.py:463-499."""
    complete = len(case_results) == len(requested_case_ids)
    all_cases_executed = complete and all(r["status"] != "execution_failed" for r in case_results)
    if not all_cases_executed:
        correctness_passed: Optional[bool] = None
        failure_category: Optional[str] = "execution" if complete else None
    elif all(r["correctness_passed"] is True for r in case_results):
        correctness_passed, failure_category = True, None
    else:
        correctness_passed, failure_category = False, "correctness"
    counts = [e["gpus"] for r in case_results for e in (r.get("gpus") or [])]
    return {
        "schema_version": SCHEMA_VERSION,
        "mode": "official_matrix",
        "gpus": max(counts) if counts else 1,
        "case_set": CASE_SET,
        "requested_case_ids": list(requested_case_ids),
        "complete": complete,
        "all_cases_executed": all_cases_executed,
        "environment": environment,
        "settings": settings,
        "failure_category": failure_category,
        "correctness_passed": correctness_passed,
        "cases": case_results,
    }


def _json_safe(value):
    if isinstance(value, float) and not math.isfinite(value):
        return None
    if isinstance(value, dict):
        return {k: _json_safe(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [_json_safe(v) for v in value]
    return value


def write_json_document(path: Path, document: Dict[str, object]) -> None:
    """Atomic write (temporary file + rename), non-finite floats as null, as runner.py:251-270."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.tmp")
    tmp.write_text(json.dumps(_json_safe(document), indent=2, allow_nan=False) + "\n", encoding="utf-8")
    tmp.replace(path)
