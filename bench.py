#!/usr/bin/env python3
"""Forward-pass throughput of the Transformer encoder stack on B200s (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2] [--impl ours|reference]

A step is one forward pass of UserOptimizedTransformer over one batch of synthetic inputs with
the benchmark configuration's shapes (x ~ N(0,1) and padding lengths from the reference's
generator with seed 100000, weights from the reference's default init under torch.manual_seed(0)).

Workloads (the benchmark configurations; the global batch is fixed, so N GPUs split the same
work — strong scaling — one process per GPU launched by torch.distributed.run):
  c2 (default)  B=8  S=512    D=768  H=12 F=3072 L=12, padding mask (lengths in [256, 512])
  c3            B=16 S=2048   D=1024 H=16 F=4096 L=4, causal
  c5            B=32 S=100000 D=1024 H=16 F=1024 L=2, causal (4 sequences per GPU on 8 GPUs)
  c1            B=2  S=128    D=256  H=4  F=1024 L=2, causal
  c4            B=1  S=32768  D=2048 H=16 F=8192 L=2, causal
With B >= N every rank runs a contiguous shard of B/N sequences (no collective in the data path);
with B < N the sequence is split over the ranks (context parallel by default, tensor parallel with
--split tp). --per-gpu-batch B' runs B' sequences on every rank instead (weak scaling).

Reported (rank 0): `value` = tokens/s of the whole job (B*S of the global batch per step) with
inputs resident in HBM, each of the K timed steps bracketed by barrier + synchronize and timed
with CUDA events on the launching stream, L2 flushed (256 MiB write) before every step, max over
ranks; `e2e` = the same forward through the public module API with each rank's input copied from
pinned host memory and the output copied back inside the timed region; `roofline` = the dominant
kernel class (by device time) against the measured peak, with its time both as launched alone
(per-launch CUDA events) and as its share of the measured step; `cpu_baseline` = the fp32 CPU
restatement of the reference (oracle/) on a bounded sample, on the host's cores.

`--impl reference` times the same CPU sample as the reference arm (fp32, all host threads, the
oracle port of BaselineTransformer.forward; median of the K steps, the statistic cpu_baseline
uses) and prints the same line with "impl": "reference"; under torch.distributed.run only rank 0
runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

# NCCL writes its version banner and log lines to stdout (the banner even at NCCL_DEBUG=WARN) and
# fixes its log file when the library first initialises, which can happen while torch imports:
# send them to stderr before torch is imported, so that stdout carries only the one JSON line.
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

import torch  # noqa: E402

ROOT = Path(__file__).resolve().parent


class stdout_to_stderr:
    """Points file descriptor 1 at stderr for the duration (output of native libraries included)."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)
        return False

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from tiktoktechjam2026track3_b200 import UserOptimizedTransformer  # noqa: E402
from tiktoktechjam2026track3_b200.cases import BASELINE_CONFIGS, TransformerConfig, generate_random_case  # noqa: E402
from tiktoktechjam2026track3_b200.models import attention_kernel_name  # noqa: E402

METRIC = "forward_tokens_per_sec"
UNIT = "tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_FLUSH_BYTES = 256 << 20
LONG_STEP_MS = 50.0
TRAFFIC_FILE = ROOT / "tiktoktechjam2026track3_b200" / "data" / "ncu_dram_traffic.json"


def dram_traffic(workload: str, world: int, kernel: str, ln_fused: bool):
    """DRAM bytes per launch of `kernel` from the committed ncu figures (None if not captured)."""
    try:
        entries = json.loads(TRAFFIC_FILE.read_text())["entries"]
    except (OSError, ValueError, KeyError):
        return None, None
    for e in entries:
        if (e["workload"], e["world"], e["kernel"], e["layernorm_fused"]) == (workload, world, kernel, ln_fused):
            return e["bytes_per_launch"], e["source"]
    return None, None


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--workload", default="c2", choices=sorted(BASELINE_CONFIGS))
    p.add_argument("--impl", default="ours", choices=("ours", "reference"))
    p.add_argument("--split", default="cp", choices=("tp", "cp"),
                   help="batch smaller than the GPU count: head/FFN tensor parallel (tp) or context parallel (cp)")
    p.add_argument("--collective", default="auto", choices=("auto", "rs", "nccl"),
                   help="tensor-parallel reduction: reduce-scatter in the GEMMs + all-gather in the LayerNorm over "
                        "NVLink (rs), or NCCL all-reduce")
    p.add_argument("--fuse-ln", default="auto", choices=("auto", "on", "off"),
                   help="LayerNorm inside the out_proj / ffn_out GEMM epilogues (auto: where the library recommends "
                        "it; nowhere in this build, it measured slower than the separate LayerNorm)")
    p.add_argument("--per-gpu-batch", type=int, default=0,
                   help="sequences per GPU (weak scaling); default 0 = split the configuration's global batch")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU time of the CPU baseline sample")
    return p.parse_args(argv)


def workload_config(name: str, batch: int = 0) -> tuple[TransformerConfig, float]:
    """The benchmark configuration `name` (its global batch, or `batch` sequences if given)."""
    w = BASELINE_CONFIGS[name]
    c = w.config
    cfg = TransformerConfig(batch or c.batch_size, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.num_layers,
                            c.causal)
    return cfg, w.padding_ratio


def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            data = json.loads(path.read_text())
            return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                    "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"]))}, "measured"
        except (KeyError, ValueError):
            pass
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0), "fallback"


# ----------------------------------------------------------------------------- algorithmic work
def gemm_flops(cfg: TransformerConfig) -> dict:
    t = cfg.batch_size * cfg.seq_len
    d, f = cfg.d_model, cfg.ffn_dim
    per_layer = {
        "gemm_qkv": 2.0 * t * d * 3 * d,
        "gemm_out": 2.0 * t * d * d,
        "gemm_ffn_in": 2.0 * t * d * f,
        "gemm_ffn_out": 2.0 * t * f * d,
    }
    return {k: v * cfg.num_layers for k, v in per_layer.items()}


def attention_flops(cfg: TransformerConfig, lengths) -> float:
    lens = [cfg.seq_len] * cfg.batch_size if lengths is None else [int(v) for v in lengths]
    pairs = sum(n * (n + 1) / 2.0 for n in lens) if cfg.causal else sum(float(n) * n for n in lens)
    return cfg.num_layers * 4.0 * cfg.d_model * pairs


def layernorm_bytes(cfg: TransformerConfig, fused: bool = False) -> float:
    """Bytes of the LayerNorm launches: the first norm reads bf16 x and writes the fp32 residual + bf16
    (8 B/elt); each other norm reads fp32 and writes bf16 (6 B/elt) — 2L of them, or only the final
    norm when norm2 / norm1 run inside the residual GEMMs (their work is then part of those launches)."""
    t, d, layers = cfg.batch_size * cfg.seq_len, cfg.d_model, cfg.num_layers
    return t * d * (8.0 + 6.0 * (1 if fused else 2 * layers))


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons of one GPU while the timed region runs.

    Reads NVML (read-only queries) from a background thread every 2 ms, so that even a timed
    region of a few milliseconds gets samples; falls back to `nvidia-smi -lms 200` without NVML.
    """

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device: torch.device):
        props = torch.cuda.get_device_properties(device)
        self.bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        self.samples: list = []
        self._stop = None
        self._thread = None
        self._proc = None
        self.source = "nvml"

    def _nvml_loop(self, nv, handle):
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetPowerUsage(handle) / 1000.0,
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(handle)))
            except Exception:  # noqa: BLE001 - a failed query only loses one sample
                pass
            self._stop.wait(0.002)

    def start(self):
        import threading

        self.samples = []
        try:
            import pynvml as nv

            nv.nvmlInit()
            handle = nv.nvmlDeviceGetHandleByPciBusId(self.bus)
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._nvml_loop, args=(nv, handle), daemon=True)
            self._thread.start()
            return
        except Exception:  # noqa: BLE001 - NVML missing: use nvidia-smi instead
            self.source = "nvidia-smi"
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.sw_power_cap,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown")
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.bus}", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            for line in out.strip().splitlines():
                parts = [x.strip() for x in line.split(",")]
                try:
                    bits = sum(bit for bit, flag in zip(self.REASONS, parts[3:7]) if flag.lower().startswith("active"))
                    self.samples.append((float(parts[0]), float(parts[1]), float(parts[2]), bits))
                except (ValueError, IndexError):
                    continue
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "unavailable"}
        reasons = sorted({name for _, _, _, bits in self.samples for bit, name in self.REASONS.items() if bits & bit})
        return {
            "sm_mhz": statistics.median(x[0] for x in self.samples) if self.samples else None,
            "sm_max_mhz": max(x[1] for x in self.samples) if self.samples else None,
            "power_w_max": max(x[2] for x in self.samples) if self.samples else None,
            "reasons": reasons,
            "samples": len(self.samples),
            "source": self.source,
        }


# ----------------------------------------------------------------------------- CPU legs (oracle)
def cpu_sample(cfg: TransformerConfig, padding_ratio: float, threads: int):
    """The bounded CPU sample of a workload: one sequence through the fp32 CPU restatement of the
    reference (all layers; for S = 100000 one of the layers, the time then scaled by the layer
    count — every layer does the same work). Returns (step, tokens per step, layer scale, text)."""
    from oracle import reference_fp32 as oracle  # CPU baseline / reference arm only

    torch.set_num_threads(threads)
    layers = 1 if cfg.seq_len >= 65536 else cfg.num_layers
    sample_cfg = TransformerConfig(1, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim, layers, cfg.causal)
    state = oracle.build_reference_state(sample_cfg, 0)
    x, mask = oracle.generate_random_case(sample_cfg, torch.device("cpu"), torch.float32, 100000, padding_ratio)
    use_mask = None if padding_ratio <= 0 else mask

    def step():
        with torch.inference_mode():
            oracle.forward(state, sample_cfg, x, use_mask, query_chunk=2048)

    text = (f"1 sequence (S={cfg.seq_len}, {layers} of {cfg.num_layers} layers) of the workload through the fp32 CPU "
            f"restatement of BaselineTransformer.forward (oracle/reference_fp32.py, attention in 2048-query chunks), "
            f"{threads} threads")
    return step, cfg.seq_len, cfg.num_layers / layers, text


def reference_path_record(cfg: TransformerConfig):
    """Whether the reference's own path (BaselineSelfAttention materialises [B, H, S, S] scores,
    models.py:55-75) fits this host for one sequence; None when it does. The reference's runner
    records a run that dies of memory as execution_failed / out_of_memory (runner.py:445-460,
    527-531); here the need is computed instead of provoked on a shared host."""
    try:
        import psutil

        host = psutil.virtual_memory().total
    except Exception:  # noqa: BLE001 - psutil missing: no prediction
        return None
    scores = cfg.num_heads * float(cfg.seq_len) ** 2 * 4  # one fp32 [1, H, S, S] copy
    need = 4 * scores  # scores, scaled/masked copy, softmax output and its bf16/fp32 round trip
    if need <= 0.8 * host:
        return None
    return {"status": "execution_failed", "failure_category": "out_of_memory",
            "error": (f"not run (predicted): one sequence needs ~4 fp32 [1, {cfg.num_heads}, {cfg.seq_len}, "
                      f"{cfg.seq_len}] score copies = {need / 1e9:.0f} GB against {host / 1e9:.0f} GB of host memory")}


def cpu_times(step, target_seconds: float, max_samples: int, min_samples: int = 1):
    """Runs `step` until target_seconds have passed (at least min_samples, at most max_samples),
    after one warm-up unless a single step is longer than a quarter of the target."""
    t_begin = t0 = time.perf_counter()
    step()
    first = time.perf_counter() - t0
    times = [] if first < target_seconds / 4 else [first]
    if times:  # a single step already took a quarter of the budget: time from here on
        t_begin = t0
    else:
        t_begin = time.perf_counter()
    while len(times) < max_samples and (len(times) < min_samples or time.perf_counter() - t_begin < target_seconds):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return times


def run_cpu_baseline(cfg, padding_ratio, target_seconds: float) -> dict:
    threads = os.cpu_count() or 1
    step, tokens, layer_scale, text = cpu_sample(cfg, padding_ratio, threads)
    times = cpu_times(step, target_seconds, max_samples=50)
    per = statistics.median(times) * layer_scale
    rec = {
        "value": tokens / per,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"median of {len(times)} forwards of {text}: {per * 1e3:.1f} ms per sequence",
    }
    ref_path = reference_path_record(cfg)
    if ref_path is not None:
        rec["reference_path"] = ref_path
    return rec


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, pad = workload_config(args.workload)
    threads = os.cpu_count() or 1
    step, tokens, layer_scale, text = cpu_sample(cfg, pad, threads)
    for _ in range(max(args.warmup, 0)):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    per = statistics.median(times) * layer_scale
    value = tokens / per
    sample = f"each step: {text}; median of the {args.steps} steps"
    cpu = {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
    ref_path = reference_path_record(cfg)
    if ref_path is not None:
        cpu["reference_path"] = ref_path
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": args.workload, "model": "transformer_encoder", "global_batch": cfg.batch_size,
                   "seq_len": cfg.seq_len, "d_model": cfg.d_model, "layers": cfg.num_layers,
                   "parallelism": "cpu", "sample_sequences_per_step": 1},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def class_times(log, reps: int):
    """Per launch kind: device ms per forward and launches per forward, from a launch log."""
    kind_ms: dict = {}
    kind_n: dict = {}
    for kind, s, e in log:
        kind_ms[kind] = kind_ms.get(kind, 0.0) + s.elapsed_time(e) / reps
        kind_n[kind] = kind_n.get(kind, 0) + 1
    return kind_ms, {k: v // reps for k, v in kind_n.items()}


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist

        # The communicator is created here (device_id: eager init) and by the first barrier; anything
        # NCCL prints to file descriptor 1 while it starts goes to stderr.
        with stdout_to_stderr():
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
            dist.barrier()

    weak = args.per_gpu_batch > 0
    gcfg, pad = workload_config(args.workload, args.per_gpu_batch * world if weak else 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    # The global batch is split over the ranks: B >= N gives every rank a contiguous shard of
    # whole sequences (no collective in the data path); B < N splits each sequence over the ranks
    # (context parallel by default, tensor parallel with --split tp).
    split_sequences = world > 1 and gcfg.batch_size < world
    x_all, mask_all = generate_random_case(gcfg, device, torch.bfloat16, 100000, pad)
    if split_sequences:
        from tiktoktechjam2026track3_b200.sharding import ContextParallelTransformer, TensorParallelTransformer

        cfg = gcfg
        full = UserOptimizedTransformer(cfg)
        if args.split == "cp":
            model = ContextParallelTransformer(cfg, full.state_dict(), device)
        else:
            model = TensorParallelTransformer(cfg, full.state_dict(), device, collective=args.collective)
        del full
        x, mask = x_all, mask_all
        shard = (0, gcfg.batch_size)
    else:
        from tiktoktechjam2026track3_b200.sharding import batch_shard

        shard = batch_shard(gcfg.batch_size, world, rank)
        cfg = TransformerConfig(shard[1] - shard[0], gcfg.seq_len, gcfg.d_model, gcfg.num_heads, gcfg.ffn_dim,
                                gcfg.num_layers, gcfg.causal)
        model = UserOptimizedTransformer(cfg).to(device=device, dtype=torch.bfloat16).eval()
        model.fuse_layernorm = {"auto": "auto", "on": True, "off": False}[args.fuse_ln]
        x = x_all[shard[0]:shard[1]].contiguous()
        mask = mask_all[shard[0]:shard[1]].contiguous()
    del x_all, mask_all
    ln_fused = (not split_sequences) and model.layernorm_fused(cfg.batch_size * cfg.seq_len)
    lengths = mask.sum(1).tolist() if pad > 0 else None
    use_mask = mask  # the harness always passes a mask; all-true masks are elided by the model
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=device, dtype=torch.float32)

    def barrier():
        if dist is not None:
            dist.barrier()

    def gather(obj):
        if dist is None:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x, use_mask)
        torch.cuda.synchronize()

        # ---------------- device-timed steps (inputs resident in HBM)
        stream = torch.cuda.current_stream(device)
        sampler = ClockSampler(device)
        sampler.start()
        step_ms = []
        for _ in range(args.steps):
            flush.fill_(1.0)
            barrier()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            model(x, use_mask)
            end.record(stream)
            torch.cuda.synchronize()
            barrier()
            step_ms.append(start.elapsed_time(end))
        clocks = sampler.stop()
        total_ms = torch.tensor([sum(step_ms)], device=device, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
        total_ms = float(total_ms.item())
        ms_per_step = total_ms / args.steps
        tokens_per_step = gcfg.batch_size * gcfg.seq_len
        value = tokens_per_step / (ms_per_step / 1e3)

        # ---------------- end to end through the public API, host buffers
        x_host = x.cpu().pin_memory()
        m_host = use_mask.cpu().pin_memory()
        y_host = torch.empty(x.shape, dtype=torch.bfloat16).pin_memory()
        e2e_ms = []
        for i in range(args.warmup + args.steps):
            flush.fill_(1.0)
            barrier()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            xd = x_host.to(device, non_blocking=True)
            md = m_host.to(device, non_blocking=True)
            y = model(xd, md)
            y_host.copy_(y, non_blocking=True)
            end.record(stream)
            torch.cuda.synchronize()
            barrier()
            if i >= args.warmup:
                e2e_ms.append(start.elapsed_time(end))
        e2e_total = torch.tensor([sum(e2e_ms)], device=device, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
        e2e_per_step = float(e2e_total.item()) / args.steps
        h2d = x_host.numel() * x_host.element_size() + m_host.numel() * m_host.element_size()
        d2h = y_host.numel() * y_host.element_size()
        # Every rank copies its own shard (sequence-split plans: the whole, replicated, input).
        io_bytes = gather((h2d, d2h))

        # ---------------- per-kernel device times (roofline of the dominant kernel)
        # Each eager forward is queued behind a ~20 ms GPU sleep, so the host enqueues every launch
        # before the GPU reaches it and the per-launch events time the kernels, not launch overhead.
        # Events between launches break the programmatic-dependent-launch overlap of the graph
        # replayed in the timed steps, so these are launch-alone times; each class is also
        # reported as its share of the measured step.
        model.record_launches(True)
        reps = 3
        for _ in range(reps):
            flush.fill_(1.0)
            torch.cuda._sleep(40_000_000)
            model(x, use_mask)
        torch.cuda.synchronize()
        log = model.take_launch_log()
        model.record_launches(False)
        model._status.check(wait=True)  # a timed-out kernel invalidates the run

    kind_ms, kind_n = class_times(log, reps)
    per_rank = gather({"rank": rank, "ms_per_step": sum(step_ms) / args.steps,
                       "sequences": shard[1] - shard[0] if not split_sequences else gcfg.batch_size,
                       "tokens_valid": int(sum(lengths)) if lengths is not None else cfg.batch_size * cfg.seq_len,
                       "ms_by_launch_kind": {k: round(v, 4) for k, v in sorted(kind_ms.items())}})
    flops = gemm_flops(cfg)
    attn = attention_flops(cfg, lengths)
    gemm_total = sum(flops.values())
    if split_sequences:  # per-rank work: heads / FFN columns or token rows are split over the ranks
        gemm_total /= world
        attn /= world
    peaks, peak_src = measured_peaks()
    # A kernel inside a long step runs at the power-capped clock: compare it with the sustained
    # GEMM figure; short steps run at boost clock: the burst figure.
    long_step = ms_per_step > LONG_STEP_MS
    tensor_peak = peaks["bf16_tflops_sustained"] if long_step else peaks["bf16_tflops"]
    tensor_peak_name = "bf16 sustained" if long_step else "bf16 burst"
    classes = {
        "gemm_tc_kernel": {"ms": sum(v for k, v in kind_ms.items() if k.startswith("gemm")), "work": gemm_total,
                           "bound": "tensor",
                           "launches": sum(v for k, v in kind_n.items() if k.startswith("gemm"))},
        attention_kernel_name(cfg.head_dim): {"ms": kind_ms.get("attention", 0.0), "work": attn, "bound": "tensor",
                                               "launches": kind_n.get("attention", 0)},
        "layernorm_vec_kernel": {"ms": kind_ms.get("layernorm", 0.0), "work": layernorm_bytes(cfg, ln_fused),
                                 "bound": "hbm", "launches": kind_n.get("layernorm", 0)},
    }
    if split_sequences:
        classes["layernorm_vec_kernel"]["work"] /= world
    # This rank's step time spread over its launch kinds in proportion to their launch-alone times.
    my_step = sum(step_ms) / args.steps
    alone_sum = sum(kind_ms.values())
    in_step_scale = my_step / alone_sum if alone_sum > 0 else 0.0
    kernels = {}
    for name, c in classes.items():
        if c["ms"] <= 0:
            continue
        peak = tensor_peak if c["bound"] == "tensor" else peaks["hbm_gbs"]
        div = 1e12 if c["bound"] == "tensor" else 1e9
        achieved = c["work"] / (c["ms"] / 1e3) / div
        in_step_ms = c["ms"] * in_step_scale
        achieved_in_step = c["work"] / (in_step_ms / 1e3) / div
        kernels[name] = {"ms_per_step": c["ms"], "launches_per_step": c["launches"], "achieved": achieved,
                         "unit": "TFLOP/s" if c["bound"] == "tensor" else "GB/s", "frac": achieved / peak,
                         "in_step_ms": in_step_ms, "achieved_in_step": achieved_in_step,
                         "frac_in_step": achieved_in_step / peak}
    dominant = max(classes, key=lambda k: classes[k]["ms"])
    dk = kernels[dominant]
    traffic, traffic_src = dram_traffic(args.workload, world, dominant, ln_fused) if not weak else (None, None)
    roofline = {
        "kernel": dominant,
        "bound": classes[dominant]["bound"],
        "achieved": dk["achieved"],
        "peak": tensor_peak if classes[dominant]["bound"] == "tensor" else peaks["hbm_gbs"],
        "peak_source": f"{peak_src} ({tensor_peak_name if classes[dominant]['bound'] == 'tensor' else 'HBM copy'})",
        "unit": dk["unit"],
        "frac": dk["frac"],
        "achieved_in_step": dk["achieved_in_step"],
        "frac_in_step": dk["frac_in_step"],
        "timing": ("achieved/frac: launch-alone CUDA events around each launch of the class (eager pass); "
                   "*_in_step: the measured step time split over the launch kinds in proportion to those times "
                   f"(launch-alone sum {alone_sum:.4f} ms vs step {my_step:.4f} ms on rank {rank})"),
        "traffic": traffic,
        "traffic_source": traffic_src,
        "work_per_launch": classes[dominant]["work"] / max(1, classes[dominant]["launches"]),
    }
    total_flops = gemm_total + attn  # per rank
    mfu = total_flops / (ms_per_step / 1e3) / 1e12 / tensor_peak

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline(gcfg, pad, args.cpu_seconds)

    if rank == 0:
        slowest = max(per_rank, key=lambda r: r["ms_per_step"])
        slow_kinds = slowest["ms_by_launch_kind"]
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak" if weak else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": args.workload,
                "model": "transformer_encoder",
                "global_batch": gcfg.batch_size,
                "seq_len": gcfg.seq_len,
                "d_model": gcfg.d_model,
                "heads": gcfg.num_heads,
                "ffn_dim": gcfg.ffn_dim,
                "layers": gcfg.num_layers,
                "causal": gcfg.causal,
                "padding_ratio": pad,
                "parallelism": (f"cp{world} (each sequence's tokens in 2 x {world} zigzag chunks; Q/K/V rows "
                                "all-gathered over NVLink into every GPU's full-length buffer, attention of the "
                                "rank's query rows, LayerNorms and GEMMs on its own rows; 1 flag barrier per block)")
                if split_sequences and model.collective == "cp" else
                (f"tp{world} (heads / FFN columns; " + {
                    "rs": "out_proj / ffn_out GEMM epilogues add each row into its owner's fp32 residual over "
                          "NVLink (reduce-scatter), owners' LayerNorm rows stored into every GPU's buffer (all-gather), "
                          "4 flag barriers per block)",
                    "nccl": "2 NCCL all-reduces of the fp32 [T, D] partial per block)"}[model.collective])
                if split_sequences else
                f"dp{world} (batch shards, {'/'.join(str(r['sequences']) for r in per_rank)} sequences per GPU, "
                "no collective)",
                "l2": "flushed (256 MiB write) before every timed step",
                "launches": (f"eager launches ({model.collective})" if split_sequences else
                             "first/final LayerNorm eager, the block launches replayed from a CUDA graph"),
                "layernorm": ("norm2 and the next block's norm1 in the out_proj / ffn_out GEMM epilogues "
                              "(clusters spanning each row)") if ln_fused else "separate LayerNorm launches",
            },
            "roofline": roofline,
            "kernels": kernels,
            "model_flops_per_step": total_flops * world,
            "ms_per_step_by_launch_kind": {k: round(v, 4) for k, v in sorted(kind_ms.items())},
            "per_rank": per_rank if world > 1 else None,
            "limiter": ({"rank": slowest["rank"], "ms_per_step": slowest["ms_per_step"],
                         "kind": max(slow_kinds, key=slow_kinds.get) if slow_kinds else None,
                         "note": "the slowest rank sets the step; its largest launch kind (launch-alone times)"}
                        if world > 1 else None),
            "mfu_of_bf16_peak": mfu,
            "cpu_baseline": cpu,
            "e2e": {"value": tokens_per_step / (e2e_per_step / 1e3), "unit": UNIT, "ms_per_step": e2e_per_step,
                    "h2d_bytes_per_step": sum(b[0] for b in io_bytes),
                    "d2h_bytes_per_step": sum(b[1] for b in io_bytes)},
            "gpu_launches": args.steps * (model.launches_per_forward(cfg.num_layers) if split_sequences else
                                          UserOptimizedTransformer.launches_per_forward(cfg.num_layers, ln_fused)),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        torch.cuda.synchronize()
        if split_sequences:
            model.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
