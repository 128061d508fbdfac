"""Generates the golden vectors that pin oracle/reference_fp32.py to the reference itself.

Run in a container where the reference source tree is importable (it is not on GPU boxes):

    REFERENCE_ROOT=<path to Sober7135/TikTokTechJam2026Track3 checkout> python tests/golden/make_golden.py

For each case it imports the reference's own modules — TransformerConfig and
generate_random_case (transformer_benchmark/cases.py:11-98), BaselineTransformer
(transformer_benchmark/models.py:895-919) — seeds exactly as the reference runner does
(torch.manual_seed(seed) before building the model, transformer_benchmark/runner.py:316-321),
draws the inputs on CPU with the reference generator, and runs the reference forward pass in
fp32 on CPU twice: with the model's fp32 weights and inputs, and with weights and inputs
rounded to bf16 (the values the GPU path computes with). It stores:
  * per-parameter (sum, sum of squares) in float64 — pins the weight construction;
  * (sum, sum of squares) and the first 256 values of the input x, and the valid-token mask —
    pins the input generator;
  * both outputs in float32.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, batch, seq_len, d_model, heads, ffn_dim, layers, causal, padding_ratio, seed)
CASES = [
    # Benchmark config 1 (the reference's CPU-runnable case).
    ("c1_causal", 2, 128, 256, 4, 1024, 2, True, 0.0, 0),
    # Padding mask, non-causal, ragged lengths, S not a multiple of 128.
    ("pad_noncausal", 3, 96, 128, 2, 256, 2, False, 0.5, 1),
    # Causal and padding together, head_dim 128.
    ("causal_pad_hd128", 2, 160, 128, 1, 512, 1, True, 0.3, 2),
]


def main() -> None:
    ref_root = os.environ.get("REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, ref_root)
    from transformer_benchmark.cases import TransformerConfig, generate_random_case
    from transformer_benchmark.models import BaselineTransformer

    manifest = {}
    for name, b, s, d, h, f, l, causal, pad, seed in CASES:
        config = TransformerConfig(b, s, d, h, f, l, causal)
        config.validate()
        torch.manual_seed(seed)
        model = BaselineTransformer(config).eval()
        state = model.state_dict()
        x, mask = generate_random_case(config, torch.device("cpu"), torch.float32, seed, pad, 1.0)
        with torch.inference_mode():
            out_fp32 = model(x, mask)
            model_b = BaselineTransformer(config).eval()
            model_b.load_state_dict({k: v.to(torch.bfloat16).float() for k, v in state.items()})
            xb = x.to(torch.bfloat16).float()
            out_bf16w = model_b(xb, mask)
        keys = sorted(state.keys())
        sums = np.array([[state[k].double().sum().item(), (state[k].double() ** 2).sum().item()] for k in keys])
        np.savez_compressed(
            HERE / f"{name}.npz",
            x_sums=np.array([x.double().sum().item(), (x.double() ** 2).sum().item()]),
            x_head=x.reshape(-1)[:256].numpy().astype(np.float32),
            mask=mask.numpy(),
            out_fp32=out_fp32.numpy().astype(np.float32),
            out_bf16_inputs=out_bf16w.numpy().astype(np.float32),
            param_keys=np.array(keys),
            param_sums=sums,
        )
        manifest[name] = {
            "batch_size": b, "seq_len": s, "d_model": d, "num_heads": h, "ffn_dim": f, "num_layers": l,
            "causal": causal, "padding_ratio": pad, "seed": seed, "torch": torch.__version__,
        }
        print(name, "max|out|", float(out_fp32.abs().max()))
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
