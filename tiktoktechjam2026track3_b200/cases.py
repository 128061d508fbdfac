"""Benchmark case record and the benchmark configurations (c1-c5) this build is measured on.

`TransformerConfig` mirrors the reference's frozen dataclass (transformer_benchmark/cases.py:11-38):
same field names and order, same validation messages, so a reference TransformerConfig and this
one are interchangeable wherever a config is read by attribute.

`BASELINE_CONFIGS` are the five configurations the build is measured and checked on (C1 is the
reference's CPU-runnable case; C2..C5 are the B200 workloads). `input_seed`/`padding_ratio`
feed the reference's generator (transformer_benchmark/cases.py:60-98); C2's ratio 0.5 gives
sequence lengths uniform in [256, 512].
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import torch


@dataclass(frozen=True)
class TransformerConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def tokens(self) -> int:
        return self.batch_size * self.seq_len


@dataclass(frozen=True)
class Workload:
    name: str
    config: TransformerConfig
    padding_ratio: float
    description: str


BASELINE_CONFIGS: Dict[str, Workload] = {
    "c1": Workload("c1", TransformerConfig(2, 128, 256, 4, 1024, 2, True), 0.0,
                   "reference CPU-runnable case, causal"),
    "c2": Workload("c2", TransformerConfig(8, 512, 768, 12, 3072, 12, False), 0.5,
                   "encoder stack with padding key mask, lengths uniform in [256, 512]"),
    "c3": Workload("c3", TransformerConfig(16, 2048, 1024, 16, 4096, 4, True), 0.0,
                   "causal, batch-sharded across GPUs"),
    "c4": Workload("c4", TransformerConfig(1, 32768, 2048, 16, 8192, 2, True), 0.0,
                   "single long sequence, causal, head/FFN tensor parallel on several GPUs"),
    "c5": Workload("c5", TransformerConfig(32, 100000, 1024, 16, 1024, 2, True), 0.0,
                   "very long sequences, causal, 4 sequences per GPU on 8 GPUs"),
}


def config_from(obj) -> TransformerConfig:
    """Accepts this module's or the reference's TransformerConfig (or any object with its fields)."""
    if isinstance(obj, TransformerConfig):
        return obj
    return TransformerConfig(
        int(obj.batch_size),
        int(obj.seq_len),
        int(obj.d_model),
        int(obj.num_heads),
        int(obj.ffn_dim),
        int(obj.num_layers),
        bool(obj.causal),
    )


def generate_random_case(
    config,
    device: torch.device,
    dtype: torch.dtype,
    seed: int,
    padding_ratio: float,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded inputs with the reference generator's calls and order (cases.py:60-98).

    x ~ N(0, 1) * input_scale drawn from a generator on `device`; with padding_ratio > 0,
    per-sequence lengths uniform in [max(1, round(S * (1 - ratio))), S], a prefix mask, and padded
    positions of x zeroed. Returns (x [B, S, D], valid_token_mask [B, S] bool).
    """
    cfg = config_from(config)
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, generator=generator, device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(cfg.batch_size, cfg.seq_len, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=cfg.seq_len + 1, size=(cfg.batch_size,), generator=generator,
                            device=device)
    positions = torch.arange(cfg.seq_len, device=device)[None, :]
    mask = positions < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


# The reference's official case matrix (competition appendix 3.7; transformer_benchmark/cases.py:
# 42-57): case ids are one-based positions in this tuple, as the reference numbers them.
OFFICIAL_TEST_CASES: Tuple[TransformerConfig, ...] = (
    TransformerConfig(64, 128, 128, 4, 128, 4, True),
    TransformerConfig(1, 128, 128, 4, 128, 4, True),
    TransformerConfig(4, 128, 128, 4, 128, 4, True),
    TransformerConfig(16, 128, 128, 4, 128, 4, True),
    TransformerConfig(128, 128, 128, 4, 128, 4, True),
    TransformerConfig(10000, 128, 128, 4, 128, 4, True),
    TransformerConfig(64, 128, 32, 4, 32, 4, True),
    TransformerConfig(64, 128, 1024, 4, 1024, 4, True),
    TransformerConfig(64, 128, 128, 1, 128, 4, True),
    TransformerConfig(64, 128, 128, 2, 128, 4, True),
    TransformerConfig(64, 128, 128, 16, 128, 4, True),
    TransformerConfig(64, 32, 128, 4, 128, 4, True),
    TransformerConfig(64, 1024, 128, 4, 128, 4, True),
    TransformerConfig(32, 100000, 1024, 16, 1024, 2, True),
)
