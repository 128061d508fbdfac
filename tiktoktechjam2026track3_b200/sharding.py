"""Multi-GPU execution of the encoder stack: batch shards and head/FFN-column tensor parallelism.

The reference runs on one GPU only (it has no torch.distributed or NCCL call site); these plans
are this build's own, one process per GPU with torch.distributed (NCCL) for the plumbing:

* Batch shards (B >= number of GPUs): sequences are independent, so rank r runs the whole stack on
  its contiguous slice of the batch (`batch_shard`) with no collective in the data path. The
  kernels are row- and batch-invariant, so a shard's output is bit-identical to the same rows of
  a single-GPU run.

* Tensor parallelism (B < number of GPUs, e.g. one 32768-token sequence): attention heads and FFN
  columns are split across ranks (Megatron-style). Rank r owns heads [r*H/n, (r+1)*H/n): rows of
  q/k/v_proj and the matching columns of out_proj; and FFN columns [r*F/n, (r+1)*F/n): rows of
  ffn_in and columns of ffn_out. LayerNorms are replicated. Each residual sub-block ends in a
  per-rank fp32 partial sum [T, D] that is all-reduced over NCCL (two all-reduces per block, one
  per residual sub-block); the biases of out_proj/ffn_out are added once, after the reduction,
  in the fused residual + LayerNorm kernel (b2_add_layernorm_fwd).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from . import _capi
from .cases import TransformerConfig, config_from
from .models import MaskLengths


def batch_shard(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of the batch owned by `rank` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def tp_check(config: TransformerConfig, world: int) -> None:
    """Raises ValueError unless heads and FFN columns split evenly into 64-aligned shards."""
    cfg = config_from(config)
    if cfg.num_heads % world:
        raise ValueError(f"num_heads={cfg.num_heads} is not divisible by {world} ranks")
    if cfg.ffn_dim % world or (cfg.ffn_dim // world) % 64:
        raise ValueError(f"ffn_dim={cfg.ffn_dim} does not split into 64-aligned shards over {world} ranks")
    if (cfg.d_model // world) % 64:
        raise ValueError(f"d_model/{world} must be a multiple of 64")


def tp_shard_state(state: Dict[str, torch.Tensor], config, world: int, rank: int) -> List[Dict[str, torch.Tensor]]:
    """Per-layer weight shards of `rank` from a full state dict with the reference's key names."""
    cfg = config_from(config)
    tp_check(cfg, world)
    hd = cfg.head_dim
    heads = cfg.num_heads // world
    c0, c1 = rank * heads * hd, (rank + 1) * heads * hd
    fw = cfg.ffn_dim // world
    f0, f1 = rank * fw, (rank + 1) * fw
    out = []
    for i in range(cfg.num_layers):
        p = f"layers.{i}"
        a = f"{p}.attention"
        shard = {
            "ln1_w": state[f"{p}.norm1.weight"],
            "ln1_b": state[f"{p}.norm1.bias"],
            "w_qkv": torch.cat([state[f"{a}.{n}_proj.weight"][c0:c1] for n in ("q", "k", "v")], 0),
            "b_qkv": torch.cat([state[f"{a}.{n}_proj.bias"][c0:c1] for n in ("q", "k", "v")], 0),
            "w_o": state[f"{a}.out_proj.weight"][:, c0:c1],
            "b_o": state[f"{a}.out_proj.bias"],
            "ln2_w": state[f"{p}.norm2.weight"],
            "ln2_b": state[f"{p}.norm2.bias"],
            "w_1": state[f"{p}.ffn_in.weight"][f0:f1],
            "b_1": state[f"{p}.ffn_in.bias"][f0:f1],
            "w_2": state[f"{p}.ffn_out.weight"][:, f0:f1],
            "b_2": state[f"{p}.ffn_out.bias"],
        }
        out.append({k: v.contiguous() for k, v in shard.items()})
    return out


class TensorParallelTransformer:
    """Forward pass of the stack with heads/FFN columns split over a process group.

    Every rank passes the same x [B, S, D] (bf16, on its own GPU) and mask, and receives the full
    output. Built from the full model's state dict (reference key names).
    """

    def __init__(self, config, state: Dict[str, torch.Tensor], device: torch.device, group=None) -> None:
        import torch.distributed as dist

        self.config = config_from(config)
        self.config.validate()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        tp_check(self.config, self.world)
        full = {k: v.to(device=device, dtype=torch.bfloat16) for k, v in state.items()}
        self.shards = tp_shard_state(full, self.config, self.world, self.rank)
        self.final_w = full["final_norm.weight"].contiguous()
        self.final_b = full["final_norm.bias"].contiguous()
        self.eps = 1e-5
        self._mask_lengths = MaskLengths()
        self._launch_log: Optional[list] = None

    def record_launches(self, enabled: bool) -> None:
        """When enabled, every kernel launch and all-reduce is bracketed by CUDA events."""
        self._launch_log = [] if enabled else None

    def take_launch_log(self) -> list:
        log = self._launch_log or []
        if self._launch_log is not None:
            self._launch_log = []
        return log

    def _timed(self, kind: str, fn, *args, **kwargs) -> None:
        if self._launch_log is None:
            fn(*args, **kwargs)
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn(*args, **kwargs)
        end.record()
        self._launch_log.append((kind, start, end))

    def _all_reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_reduce(t, group=self.group)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        cfg = self.config
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("TensorParallelTransformer needs a bf16 CUDA input")
        batch, seq_len, d = x.shape
        if valid_token_mask is not None and valid_token_mask.device != x.device:
            raise ValueError("valid_token_mask must be on x's device")
        kv_len, row_mask = self._mask_lengths(valid_token_mask, batch, seq_len)
        n = self.world
        tokens = batch * seq_len
        h_loc = cfg.num_heads // n
        hd = cfg.head_dim
        d_loc = h_loc * hd
        f_loc = cfg.ffn_dim // n
        dev = x.device
        resid = torch.empty(tokens, d, device=dev, dtype=torch.float32)
        ln = torch.empty(tokens, d, device=dev, dtype=torch.bfloat16)
        qkv = torch.empty(tokens, 3 * d_loc, device=dev, dtype=torch.bfloat16)
        ctx = torch.empty(tokens, d_loc, device=dev, dtype=torch.bfloat16)
        hidden = torch.empty(tokens, f_loc, device=dev, dtype=torch.bfloat16)
        part = torch.empty(tokens, d, device=dev, dtype=torch.float32)
        out = torch.empty(batch, seq_len, d, device=dev, dtype=torch.bfloat16)
        x2 = x.contiguous().view(tokens, d)
        s0 = self.shards[0]
        t = self._timed
        t("layernorm", _capi.layernorm, x2, s0["ln1_w"], s0["ln1_b"], self.eps, ln, resid_out=resid)
        for i, s in enumerate(self.shards):
            t("gemm_qkv", _capi.linear, ln, s["w_qkv"], s["b_qkv"], _capi.EPI_BIAS, qkv)
            t("attention", _capi.attention, qkv, batch, seq_len, h_loc, hd, 0, d_loc, 2 * d_loc, kv_len, cfg.causal,
              hd**-0.5, ctx)
            t("gemm_out", _capi.linear, ctx, s["w_o"], None, _capi.EPI_STORE_F32, part)
            t("allreduce", self._all_reduce, part)
            t("layernorm", _capi.add_layernorm, resid, part, s["b_o"], s["ln2_w"], s["ln2_b"], self.eps, ln, row_mask,
              0)
            t("gemm_ffn_in", _capi.linear, ln, s["w_1"], s["b_1"], _capi.EPI_BIAS_GELU, hidden)
            t("gemm_ffn_out", _capi.linear, hidden, s["w_2"], None, _capi.EPI_STORE_F32, part)
            t("allreduce", self._all_reduce, part)
            last = i == len(self.shards) - 1
            g, b = (self.final_w, self.final_b) if last else (self.shards[i + 1]["ln1_w"], self.shards[i + 1]["ln1_b"])
            flags = _capi.ADD_LN_ZERO_ROWS | (_capi.ADD_LN_ZERO_Y if last else 0)
            t("layernorm", _capi.add_layernorm, resid, part, s["b_2"], g, b, self.eps,
              out.view(tokens, d) if last else ln, row_mask, flags)
        return out

    __call__ = forward

    @staticmethod
    def launches_per_forward(num_layers: int) -> int:
        return 1 + 7 * num_layers
