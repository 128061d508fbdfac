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
  per-rank partial sum [T, D] that has to be summed over ranks, one reduction per residual
  sub-block. Two ways to do it (`collective=`):

  - "multimem" (default where the GPUs support NVLink SHARP multicast): the fp32 residual stream
    is replicated in symmetric memory, and the out_proj / ffn_out GEMMs add their partial tiles
    (plus the bias, on rank 0 only) straight into every rank's copy with multimem.red through the
    NVSwitch (B2_EPI_MC_RESIDUAL*), tile by tile while the GEMM runs. The reduction and the
    residual add happen inside the GEMM; four cross-GPU flag barriers per layer (b2_peer_barrier)
    order the residual's readers (LayerNorms) against the adds.
  - "nccl": each GEMM writes an fp32 partial, NCCL all-reduces it, and the fused residual +
    LayerNorm kernel (b2_add_layernorm_fwd) adds it with the bias. Kept as the baseline.
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

    def __init__(self, config, state: Dict[str, torch.Tensor], device: torch.device, group=None,
                 collective: str = "auto") -> None:
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
        if collective == "auto":
            collective = "multimem" if multicast_supported(device) and self.world > 1 else "nccl"
        if collective not in ("multimem", "nccl"):
            raise ValueError(f"collective must be 'auto', 'multimem' or 'nccl', not {collective!r}")
        if collective == "multimem" and not multicast_supported(device):
            raise RuntimeError("collective='multimem' needs NVLink SHARP multicast (symmetric memory) support")
        self.collective = collective
        self._symm: Optional[Tuple[int, torch.Tensor, object, int, List[int]]] = None

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

    def _symmetric_residual(self, tokens: int, d: int):
        """fp32 residual [tokens, d] in symmetric memory plus the ranks' barrier pads.

        Returns (resid, multicast address of resid, every rank's pad address). Allocated by a
        collective rendezvous the first time a token count is seen, then reused.
        """
        if self._symm is not None and self._symm[0] == tokens:
            return self._symm[1], self._symm[3], self._symm[4]
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = None
        words = tokens * d + 64  # the pad sits after the residual, 256-byte aligned
        buf = symm_mem.empty(words, dtype=torch.float32, device=self.device)
        buf[tokens * d:].zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(buf, group)
        mc = int(handle.multicast_ptr)
        if mc == 0:
            raise RuntimeError("symmetric memory has no multicast address on this device")
        pads = [int(p) + tokens * d * 4 for p in handle.buffer_ptrs]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every pad is zero before any rank signals
        self._symm = (tokens, buf[: tokens * d].view(tokens, d), handle, mc, pads)
        return self._symm[1], mc, pads

    def _barrier(self, pads: List[int], channel: int) -> None:
        _capi.peer_barrier(pads, self.rank, channel, self.device)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.collective == "multimem":
            return self._forward_multimem(x, valid_token_mask)
        return self._forward_nccl(x, valid_token_mask)

    def _forward_multimem(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
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
        resid, mc, pads = self._symmetric_residual(tokens, d)
        ln = torch.empty(tokens, d, device=dev, dtype=torch.bfloat16)
        qkv = torch.empty(tokens, 3 * d_loc, device=dev, dtype=torch.bfloat16)
        ctx = torch.empty(tokens, d_loc, device=dev, dtype=torch.bfloat16)
        hidden = torch.empty(tokens, f_loc, device=dev, dtype=torch.bfloat16)
        out = torch.empty(batch, seq_len, d, device=dev, dtype=torch.bfloat16)
        x2 = x.contiguous().view(tokens, d)
        lead = self.rank == 0  # adds the out_proj / ffn_out biases
        s0 = self.shards[0]
        t = self._timed
        t("layernorm", _capi.layernorm, x2, s0["ln1_w"], s0["ln1_b"], self.eps, ln, resid_out=resid)
        for i, s in enumerate(self.shards):
            t("gemm_qkv", _capi.linear, ln, s["w_qkv"], s["b_qkv"], _capi.EPI_BIAS, qkv)
            t("attention", _capi.attention, qkv, batch, seq_len, h_loc, hd, 0, d_loc, 2 * d_loc, kv_len, cfg.causal,
              hd**-0.5, ctx)
            t("barrier", self._barrier, pads, 0)  # every rank is done reading its residual copy
            t("gemm_out", _capi.linear, ctx, s["w_o"], s["b_o"] if lead else None, _capi.EPI_MC_RESIDUAL, None,
              row_mask, out_ptr=mc, out_ld=d)
            t("barrier", self._barrier, pads, 1)  # every rank's adds have landed in every copy
            t("layernorm", _capi.layernorm, resid, s["ln2_w"], s["ln2_b"], self.eps, ln)
            t("gemm_ffn_in", _capi.linear, ln, s["w_1"], s["b_1"], _capi.EPI_BIAS_GELU, hidden)
            t("barrier", self._barrier, pads, 2)
            t("gemm_ffn_out", _capi.linear, hidden, s["w_2"], s["b_2"] if lead else None,
              _capi.EPI_MC_RESIDUAL_ZERO, None, row_mask, out_ptr=mc, out_ld=d)
            t("barrier", self._barrier, pads, 3)
            if i == len(self.shards) - 1:
                t("layernorm", _capi.layernorm, resid, self.final_w, self.final_b, self.eps, out.view(tokens, d),
                  row_mask=row_mask)
            else:
                nxt = self.shards[i + 1]
                t("layernorm", _capi.layernorm, resid, nxt["ln1_w"], nxt["ln1_b"], self.eps, ln)
        return out

    def _forward_nccl(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
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

    def launches_per_forward(self, num_layers: int) -> int:
        """Kernels of this library per forward (NCCL's own kernels not counted)."""
        return 1 + (11 if self.collective == "multimem" else 7) * num_layers

    def close(self) -> None:
        """Drops the symmetric-memory residual (call on every rank before destroying the group)."""
        self._symm = None


def multicast_supported(device: torch.device) -> bool:
    """True when symmetric memory on `device` has an NVLink SHARP multicast address."""
    try:
        from torch._C._distributed_c10d import _SymmetricMemory
        from torch._C._autograd import DeviceType
    except ImportError:
        return False
    idx = torch.device(device).index or 0
    try:
        return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, idx))
    except RuntimeError:
        return False
