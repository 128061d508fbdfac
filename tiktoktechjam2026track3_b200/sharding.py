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

  - "rs" (default): the token rows are split over
    the ranks (rank r owns rows [r T/n, (r+1) T/n)). The out_proj / ffn_out GEMMs add each output
    row (plus the bias, on rank 0 only) into its owner's fp32 residual with system-scope atomics
    over NVLink (b2_linear_rs_fwd: a reduce-scatter inside the GEMM epilogue); each owner then
    LayerNorms only its rows and stores the bf16 result into every rank's LayerNorm buffer over
    NVLink (b2_layernorm_gather_fwd: the all-gather inside the LayerNorm). Per
    residual sub-block a GPU receives (n-1)/n of an fp32 [T, D] partial plus one bf16 [T, D] —
    the reduce-scatter / all-gather volume — and the LayerNorm work drops by n. Four cross-GPU
    flag barriers per layer (b2_peer_barrier) order readers against writers.
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


def rs_rows(tokens: int, world: int, rank: int) -> Tuple[int, int, int]:
    """Rows [r0, r1) a rank owns in the reduce-scatter plan, and rows per rank (the last rank may
    own fewer; row r belongs to rank min(r // rows_per_rank, world - 1))."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    per = max(1, -(-tokens // world))
    return min(tokens, rank * per), min(tokens, (rank + 1) * per), per


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


def _check_status(plan) -> None:
    """Raises if a kernel of an earlier call gave up waiting. A timed-out flag barrier can leave a
    signal set in a pad, so later barriers would pair up one step out of order: the plan drops its
    symmetric-memory buffers (pads included) and refuses to run until `reset()` has been called on
    every rank, which re-creates them zeroed behind a barrier of the process group."""
    if plan._failed:
        raise RuntimeError(f"{type(plan).__name__}: an earlier call timed out on the device (status "
                           f"{plan._failed:#x}); call reset() on every rank before the next forward")
    try:
        plan._status.check()
    except RuntimeError:
        plan._failed = plan._status.status or 1
        plan.close()
        raise


def _reset(plan) -> None:
    """Clears a failed plan on this rank (every rank calls it): waits for the device, clears the
    status word, drops the buffers and synchronises with the other ranks, so that the next call's
    rendezvous allocates fresh, zeroed flag pads on all of them."""
    import torch.distributed as dist

    torch.cuda.synchronize(plan.device)
    _capi.device_status(clear=True)
    plan.close()
    plan._failed = 0
    plan._status = _capi.StatusWatch()
    dist.barrier(group=plan.group)


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
            collective = "rs" if self.world > 1 else "nccl"
        if collective not in ("rs", "nccl"):
            raise ValueError(f"collective must be 'auto', 'rs' or 'nccl', not {collective!r}")
        self.collective = collective
        self._symm_rs: Optional[dict] = None
        self._status = _capi.StatusWatch()
        self._failed = 0

    reset = _reset

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

    def _barrier(self, pads: List[int], channel: int) -> None:
        _capi.peer_barrier(pads, self.rank, channel, self.device)

    def _rs_buffers(self, tokens: int, d: int) -> dict:
        """Symmetric memory for the "rs" plan: fp32 residual [T, D], bf16 LayerNorm output [T, D]
        and the barrier pads, in one allocation (rendezvous once per token count); only peer
        mappings are used (no multicast)."""
        if self._symm_rs is not None and self._symm_rs["tokens"] == tokens:
            return self._symm_rs
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self._symm_rs = None
        n_res = tokens * d  # fp32 words of the residual
        n_ln = (tokens * d + 1) // 2  # fp32 words holding the bf16 LayerNorm rows
        buf = symm_mem.empty(n_res + n_ln + 64, dtype=torch.float32, device=self.device)
        buf[n_res + n_ln:].zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(buf, group)
        bases = [int(p) for p in handle.buffer_ptrs]  # every rank's buffer, mapped over NVLink
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every pad is zero before any rank signals
        r0, r1, rows = rs_rows(tokens, self.world, self.rank)
        self._symm_rs = {
            "tokens": tokens, "buf": buf, "handle": handle,
            "resid": buf[:n_res].view(tokens, d),
            "ln": buf[n_res:n_res + n_ln].view(torch.bfloat16)[: tokens * d].view(tokens, d),
            "ln_ranks": [b + n_res * 4 for b in bases],
            "peer_resid": bases,
            "pads": [b + (n_res + n_ln) * 4 for b in bases],
            "rows_per_rank": rows, "r0": r0, "r1": r1,
        }
        return self._symm_rs

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_status(self)
        if self.collective == "rs":
            out = self._forward_rs(x, valid_token_mask)
        else:
            out = self._forward_nccl(x, valid_token_mask)
        self._status.after_forward(self.device)
        return out

    def _forward_rs(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
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
        sb = self._rs_buffers(tokens, d)
        resid, ln, peers, pads = sb["resid"], sb["ln"], sb["peer_resid"], sb["pads"]
        r0, r1, rpr = sb["r0"], sb["r1"], sb["rows_per_rank"]
        my_resid = resid[r0:r1]
        my_ln_rows = [base + r0 * d * 2 for base in sb["ln_ranks"]]
        my_mask = row_mask[r0:r1] if row_mask is not None else None
        qkv = torch.empty(tokens, 3 * d_loc, device=dev, dtype=torch.bfloat16)
        ctx = torch.empty(tokens, d_loc, device=dev, dtype=torch.bfloat16)
        hidden = torch.empty(tokens, f_loc, device=dev, dtype=torch.bfloat16)
        x2 = x.contiguous().view(tokens, d)
        lead = self.rank == 0  # adds the out_proj / ffn_out biases
        s0 = self.shards[0]
        t = self._timed
        ch = 0

        def barrier():
            nonlocal ch
            t("barrier", self._barrier, pads, ch)
            ch = (ch + 1) % 4

        # First LayerNorm on every rank for all rows (x is replicated): local, no exchange.
        t("layernorm", _capi.layernorm, x2, s0["ln1_w"], s0["ln1_b"], self.eps, ln, resid_out=resid)
        barrier()  # every owner's residual rows exist before any rank adds into them
        for i, s in enumerate(self.shards):
            t("gemm_qkv", _capi.linear, ln, s["w_qkv"], s["b_qkv"], _capi.EPI_BIAS, qkv)
            t("attention", _capi.attention, qkv, batch, seq_len, h_loc, hd, 0, d_loc, 2 * d_loc, kv_len, cfg.causal,
              hd**-0.5, ctx)
            t("gemm_out", _capi.linear_rs, ctx, s["w_o"], s["b_o"] if lead else None, False, peers, self.rank, rpr, d,
              row_mask)
            barrier()  # this rank's rows hold every rank's contribution
            if r1 > r0:
                t("layernorm", _capi.layernorm_gather, my_resid, s["ln2_w"], s["ln2_b"], self.eps, my_ln_rows)
            barrier()  # every rank's LayerNorm rows landed in every copy
            t("gemm_ffn_in", _capi.linear, ln, s["w_1"], s["b_1"], _capi.EPI_BIAS_GELU, hidden)
            t("gemm_ffn_out", _capi.linear_rs, hidden, s["w_2"], s["b_2"] if lead else None, True, peers, self.rank,
              rpr, d, row_mask)
            barrier()
            last = i == len(self.shards) - 1
            g, b = (self.final_w, self.final_b) if last else (self.shards[i + 1]["ln1_w"], self.shards[i + 1]["ln1_b"])
            if r1 > r0:
                t("layernorm", _capi.layernorm_gather, my_resid, g, b, self.eps, my_ln_rows, my_mask if last else None)
            barrier()
        out = ln.view(batch, seq_len, d).clone()
        self._mask_lengths.raise_if_invalid()
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
        self._mask_lengths.raise_if_invalid()
        return out

    __call__ = forward

    def launches_per_forward(self, num_layers: int) -> int:
        """Kernels of this library per forward (NCCL's own kernels not counted)."""
        if self.collective == "rs":
            return 2 + 11 * num_layers
        return 1 + 7 * num_layers

    def close(self) -> None:
        """Drops the symmetric-memory buffers (call on every rank before destroying the group)."""
        self._symm_rs = None


def cp_chunks(seq_len: int, world: int, rank: int) -> Tuple[int, Tuple[int, int]]:
    """Context-parallel split of a sequence into 2 * world chunks (zigzag): rank r owns chunks r and
    2 * world - 1 - r, so every rank gets one early and one late chunk and the causal work is
    balanced. Returns (chunk rows, (first chunk index, second chunk index))."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    if seq_len % (2 * world * 128):
        raise ValueError(f"seq_len={seq_len} must be a multiple of 2 x {world} ranks x 128 for context parallelism")
    return seq_len // (2 * world), (rank, 2 * world - 1 - rank)


class ContextParallelTransformer:
    """Forward pass of the stack with each sequence's tokens split over a process group (context
    parallelism, for single long sequences): every rank holds all weights and runs the LayerNorms
    and GEMMs on its own token rows, and the attention of its query rows against every key.
    The K/V exchange is fused into the QKV GEMM: its epilogue stores the K and V columns of the
    rank's rows into every rank's full-length QKV buffer over NVLink (b2_linear_bcast_fwd).

    Token rows of each sequence are split into 2n chunks, rank r owning chunks r and 2n-1-r (zigzag:
    equal causal work per rank). Per layer a rank computes Q/K/V for its rows into its full-length
    [B*S, 3D] QKV buffer (torch symmetric memory), K and V also into every other rank's buffer —
    the all-gather of K and V, (n-1)/n of 2 bf16 [T, D] per GPU per layer, no reduction anywhere —
    then runs `b2_attention_rows_fwd` over its two query chunks in one launch
    (the later, heavier chunk's tiles first). Alternate layers use two QKV copies, so one flag
    barrier per layer (b2_peer_barrier, after the QKV GEMM: every chunk has landed before attention
    reads it) also orders the writes of layer i against the reads of layer i - 2 (at 8 GPUs the
    per-layer barriers cost 0.87 ms per C4 step with two per layer). The output is gathered to every
    rank the same way. Built from the full model's state dict (reference key names).
    """

    def __init__(self, config, state: Dict[str, torch.Tensor], device: torch.device, group=None) -> None:
        import torch.distributed as dist

        from .models import UserOptimizedTransformer

        self.config = config_from(config)
        self.config.validate()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        with torch.inference_mode(False):  # ordinary parameters even when built under inference mode
            model = UserOptimizedTransformer(self.config)
            model.load_state_dict(state, strict=True)
            self.model = model.to(device=device, dtype=torch.bfloat16).eval()
        self.collective = "cp"
        self._mask_lengths = MaskLengths()
        self._launch_log: Optional[list] = None
        self._buf: Optional[dict] = None
        self._status = _capi.StatusWatch()
        self._failed = 0

    reset = _reset

    record_launches = TensorParallelTransformer.record_launches
    take_launch_log = TensorParallelTransformer.take_launch_log
    _timed = TensorParallelTransformer._timed

    def _buffers(self, batch: int, seq_len: int) -> dict:
        if self._buf is not None and self._buf["shape"] == (batch, seq_len):
            return self._buf
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self._buf = None
        d = self.config.d_model
        tokens = batch * seq_len
        # Two full-length QKV copies, used by alternate layers: a rank writes layer i's K/V into
        # copy i % 2 of every peer, which the peers last read for layer i - 2's attention — over
        # before they arrived at layer i - 1's barrier (each barrier kernel waits for its stream's
        # earlier kernels), so one barrier per layer orders every reader against every writer.
        n_qkv, n_out = tokens * 3 * d, tokens * d
        buf = symm_mem.empty(2 * n_qkv + n_out + 64, dtype=torch.bfloat16, device=self.device)
        buf[2 * n_qkv + n_out:].zero_()
        group = self.group if self.group is not None else dist.group.WORLD
        handle = symm_mem.rendezvous(buf, group)
        total = 2 * n_qkv + n_out + 64
        peers = [handle.get_buffer(r, (total,), torch.bfloat16) for r in range(self.world)]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every pad is zero before any rank signals
        chunk, mine = cp_chunks(seq_len, self.world, self.rank)
        pieces = [(b * seq_len + c * chunk, chunk) for b in range(batch) for c in mine]  # (first row, rows)
        self._buf = {
            "shape": (batch, seq_len), "buf": buf, "handle": handle, "chunk": chunk, "mine": mine,
            "pieces": pieces,
            # [copy][rank]: every rank's two QKV buffers
            "qkv": [[p[c * n_qkv:(c + 1) * n_qkv].view(tokens, 3 * d) for p in peers] for c in range(2)],
            "out": [p[2 * n_qkv:2 * n_qkv + n_out].view(tokens, d) for p in peers],
            "pads": [int(x) + (2 * n_qkv + n_out) * 2 for x in handle.buffer_ptrs],
            "ctx": torch.empty(tokens, d, device=self.device, dtype=torch.bfloat16),
        }
        return self._buf

    def _barrier(self, pads: List[int], channel: int) -> None:
        _capi.peer_barrier(pads, self.rank, channel, self.device)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_status(self)
        out = self._forward_cp(x, valid_token_mask)
        self._status.after_forward(self.device)
        return out

    def _forward_cp(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
        cfg = self.config
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("ContextParallelTransformer needs a bf16 CUDA input")
        batch, seq_len, d = x.shape
        if valid_token_mask is not None and valid_token_mask.device != x.device:
            raise ValueError("valid_token_mask must be on x's device")
        kv_len, row_mask = self._mask_lengths(valid_token_mask, batch, seq_len)
        sb = self._buffers(batch, seq_len)
        pieces, chunk, pads = sb["pieces"], sb["chunk"], sb["pads"]
        qkv_copies, out_all, ctx = sb["qkv"], sb["out"], sb["ctx"]
        h, hd = cfg.num_heads, cfg.head_dim
        t_loc = len(pieces) * chunk
        dev = x.device
        x2 = x.contiguous().view(batch * seq_len, d)
        x_loc = torch.cat([x2[r0:r0 + n] for r0, n in pieces], 0)
        mask_loc = torch.cat([row_mask[r0:r0 + n] for r0, n in pieces], 0) if row_mask is not None else None
        resid = torch.empty(t_loc, d, device=dev, dtype=torch.float32)
        ln = torch.empty(t_loc, d, device=dev, dtype=torch.bfloat16)
        hidden = torch.empty(t_loc, cfg.ffn_dim, device=dev, dtype=torch.bfloat16)
        out_loc = torch.empty(t_loc, d, device=dev, dtype=torch.bfloat16)
        packed = self.model.packed_weights()
        t = self._timed
        ch = 0

        def barrier():
            nonlocal ch
            t("barrier", self._barrier, pads, ch)
            ch = (ch + 1) % 4

        def local(buf, k):  # rows of piece k in a local [t_loc, *] buffer
            return buf[k * chunk:(k + 1) * chunk]

        def rows(buf, k):  # rows of piece k at their absolute positions in a [B*S, *] buffer
            r0, n = pieces[k]
            return buf[r0:r0 + n]

        def broadcast(bufs, src):  # this rank's pieces of src into every other rank's copy
            for r in range(self.world):
                if r != self.rank:
                    for k in range(len(pieces)):
                        rows(bufs[r], k).copy_(rows(src, k), non_blocking=True)

        pb0 = packed[0]
        t("layernorm", _capi.layernorm, x_loc, pb0.ln1_w, pb0.ln1_b, pb0.ln1_eps, ln, resid_out=resid)
        for i, pb in enumerate(packed):
            if i > 0:
                t("layernorm", _capi.layernorm, resid, pb.ln1_w, pb.ln1_b, pb.ln1_eps, ln)
            qkv_all = qkv_copies[i % 2]  # copy i % 2: its readers (layer i - 2) are done, see _buffers
            qkv = qkv_all[self.rank]
            for k in range(len(pieces)):  # K and V columns also stored into every peer's buffer
                row0 = pieces[k][0]
                t("gemm_qkv", _capi.linear_bcast, local(ln, k), pb.w_qkv, pb.b_qkv,
                  [q.data_ptr() + row0 * 3 * d * 2 for q in qkv_all], self.rank, d, 3 * d)
            barrier()  # every rank's rows have landed in every copy
            t("attention", _capi.attention, qkv, batch, seq_len, h, hd, 0, d, 2 * d, kv_len, cfg.causal, hd**-0.5,
              ctx, q_rows=[(c * chunk, chunk) for c in sb["mine"]])
            for k in range(len(pieces)):
                t("gemm_out", _capi.linear, rows(ctx, k), pb.w_o, pb.b_o, _capi.EPI_RESIDUAL, local(resid, k),
                  local(mask_loc, k) if mask_loc is not None else None)
            t("layernorm", _capi.layernorm, resid, pb.ln2_w, pb.ln2_b, pb.ln2_eps, ln)
            t("gemm_ffn_in", _capi.linear, ln, pb.w_1, pb.b_1, _capi.EPI_BIAS_GELU, hidden)
            t("gemm_ffn_out", _capi.linear, hidden, pb.w_2, pb.b_2, _capi.EPI_RESIDUAL_ZERO, resid, mask_loc)
        fn = self.model.final_norm
        t("layernorm", _capi.layernorm, resid, fn.weight, fn.bias, float(fn.eps), out_loc, row_mask=mask_loc)
        out_mine = out_all[self.rank]
        for k in range(len(pieces)):
            rows(out_mine, k).copy_(local(out_loc, k), non_blocking=True)
        barrier()  # peers are done with their previous output copies
        t("allgather", broadcast, out_all, out_mine)
        barrier()
        out = out_mine.view(batch, seq_len, d).clone()
        self._mask_lengths.raise_if_invalid()
        return out

    __call__ = forward

    def launches_per_forward(self, num_layers: int) -> int:
        """Kernels of this library per forward (copies not counted): per layer one QKV and one
        out_proj GEMM per piece (2 pieces per sequence), 1 attention launch, 1 barrier,
        LayerNorm x 2, ffn_in, ffn_out; then the final LayerNorm and 2 barriers."""
        p = 2 * self.config.batch_size
        return num_layers * (2 * p + 6) + 3

    def close(self) -> None:
        """Drops the symmetric-memory buffers (call on every rank before destroying the group)."""
        self._buf = None
