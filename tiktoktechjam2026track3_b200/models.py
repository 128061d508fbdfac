"""Drop-in `UserOptimizedTransformer` running the encoder stack on the sm_100a kernels.

Module contract, kept from the reference (transformer_benchmark/models.py:895-930,
runner.py:316-329, correctness.py:135-146, timing.py:76-96):
  * built as `UserOptimizedTransformer(config)` from a TransformerConfig;
  * the same parameter names as BaselineTransformer (`layers.{i}.norm1`, `.attention.{q,k,v,
    out}_proj`, `.norm2`, `.ffn_in`, `.ffn_out`, `final_norm`), constructed in the same order, so
    `copy_model_weights(baseline, optimized, strict=True)` and seeded construction both match;
  * moved with `.to(device="cuda", dtype=torch.bfloat16).eval()`;
  * called as `forward(x[B, S, D], valid_token_mask[B, S] bool | None) -> [B, S, D]` on the
    current CUDA stream; the returned tensor is freshly allocated (no aliasing across calls).

The forward pass runs entirely in libb200tx.so (through the C-ABI, see _capi.py); this module only
allocates buffers and sequences 7 kernel launches per block plus one final LayerNorm:
    LN1 -> QKV GEMM (+bias) -> flash attention -> out_proj GEMM (+bias, +residual, row mask)
        -> LN2 -> ffn_in GEMM (+bias, GELU) -> ffn_out GEMM (+bias, +residual, row zero)
The residual stream is kept in fp32 between kernels; LayerNorm reads fp32 and writes bf16, all
GEMM and attention operands are bf16 with fp32 accumulation.

Masks: the harness's masks are prefix masks (generate_random_case, cases.py:87-97); a prefix mask
becomes per-sequence key lengths plus a row mask (checked on the device, without a host round trip
before the kernels are enqueued), and any other mask raises.

There is no CPU or eager-PyTorch fallback: CPU tensors, other dtypes and unsupported head
dimensions raise.
"""

from __future__ import annotations

import copy
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from . import _capi
from .cases import TransformerConfig, config_from

# 32, 64 and 128 run on the tcgen05 attention kernels; 8, 16 and 256 (the reference's official
# case matrix) on the CUDA-core one.
SUPPORTED_HEAD_DIMS = (8, 16, 32, 64, 128, 256)


def attention_kernel_name(head_dim: int) -> str:
    """The attention kernel b2_attention_fwd launches for `head_dim` (its dispatch in b200tx.cu)."""
    if head_dim in (32, 64):
        return "attention_solo_kernel"
    if head_dim == 128:
        return "attention_wide_kernel"
    return "attention_simt_kernel"


class SelfAttention(nn.Module):
    """Parameter holder with BaselineSelfAttention's names (models.py:20-33)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)


class TransformerBlock(nn.Module):
    """Parameter holder with BaselineTransformerBlock's names and order (models.py:718-725)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = SelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


class _PackedBlock:
    __slots__ = ("ln1_w", "ln1_b", "ln1_eps", "w_qkv", "b_qkv", "w_o", "b_o", "ln2_w", "ln2_b", "ln2_eps",
                 "w_1", "b_1", "w_2", "b_2")


class MaskLengths:
    """Turns the harness's valid-token mask into what the kernels take, with a one-entry cache.

    Returns (None, None) for no mask, and (kv_len int32 [B], row_mask uint8 [B*S]) for a prefix
    mask (positions < length, the form generate_random_case produces, cases.py:87-97); any other
    mask is rejected with NotImplementedError. For a CUDA mask nothing is read back on the host
    while the forward pass is being enqueued: the prefix check runs on the device, its verdict
    lands in pinned memory, and `raise_if_invalid()` (called after the kernels are enqueued, before
    the output is returned) waits only for that check. An all-true CUDA mask therefore takes the
    masked kernels, which compute exactly what the unmasked ones do; a CPU mask is checked at once
    and an all-true one elided (as the reference candidate does, models.py:1137-1161).
    The result is reused while the same mask storage is passed with an unchanged version counter
    (inference tensors carry no version counter and are re-derived on every call). The cache entry
    holds the mask tensor itself, so its storage cannot be freed and handed to a different mask
    while the entry could still match it.
    """

    _MESSAGE = "valid_token_mask must mark a prefix of each sequence (the form generate_random_case produces)"

    def __init__(self) -> None:
        self._cache: Optional[tuple] = None
        self._flag: Optional[torch.Tensor] = None
        self._flag_rows = 0
        self._pending: Optional[torch.cuda.Event] = None

    def __call__(
        self, valid_token_mask: Optional[torch.Tensor], batch: int, seq_len: int
    ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        self._pending = None
        if valid_token_mask is None:
            return None, None
        m = valid_token_mask
        if m.dtype != torch.bool or tuple(m.shape) != (batch, seq_len):
            raise ValueError(f"valid_token_mask must be bool [{batch}, {seq_len}], got {m.dtype} {tuple(m.shape)}")
        versioned = not m.is_inference()
        key = None
        if versioned:
            key = (m.data_ptr(), m._version, tuple(m.shape), tuple(m.stride()), m.device)
            if self._cache is not None and self._cache[0] == key:
                return self._cache[2]
        if m.is_cuda:
            # One launch (b2_mask_lengths): per-sequence lengths and a per-row "not a prefix" byte,
            # copied into pinned memory behind it; the mask bytes themselves are the row mask.
            mc = m.contiguous()
            lengths = torch.empty(batch, dtype=torch.int32, device=m.device)
            verdict = torch.empty(batch, dtype=torch.uint8, device=m.device)
            _capi.mask_lengths(mc, lengths, verdict)
            if self._flag is None or self._flag.numel() < batch:
                self._flag = torch.zeros(batch, dtype=torch.uint8, pin_memory=True)
            self._flag[:batch].copy_(verdict, non_blocking=True)
            self._flag_rows = batch
            self._pending = torch.cuda.Event()
            self._pending.record(torch.cuda.current_stream(m.device))
            result: Tuple[Optional[torch.Tensor], Optional[torch.Tensor]] = (lengths, mc.view(-1).view(torch.uint8))
        else:
            lengths = m.sum(dim=1, dtype=torch.int32)
            positions = torch.arange(seq_len, device=m.device, dtype=torch.int32)
            prefix = positions[None, :] < lengths[:, None]
            if not torch.equal(m, prefix):
                raise NotImplementedError(self._MESSAGE)
            if bool((lengths == seq_len).all()):
                result = (None, None)
            else:
                result = (lengths.contiguous(), m.reshape(-1).contiguous().view(torch.uint8))
        if versioned:
            self._cache = (key, m, result)
        return result

    def raise_if_invalid(self) -> None:
        """Waits for the pending device-side prefix check (if any) and raises if it failed."""
        ev, self._pending = self._pending, None
        if ev is None:
            return
        ev.synchronize()
        if bool(self._flag[: self._flag_rows].any()):
            self._cache = None
            raise NotImplementedError(self._MESSAGE)


class UserOptimizedTransformer(nn.Module):
    """Transformer encoder stack forward on B200 tensor cores (drop-in for the reference slot)."""

    def __init__(self, config) -> None:
        super().__init__()
        config = config_from(config)
        config.validate()
        self.config = config
        self.layers = nn.ModuleList(
            [TransformerBlock(config.d_model, config.num_heads, config.ffn_dim) for _ in range(config.num_layers)]
        )
        self.final_norm = nn.LayerNorm(config.d_model)
        self._packed: Optional[List[_PackedBlock]] = None
        self._packed_key: Optional[tuple] = None
        self._mask_lengths = MaskLengths()
        self._status = _capi.StatusWatch()
        self._launch_log: Optional[list] = None
        # CUDA-graph replay of the per-block launches (launch amortisation only: the graph holds
        # exactly the kernels the eager path launches). Keyed by shape, device and mask presence.
        self.use_cuda_graph = True
        self._graphs: Dict[tuple, "_GraphedStack"] = {}
        # LayerNorm fused into the residual GEMMs (b2_linear_ln_fwd): "auto" where the library
        # recommends it for d_model (nowhere in this build: the fused launch measured slower than
        # GEMM + LayerNorm on B200), True / False to force it on (where d_model has a plan) or off.
        # The choice depends on the model's widths only, never on the token count, so a batch shard
        # computes its rows exactly as the full batch does.
        self.fuse_layernorm = "auto"
        self._fused_cache: Dict[tuple, bool] = {}

    # ------------------------------------------------------------------ weights
    def _weights_key(self) -> tuple:
        """Storage address and version of every parameter, read through the fixed module structure
        (the modules' own dicts): the generic parameters() walk cost ~280 us of host time per
        forward at 12 layers, time during which the GPU sits idle before the first launch."""
        key = []
        try:
            for layer in self.layers:
                lm = layer._modules
                am = lm["attention"]._modules
                for mod in (lm["norm1"], am["q_proj"], am["k_proj"], am["v_proj"], am["out_proj"], lm["norm2"],
                            lm["ffn_in"], lm["ffn_out"]):
                    ps = mod._parameters
                    w, b = ps["weight"], ps["bias"]
                    key.append((w.data_ptr(), w._version))
                    key.append((b.data_ptr(), b._version))
            fp = self.final_norm._parameters
            key.append((fp["weight"].data_ptr(), fp["weight"]._version))
            key.append((fp["bias"].data_ptr(), fp["bias"]._version))
        except RuntimeError:  # inference tensors have no version counter
            return None
        return tuple(key)

    def _storage_key(self) -> tuple:
        return tuple(p.data_ptr() for p in self.parameters())

    def packed_weights(self) -> List[_PackedBlock]:
        """Per-block bf16 weights, with q/k/v packed into one [3D, D] projection (cached).

        The packing mirrors the reference candidate's qkv_proj (models.py:96, 105-158): rows
        [0, D) are q_proj, [D, 2D) k_proj, [2D, 3D) v_proj. Rebuilt when any parameter changes.
        """
        key = self._weights_key()
        if key is None:
            # Parameters created under torch.inference_mode carry no version counter, so an
            # in-place update cannot be seen: the packed q/k/v copies (the only weights held as
            # copies; every other packed tensor is the parameter itself) are refreshed in place on
            # every call, which keeps captured graphs valid, and storage changes repack.
            skey = ("storage",) + self._storage_key()
            if self._packed is not None and self._packed_key == skey:
                self._refresh_qkv_copies()
                return self._packed
            key = skey
        if self._packed is not None and self._packed_key == key:
            return self._packed
        self._graphs.clear()  # graphs replay the packed tensors they were captured with
        packed = []
        with torch.no_grad():
            for layer in self.layers:
                att = layer.attention
                pb = _PackedBlock()
                pb.ln1_w, pb.ln1_b, pb.ln1_eps = layer.norm1.weight, layer.norm1.bias, float(layer.norm1.eps)
                pb.w_qkv = torch.cat([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight], 0).contiguous()
                pb.b_qkv = torch.cat([att.q_proj.bias, att.k_proj.bias, att.v_proj.bias], 0).contiguous()
                pb.w_o, pb.b_o = att.out_proj.weight.contiguous(), att.out_proj.bias.contiguous()
                pb.ln2_w, pb.ln2_b, pb.ln2_eps = layer.norm2.weight, layer.norm2.bias, float(layer.norm2.eps)
                pb.w_1, pb.b_1 = layer.ffn_in.weight.contiguous(), layer.ffn_in.bias.contiguous()
                pb.w_2, pb.b_2 = layer.ffn_out.weight.contiguous(), layer.ffn_out.bias.contiguous()
                packed.append(pb)
        self._packed = packed
        self._packed_key = key
        return packed

    def _refresh_qkv_copies(self) -> None:
        with torch.no_grad():
            for layer, pb in zip(self.layers, self._packed):
                att = layer.attention
                d = att.d_model
                for i, lin in enumerate((att.q_proj, att.k_proj, att.v_proj)):
                    pb.w_qkv[i * d:(i + 1) * d].copy_(lin.weight)
                    pb.b_qkv[i * d:(i + 1) * d].copy_(lin.bias)

    # ------------------------------------------------------------------ masks
    def mask_to_lengths(
        self, valid_token_mask: Optional[torch.Tensor], batch: int, seq_len: int
    ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """(kv_len int32 [B] or None, row_mask uint8 [B*S] or None); see MaskLengths."""
        return self._mask_lengths(valid_token_mask, batch, seq_len)

    # ------------------------------------------------------------------ launch timing hook
    def record_launches(self, enabled: bool) -> None:
        """When enabled, every kernel launch is bracketed by CUDA events (for kernel roofline)."""
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

    def layernorm_fused(self, tokens: int) -> bool:
        """Whether a forward over `tokens` rows runs norm2 and the next block's norm1 inside the
        out_proj / ffn_out GEMMs (b2_linear_ln_fwd) instead of as LayerNorm launches. Depends on
        d_model and the mode only (tokens > 0 just needs a valid plan query)."""
        mode = self.fuse_layernorm
        if mode is False or tokens <= 0:
            return False
        hit = self._fused_cache.get(mode)
        if hit is None:
            cfg = self.config
            plans = [_capi.linear_ln_plan(1, cfg.d_model, cfg.d_model, sm_count=1),
                     _capi.linear_ln_plan(1, cfg.d_model, cfg.ffn_dim, sm_count=1)]
            if any(p is None for p in plans):
                hit = False
            else:
                hit = True if mode is True else all(p[2] for p in plans)
            self._fused_cache[mode] = hit
        return hit

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        cfg: TransformerConfig = self.config
        if x.dim() != 3 or x.shape[-1] != cfg.d_model:
            raise ValueError(f"x must be [B, S, {cfg.d_model}], got {tuple(x.shape)}")
        if not x.is_cuda:
            raise RuntimeError("UserOptimizedTransformer runs on CUDA (sm_100a) only; x is on the CPU")
        if x.dtype != torch.bfloat16:
            raise RuntimeError(f"UserOptimizedTransformer computes in bfloat16; got x.dtype={x.dtype}")
        if cfg.head_dim not in SUPPORTED_HEAD_DIMS:
            raise NotImplementedError(f"head_dim {cfg.head_dim} is not supported {SUPPORTED_HEAD_DIMS}")
        batch, seq_len, d_model = x.shape
        if valid_token_mask is not None and valid_token_mask.device != x.device:
            raise ValueError("valid_token_mask must be on x's device")
        # Launch first, check the weights after: comparing every parameter's storage and version
        # with the packed copies costs host time that would otherwise leave the GPU idle before the
        # first kernel. The launches use the packed weights of the previous call (memory they keep
        # alive, on x's device); if the parameters changed since then, the weights are repacked and
        # the pass runs again, and the stale result is never returned.
        # A kernel of an earlier call that gave up waiting (status word, read without a sync).
        self._status.check()
        packed = self._packed
        speculative = (packed is not None and packed[0].w_qkv.device == x.device
                       and packed[0].w_qkv.dtype == torch.bfloat16 and self._packed_key is not None
                       and self._packed_key[0] != "storage")
        if not speculative:
            packed = self._checked_packed(x.device)
        kv_len, row_mask = self.mask_to_lengths(valid_token_mask, batch, seq_len)
        xc = x.contiguous()
        out = self._forward_tokens(xc, batch, seq_len, kv_len, row_mask, packed)
        if speculative and self._weights_key() != self._packed_key:
            packed = self._checked_packed(x.device)
            out = self._forward_tokens(xc, batch, seq_len, kv_len, row_mask, packed)
        self._status.after_forward(x.device)
        self._mask_lengths.raise_if_invalid()
        return out

    def check_device_status(self) -> None:
        """Waits for the last forward pass and raises RuntimeError if any of its kernels (or an
        earlier one) gave up waiting; forward() itself reports this, without waiting, at the
        latest on the call after the one that timed out."""
        self._status.check(wait=True)

    def _checked_packed(self, device: torch.device) -> List[_PackedBlock]:
        packed = self.packed_weights()
        if packed[0].w_qkv.device != device or packed[0].w_qkv.dtype != torch.bfloat16:
            raise RuntimeError("model weights must be bfloat16 on x's device: call .to(device, torch.bfloat16)")
        return packed

    def _forward_tokens(
        self,
        x: torch.Tensor,
        batch: int,
        seq_len: int,
        kv_len: Optional[torch.Tensor],
        row_mask: Optional[torch.Tensor],
        packed: List[_PackedBlock],
    ) -> torch.Tensor:
        cfg = self.config
        tokens, d = batch * seq_len, cfg.d_model
        out = torch.empty(batch, seq_len, d, device=x.device, dtype=torch.bfloat16)
        fused = self.layernorm_fused(tokens)
        if self.use_cuda_graph and self._launch_log is None:
            shape_key = (batch, seq_len, x.device, kv_len is not None, fused)
            stack = self._graphs.get(shape_key)
            if stack is None or stack.packed is not packed:  # new shape, or weights changed: (re)capture
                self._graphs.pop(shape_key, None)
                stack = _GraphedStack(self, batch, seq_len, x.device, kv_len is not None, packed, fused)
                self._graphs[shape_key] = stack
            stack.run(x.view(tokens, d), kv_len, row_mask, out.view(tokens, d))
            return out
        ws = _Workspace(cfg, batch, seq_len, x.device)
        pb0 = packed[0]
        self._timed("layernorm", _capi.layernorm, x.view(tokens, d), pb0.ln1_w, pb0.ln1_b, pb0.ln1_eps, ws.ln,
                    resid_out=ws.resid)
        self._blocks(ws, batch, seq_len, kv_len, row_mask, packed, fused)
        fn = self.final_norm
        self._timed("layernorm", _capi.layernorm, ws.resid, fn.weight, fn.bias, float(fn.eps), out.view(tokens, d),
                    row_mask=row_mask)
        return out

    def _blocks(self, ws: "_Workspace", batch: int, seq_len: int, kv_len, row_mask, packed, fused: bool) -> None:
        """Every launch between the first LayerNorm (done) and the final LayerNorm.

        With `fused`, norm2 runs in out_proj's epilogue and the next block's norm1 in ffn_out's
        (b2_linear_ln_fwd); the last block's ffn_out is the plain residual GEMM.
        """
        cfg = self.config
        d, h, hd = cfg.d_model, cfg.num_heads, cfg.head_dim
        scale = hd**-0.5
        t = self._timed
        for i, pb in enumerate(packed):
            if i > 0 and not fused:
                t("layernorm", _capi.layernorm, ws.resid, pb.ln1_w, pb.ln1_b, pb.ln1_eps, ws.ln)
            t("gemm_qkv", _capi.linear, ws.ln, pb.w_qkv, pb.b_qkv, _capi.EPI_BIAS, ws.qkv)
            t("attention", _capi.attention, ws.qkv, batch, seq_len, h, hd, 0, d, 2 * d, kv_len, cfg.causal, scale,
              ws.ctx)
            if fused:
                t("gemm_out", _capi.linear_ln, ws.ctx, pb.w_o, pb.b_o, ws.resid, pb.ln2_w, pb.ln2_b, pb.ln2_eps, ws.ln,
                  False, row_mask)
            else:
                t("gemm_out", _capi.linear, ws.ctx, pb.w_o, pb.b_o, _capi.EPI_RESIDUAL, ws.resid, row_mask)
                t("layernorm", _capi.layernorm, ws.resid, pb.ln2_w, pb.ln2_b, pb.ln2_eps, ws.ln)
            t("gemm_ffn_in", _capi.linear, ws.ln, pb.w_1, pb.b_1, _capi.EPI_BIAS_GELU, ws.hidden)
            if fused and i + 1 < len(packed):
                nxt = packed[i + 1]
                t("gemm_ffn_out", _capi.linear_ln, ws.hidden, pb.w_2, pb.b_2, ws.resid, nxt.ln1_w, nxt.ln1_b,
                  nxt.ln1_eps, ws.ln, True, row_mask)
            else:
                t("gemm_ffn_out", _capi.linear, ws.hidden, pb.w_2, pb.b_2, _capi.EPI_RESIDUAL_ZERO, ws.resid, row_mask)

    def release_graphs(self) -> None:
        """Drops captured CUDA graphs and their static buffers."""
        self._graphs.clear()

    @staticmethod
    def launches_per_forward(num_layers: int, fused: bool = False) -> int:
        return 5 * num_layers + 2 if fused else 7 * num_layers + 1


class _Workspace:
    """Activation buffers of one forward pass (token-major, T = B*S rows)."""

    def __init__(self, cfg: TransformerConfig, batch: int, seq_len: int, device: torch.device) -> None:
        tokens, d, f = batch * seq_len, cfg.d_model, cfg.ffn_dim
        self.resid = torch.empty(tokens, d, device=device, dtype=torch.float32)
        self.ln = torch.empty(tokens, d, device=device, dtype=torch.bfloat16)
        self.qkv = torch.empty(tokens, 3 * d, device=device, dtype=torch.bfloat16)
        self.ctx = torch.empty(tokens, d, device=device, dtype=torch.bfloat16)
        self.hidden = torch.empty(tokens, f, device=device, dtype=torch.bfloat16)


class _GraphedStack:
    """A CUDA graph of UserOptimizedTransformer._blocks over static buffers.

    Per call: the mask-derived lengths/row mask are copied into static tensors, the first
    LayerNorm reads the caller's x directly into the static buffers, the graph replays every
    launch of the blocks, and the final LayerNorm writes the caller's fresh output tensor.
    """

    def __init__(self, model: "UserOptimizedTransformer", batch: int, seq_len: int, device: torch.device,
                 masked: bool, packed: List[_PackedBlock], fused: bool) -> None:
        self.model = model
        self.packed = packed
        self.ws = _Workspace(model.config, batch, seq_len, device)
        self._src = (None, None)  # the mask tensors last copied into kv_len / row_mask
        self.kv_len = torch.zeros(batch, device=device, dtype=torch.int32) if masked else None
        self.row_mask = torch.zeros(batch * seq_len, device=device, dtype=torch.uint8) if masked else None
        self.ws.resid.zero_()
        self.ws.ln.zero_()
        if masked:
            self.kv_len.fill_(seq_len)
            self.row_mask.fill_(1)
        # One eager pass (first use of each kernel sets its attributes outside capture), then capture.
        model._blocks(self.ws, batch, seq_len, self.kv_len, self.row_mask, packed, fused)
        torch.cuda.current_stream(device).synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            model._blocks(self.ws, batch, seq_len, self.kv_len, self.row_mask, packed, fused)

    def run(self, x2: torch.Tensor, kv_len, row_mask, out2: torch.Tensor) -> None:
        if self.kv_len is not None and (kv_len is not self._src[0] or row_mask is not self._src[1]):
            # The mask cache hands back the same tensors only for an unchanged mask (same storage
            # and version), so their copies are already in the static buffers.
            self.kv_len.copy_(kv_len)
            self.row_mask.copy_(row_mask)
            self._src = (kv_len, row_mask)
        pb0 = self.packed[0]
        _capi.layernorm(x2, pb0.ln1_w, pb0.ln1_b, pb0.ln1_eps, self.ws.ln, resid_out=self.ws.resid)
        self.graph.replay()
        fn = self.model.final_norm
        _capi.layernorm(self.ws.resid, fn.weight, fn.bias, float(fn.eps), out2, row_mask=self.row_mask)


def copy_model_weights(baseline: nn.Module, optimized: nn.Module, strict: bool = True) -> None:
    """Same contract as the reference's copy_model_weights (models.py:1242-1255)."""
    state_dict = copy.deepcopy(baseline.state_dict())
    incompatible = optimized.load_state_dict(state_dict, strict=strict)
    if not strict:
        if incompatible.missing_keys:
            print(f"[warning] missing optimized keys: {incompatible.missing_keys}")
        if incompatible.unexpected_keys:
            print(f"[warning] unexpected optimized keys: {incompatible.unexpected_keys}")


def load_reference_state(model: nn.Module, state: Dict[str, torch.Tensor]) -> None:
    """Loads a state dict with the reference's key names (strict)."""
    model.load_state_dict(state, strict=True)
