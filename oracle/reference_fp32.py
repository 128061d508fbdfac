"""fp32 restatement of the reference Transformer encoder forward pass — TEST INFRASTRUCTURE.

This module is the checker, never the product: only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm import it. The product path
(tiktoktechjam2026track3_b200) never calls it and has no CPU fallback.

It restates, in plain PyTorch fp32 ops, the computation of
  BaselineTransformer.forward            transformer_benchmark/models.py:909-919
  BaselineTransformerBlock.forward       transformer_benchmark/models.py:727-738
  BaselineSelfAttention.forward          transformer_benchmark/models.py:43-80
with the same parameter construction order (so torch.manual_seed(seed) yields the same weights
as the reference's `BaselineTransformer(config)` built after the runner's seeding,
transformer_benchmark/runner.py:316-321), and the reference's input generator
  generate_random_case                   transformer_benchmark/cases.py:60-98.

Pinned by tests/test_oracle_golden.py against golden vectors that tests/golden/make_golden.py
produced by importing and running the reference itself.

Attention is evaluated in query-row chunks (same math as materialising the [B, H, S, S] score
tensor, O(chunk * S) memory), so the same code checks long sequences; it runs on any torch
device (CPU for golden checks and the CPU baseline, CUDA in fp32 with TF32 disabled for the
full-size parity tests).
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def _config_fields(config) -> Tuple[int, int, int, int, int, int, bool]:
    return (
        int(config.batch_size),
        int(config.seq_len),
        int(config.d_model),
        int(config.num_heads),
        int(config.ffn_dim),
        int(config.num_layers),
        bool(config.causal),
    )


def build_reference_state(config, seed: int) -> Dict[str, torch.Tensor]:
    """Weights of BaselineTransformer(config) built right after torch.manual_seed(seed).

    Module construction order, and hence RNG consumption, follows
    BaselineTransformerBlock.__init__ (models.py:719-725: norm1, attention{q,k,v,out}_proj,
    norm2, ffn_in, ffn_out) per layer, then final_norm (models.py:907). nn.Linear and
    nn.LayerNorm are constructed exactly as the reference constructs them.
    """
    _, _, d_model, _, ffn_dim, num_layers, _ = _config_fields(config)
    torch.manual_seed(seed)
    state: Dict[str, torch.Tensor] = {}

    def put(prefix: str, module: nn.Module) -> None:
        for name, tensor in module.state_dict().items():
            state[f"{prefix}.{name}"] = tensor.detach().clone()

    for i in range(num_layers):
        p = f"layers.{i}"
        put(f"{p}.norm1", nn.LayerNorm(d_model))
        put(f"{p}.attention.q_proj", nn.Linear(d_model, d_model, bias=True))
        put(f"{p}.attention.k_proj", nn.Linear(d_model, d_model, bias=True))
        put(f"{p}.attention.v_proj", nn.Linear(d_model, d_model, bias=True))
        put(f"{p}.attention.out_proj", nn.Linear(d_model, d_model, bias=True))
        put(f"{p}.norm2", nn.LayerNorm(d_model))
        put(f"{p}.ffn_in", nn.Linear(d_model, ffn_dim))
        put(f"{p}.ffn_out", nn.Linear(ffn_dim, d_model))
    put("final_norm", nn.LayerNorm(d_model))
    return state


def round_state_to_bf16(state: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """The weights a bf16 model holds, widened back to fp32 (the GPU path's exact weights)."""
    return {k: v.to(torch.bfloat16).to(torch.float32) for k, v in state.items()}


def generate_random_case(
    config,
    device: torch.device,
    dtype: torch.dtype,
    seed: int,
    padding_ratio: float,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Restatement of transformer_benchmark/cases.py:60-98 (same generator calls, same order)."""
    batch, seq_len, d_model, *_ = _config_fields(config)
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    x = torch.randn(batch, seq_len, d_model, generator=generator, device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(batch, seq_len, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=seq_len + 1, size=(batch,), generator=generator, device=device)
    positions = torch.arange(seq_len, device=device)[None, :]
    mask = positions < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def _linear(x: torch.Tensor, state: Dict[str, torch.Tensor], prefix: str) -> torch.Tensor:
    return F.linear(x, state[f"{prefix}.weight"], state[f"{prefix}.bias"])


def _layer_norm(x: torch.Tensor, state: Dict[str, torch.Tensor], prefix: str, eps: float = 1e-5) -> torch.Tensor:
    d = x.shape[-1]
    return F.layer_norm(x, (d,), state[f"{prefix}.weight"], state[f"{prefix}.bias"], eps)


def attention_core(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    key_mask: Optional[torch.Tensor],
    causal: bool,
    scale: float,
    query_chunk: int = 1024,
) -> torch.Tensor:
    """softmax(mask(q k^T * scale)) v for q, k, v [B, H, S, hd] (models.py:55-71).

    key_mask [B, S] bool marks valid keys (models.py:63-66); causal hides keys after the query
    (models.py:57-61). Rows are processed `query_chunk` at a time.
    """
    batch, heads, seq_len, hd = q.shape
    out = torch.empty_like(q)
    key_pos = torch.arange(seq_len, device=q.device)
    for b in range(batch):
        kb = k[b]
        vb = v[b]
        for r0 in range(0, seq_len, query_chunk):
            r1 = min(seq_len, r0 + query_chunk)
            k_stop = r1 if causal else seq_len
            scores = torch.matmul(q[b, :, r0:r1], kb[:, :k_stop].transpose(-2, -1)) * scale
            if causal:
                q_pos = torch.arange(r0, r1, device=q.device)
                hidden = key_pos[None, :k_stop] > q_pos[:, None]
                scores = scores.masked_fill(hidden[None], float("-inf"))
            if key_mask is not None:
                scores = scores.masked_fill(~key_mask[b, None, None, :k_stop], float("-inf"))
            probs = torch.softmax(scores.float(), dim=-1).to(scores.dtype)  # fp32 softmax (models.py:69)
            out[b, :, r0:r1] = torch.matmul(probs, vb[:, :k_stop])
    return out


def self_attention(
    x: torch.Tensor,
    state: Dict[str, torch.Tensor],
    prefix: str,
    num_heads: int,
    key_mask: Optional[torch.Tensor],
    causal: bool,
    query_chunk: int = 1024,
) -> torch.Tensor:
    """BaselineSelfAttention.forward (models.py:43-80) in fp32."""
    batch, seq_len, d_model = x.shape
    hd = d_model // num_heads

    def split(t: torch.Tensor) -> torch.Tensor:
        return t.view(batch, seq_len, num_heads, hd).transpose(1, 2)

    q = split(_linear(x, state, f"{prefix}.q_proj"))
    k = split(_linear(x, state, f"{prefix}.k_proj"))
    v = split(_linear(x, state, f"{prefix}.v_proj"))
    ctx = attention_core(q, k, v, key_mask, causal, hd**-0.5, query_chunk)
    ctx = ctx.transpose(1, 2).reshape(batch, seq_len, d_model)
    out = _linear(ctx, state, f"{prefix}.out_proj")
    if key_mask is not None:
        out = out.masked_fill(~key_mask[..., None], 0)
    return out


def forward(
    state: Dict[str, torch.Tensor],
    config,
    x: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
    query_chunk: int = 1024,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """BaselineTransformer.forward (models.py:909-919) on x's device, in fp32 by default.

    With dtype=torch.bfloat16 (and a bf16 state) every op runs in bf16 with the softmax in fp32,
    as the reference's baseline module does on the GPU in the harness's bf16 mode.
    """
    _, _, _, num_heads, _, num_layers, causal = _config_fields(config)
    x = x.to(dtype)
    for i in range(num_layers):
        p = f"layers.{i}"
        x = x + self_attention(_layer_norm(x, state, f"{p}.norm1"), state, f"{p}.attention", num_heads,
                               valid_token_mask, causal, query_chunk)
        h = F.gelu(_linear(_layer_norm(x, state, f"{p}.norm2"), state, f"{p}.ffn_in"), approximate="none")
        x = x + _linear(h, state, f"{p}.ffn_out")
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
    x = _layer_norm(x, state, "final_norm")
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[..., None], 0)
    return x


def state_checksums(state: Dict[str, torch.Tensor]) -> Dict[str, Tuple[float, float]]:
    """(sum, sum of squares) in float64 per tensor, used to pin the weight construction."""
    out = {}
    for k, v in state.items():
        d = v.detach().to(torch.float64)
        out[k] = (float(d.sum()), float((d * d).sum()))
    return out


def flops_per_forward(config, lengths: Optional[torch.Tensor] = None) -> Dict[str, float]:
    """Algorithmic FLOPs of one forward pass (GEMMs; attention over useful query/key pairs).

    GEMMs: 8*T*D^2 + 4*T*D*F per layer. Attention: 4*D*pairs per layer, pairs = S(S+1)/2 per
    sequence when causal, len_b^2 with a padding mask (len_b(len_b+1)/2 if both), S^2 otherwise.
    """
    batch, seq_len, d_model, _, ffn_dim, num_layers, causal = _config_fields(config)
    tokens = batch * seq_len
    gemm = num_layers * (8.0 * tokens * d_model * d_model + 4.0 * tokens * d_model * ffn_dim)
    if lengths is None:
        lens = [seq_len] * batch
    else:
        lens = [int(v) for v in lengths.tolist()]
    if causal:
        pairs = sum(n * (n + 1) / 2.0 for n in lens)
    else:
        pairs = sum(float(n) * n for n in lens)
    attn = num_layers * 4.0 * d_model * pairs
    return {"gemm": gemm, "attention": attn, "total": gemm + attn}


def layernorm_bytes_per_forward(config, in_bytes: int = 4, out_bytes: int = 2) -> float:
    """(2L+1) LayerNorm calls, each reading and writing T*D elements."""
    batch, seq_len, d_model, _, _, num_layers, _ = _config_fields(config)
    return (2 * num_layers + 1) * batch * seq_len * d_model * float(in_bytes + out_bytes)


__all__ = [
    "attention_core",
    "build_reference_state",
    "flops_per_forward",
    "forward",
    "generate_random_case",
    "layernorm_bytes_per_forward",
    "round_state_to_bf16",
    "self_attention",
    "state_checksums",
]
