"""ctypes binding of libb200tx.so (C-ABI declared in include/b200tx.h).

Follows the reference's binding conventions: the library is loaded lazily, once, under a
lock (transformer_benchmark/native_softmax_bf16.py:16-17, 129-160), every foreign function has
explicit argtypes/restype, and a non-zero status becomes a RuntimeError carrying the library's
own message (transformer_benchmark/cublaslt_linear.py:63-145).

There is no fallback: if the library is missing or the device is not an sm_100 GPU, the call
raises. The wrappers here take torch tensors only to read their pointers, shapes and the current
CUDA stream; all arithmetic happens in the CUDA kernels.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Optional, Tuple

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libb200tx.so"

EPI_BIAS = 0
EPI_BIAS_GELU = 1
EPI_RESIDUAL = 2
EPI_RESIDUAL_ZERO = 3
EPI_STORE_F32 = 4
TILE_PAIR = 0x10000

# Every symbol include/b200tx.h declares, with its ctypes signature.
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
SIGNATURES = {
    "b2_abi_version": (ctypes.c_int, []),
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "b2_device_status_async": (ctypes.c_int, [_vp, _vp]),
    "b2_set_wait_limit": (ctypes.c_int, [ctypes.c_uint64]),
    "b2_mask_lengths": (ctypes.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "b2_test_set_fault": (ctypes.c_int, [ctypes.c_int]),
    "b2_layernorm_fwd": (
        ctypes.c_int,
        [_vp, ctypes.c_int, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _i64, _i64, _vp],
    ),
    "b2_add_layernorm_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_float, _vp, _i64, _i64, _vp],
    ),
    "b2_linear_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_int, _vp, _i64, _vp, ctypes.c_int, _vp],
    ),
    "b2_linear_ln_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp],
    ),
    "b2_linear_ln_plan": (
        ctypes.c_int,
        [_i64, _i64, _i64, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
         ctypes.POINTER(ctypes.c_int)],
    ),
    "b2_attention_fwd": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, ctypes.c_int, ctypes.c_float, _vp, _i64, _vp],
    ),
    "b2_attention_rows_fwd": (
        ctypes.c_int,
        [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, ctypes.c_int, ctypes.c_float, ctypes.POINTER(_i64),
         ctypes.c_int, _vp, _i64, _vp],
    ),
    "b2_peer_barrier": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    "b2_linear_rs_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_int, ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int, _i64, _i64,
         _vp, ctypes.c_int, _vp],
    ),
    "b2_linear_bcast_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _i64, _i64, _i64, ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int, _i64, _i64, ctypes.c_int,
         _vp],
    ),
    "b2_layernorm_gather_fwd": (
        ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, ctypes.POINTER(_vp), ctypes.c_int, _vp, _i64, _i64, _vp],
    ),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load_library() -> ctypes.CDLL:
    """Loads libb200tx.so once and binds every entry point; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m tiktoktechjam2026track3_b200.build` "
                "(this package has no CPU or PyTorch fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.b2_abi_version()
        if version != 1:
            raise RuntimeError(f"libb200tx.so ABI version {version}, expected 1")
        _lib = lib
        return lib


def _check(status: int, what: str) -> None:
    if status != 0:
        message = load_library().b2_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed with status {status}: {message}")


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this package has no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def device_status(clear: bool = True) -> int:
    """Pipeline status word of the current device (0 = no kernel gave up waiting)."""
    lib = load_library()
    out = ctypes.c_uint32(0)
    _check(lib.b2_device_status(ctypes.byref(out), 1 if clear else 0), "b2_device_status")
    return int(out.value)


def mask_lengths(mask: torch.Tensor, kv_len: torch.Tensor, not_prefix: torch.Tensor,
                 row_mask_out: Optional[torch.Tensor] = None) -> None:
    """kv_len[b] = valid keys of row b, not_prefix[b] = 1 where row b is not a prefix (see
    b2_mask_lengths); mask is a contiguous bool [B, S] CUDA tensor."""
    if mask.dtype != torch.bool or mask.dim() != 2:
        raise ValueError("mask must be bool [batch, seq_len]")
    _require(mask, torch.bool, "mask")
    _require(kv_len, torch.int32, "kv_len")
    _require(not_prefix, torch.uint8, "not_prefix")
    batch, seq_len = mask.shape
    if kv_len.numel() < batch or not_prefix.numel() < batch:
        raise ValueError("kv_len and not_prefix need one entry per sequence")
    if row_mask_out is not None:
        _require(row_mask_out, torch.uint8, "row_mask_out")
    _check(load_library().b2_mask_lengths(_ptr(mask), batch, seq_len, _ptr(kv_len), _ptr(row_mask_out),
                                          _ptr(not_prefix), _stream_ptr(mask.device)), "b2_mask_lengths")


def set_wait_limit(limit_ns: int = 0) -> None:
    """Limit of one pipeline wait on the current device in ns (0 = the default 4 s)."""
    _check(load_library().b2_set_wait_limit(int(limit_ns)), "b2_set_wait_limit")


def test_set_fault(fault: int) -> None:
    """Test-only fault selector (see b2_test_set_fault); 0 turns it off."""
    _check(load_library().b2_test_set_fault(int(fault)), "b2_test_set_fault")


class StatusWatch:
    """Checks every forward pass for a kernel pipeline timeout without synchronising.

    `after_forward()` enqueues a copy of the device's status word into pinned host memory behind
    the pass's kernels (b2_device_status_async) and records an event; `check()` reads the copy of
    an earlier pass once its event has completed (never waiting for it unless `wait=True`) and
    raises RuntimeError if a kernel gave up waiting, so a timed-out pass is reported at the latest
    by the next call. The status word is sticky until cleared (b2_device_status(clear=1)), so a
    timeout is never missed, only reported one call late when its copy has not landed yet.
    """

    def __init__(self) -> None:
        self._host: Optional[torch.Tensor] = None
        self._event: Optional[torch.cuda.Event] = None
        self.status = 0

    def check(self, wait: bool = False) -> int:
        ev = self._event
        if ev is None:
            return 0
        if not wait and not ev.query():
            return 0
        ev.synchronize()
        self._event = None
        value = int(self._host[0].item())
        if value:
            self.status = value
            kernel, site, reason = value >> 16, (value >> 8) & 0xFF, value & 0xFF
            names = {1: "layernorm", 2: "linear", 3: "attention", 4: "peer barrier"}
            raise RuntimeError(
                f"a {names.get(kernel, kernel)} kernel gave up waiting (status {value:#x}: site {site}, reason "
                f"{reason}); outputs computed since then are not valid. Clear the status with "
                "_capi.device_status(clear=True) after handling it")
        return 0

    def after_forward(self, device: torch.device) -> None:
        if self._host is None:
            self._host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        if self._event is not None and not self._event.query():
            return  # the previous copy is still in flight: it will report the same sticky word
        self._event = None
        lib = load_library()
        _check(lib.b2_device_status_async(self._host.data_ptr(), _stream_ptr(device)), "b2_device_status_async")
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        self._event = ev


def layernorm(
    x: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    y: torch.Tensor,
    resid_out: Optional[torch.Tensor] = None,
    row_mask: Optional[torch.Tensor] = None,
) -> None:
    """y = LayerNorm(x) in bf16 (see b2_layernorm_fwd)."""
    d_model = x.shape[-1]
    rows = x.numel() // d_model
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("x must be float32 or bfloat16")
    _require(x, x.dtype, "x")
    _require(gamma, torch.bfloat16, "gamma")
    _require(beta, torch.bfloat16, "beta")
    _require(y, torch.bfloat16, "y")
    if y.numel() != x.numel():
        raise ValueError("y must have x's shape")
    if resid_out is not None:
        _require(resid_out, torch.float32, "resid_out")
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    status = load_library().b2_layernorm_fwd(
        _ptr(x), 1 if x.dtype == torch.bfloat16 else 0, _ptr(gamma), _ptr(beta), float(eps), _ptr(y),
        _ptr(resid_out), _ptr(row_mask), rows, d_model, _stream_ptr(x.device),
    )
    _check(status, "b2_layernorm_fwd")


ADD_LN_ZERO_ROWS = 1
ADD_LN_ZERO_Y = 2


def add_layernorm(
    resid: torch.Tensor,
    delta: torch.Tensor,
    bias: Optional[torch.Tensor],
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    y: torch.Tensor,
    row_mask: Optional[torch.Tensor] = None,
    flags: int = 0,
) -> None:
    """resid = mask ? resid + delta + bias : (resid | 0); y = LayerNorm(resid) (b2_add_layernorm_fwd)."""
    d_model = resid.shape[-1]
    rows = resid.numel() // d_model
    _require(resid, torch.float32, "resid")
    _require(delta, torch.float32, "delta")
    _require(gamma, torch.bfloat16, "gamma")
    _require(beta, torch.bfloat16, "beta")
    _require(y, torch.bfloat16, "y")
    if delta.numel() != resid.numel() or y.numel() != resid.numel():
        raise ValueError("resid, delta and y must have the same number of elements")
    if bias is not None:
        _require(bias, torch.bfloat16, "bias")
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    status = load_library().b2_add_layernorm_fwd(
        _ptr(resid), _ptr(delta), _ptr(bias), _ptr(row_mask), int(flags), _ptr(gamma), _ptr(beta), float(eps),
        _ptr(y), rows, d_model, _stream_ptr(resid.device),
    )
    _check(status, "b2_add_layernorm_fwd")


def linear(
    a: torch.Tensor,
    w: torch.Tensor,
    bias: Optional[torch.Tensor],
    epilogue: int,
    out: torch.Tensor,
    row_mask: Optional[torch.Tensor] = None,
    tile_n: int = 0,
) -> None:
    """out = epilogue(a @ w.T + bias) (see b2_linear_fwd)."""
    _require(a, torch.bfloat16, "a")
    _require(w, torch.bfloat16, "w")
    m, k = a.shape[0] if a.dim() == 2 else a.numel() // a.shape[-1], a.shape[-1]
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"w has shape {tuple(w.shape)}, expected [n, {k}]")
    if bias is not None:
        _require(bias, torch.bfloat16, "bias")
    out_dtype = torch.bfloat16 if epilogue in (EPI_BIAS, EPI_BIAS_GELU) else torch.float32
    _require(out, out_dtype, "out")
    if out.numel() < m * n:
        raise ValueError("out is too small")
    dst, ldo = out.data_ptr(), out.shape[-1]
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    status = load_library().b2_linear_fwd(
        _ptr(a), _ptr(w), _ptr(bias), m, n, k, int(epilogue), dst, ldo, _ptr(row_mask), int(tile_n),
        _stream_ptr(a.device),
    )
    _check(status, "b2_linear_fwd")


def linear_ln_plan(m: int, n: int, k: int, sm_count: int = 0) -> Optional[Tuple[int, int, bool]]:
    """(tile_n, cluster, recommended) of b2_linear_ln_fwd for an m x n x k problem, or None when n
    has no fused plan (see b2_linear_ln_plan). sm_count 0 asks the current device."""
    lib = load_library()
    tile, cluster, rec = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    status = lib.b2_linear_ln_plan(int(m), int(n), int(k), int(sm_count), ctypes.byref(tile), ctypes.byref(cluster),
                                   ctypes.byref(rec))
    if status == 2:
        return None
    _check(status, "b2_linear_ln_plan")
    return int(tile.value), int(cluster.value), bool(rec.value)


def linear_ln(
    a: torch.Tensor,
    w: torch.Tensor,
    bias: Optional[torch.Tensor],
    resid: torch.Tensor,
    gamma: torch.Tensor,
    beta: torch.Tensor,
    eps: float,
    ln_out: torch.Tensor,
    zero_masked_rows: bool,
    row_mask: Optional[torch.Tensor] = None,
) -> None:
    """resid = mask ? resid + a @ w.T + bias : (0 | resid); ln_out = LayerNorm(resid) (b2_linear_ln_fwd)."""
    _require(a, torch.bfloat16, "a")
    _require(w, torch.bfloat16, "w")
    _require(resid, torch.float32, "resid")
    _require(gamma, torch.bfloat16, "gamma")
    _require(beta, torch.bfloat16, "beta")
    _require(ln_out, torch.bfloat16, "ln_out")
    k = a.shape[-1]
    m = a.numel() // k
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"w has shape {tuple(w.shape)}, expected [n, {k}]")
    if resid.numel() != m * n or ln_out.numel() != m * n or resid.shape[-1] != n:
        raise ValueError(f"resid and ln_out must be [{m}, {n}]")
    if bias is not None:
        _require(bias, torch.bfloat16, "bias")
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    status = load_library().b2_linear_ln_fwd(
        _ptr(a), _ptr(w), _ptr(bias), m, n, k, 1 if zero_masked_rows else 0, _ptr(resid), _ptr(row_mask), _ptr(gamma),
        _ptr(beta), float(eps), _ptr(ln_out), _stream_ptr(a.device),
    )
    _check(status, "b2_linear_ln_fwd")


def attention(
    qkv: torch.Tensor,
    batch: int,
    seq_len: int,
    num_heads: int,
    head_dim: int,
    q_col: int,
    k_col: int,
    v_col: int,
    kv_len: Optional[torch.Tensor],
    causal: bool,
    scale: float,
    ctx: torch.Tensor,
    q_rows=None,
) -> None:
    """ctx = softmax(mask(q k^T * scale)) v per head (see b2_attention_fwd).

    q_rows = (q_begin, q_count), or a list of up to two such ranges in sequence order, computes
    only those query rows of every sequence (b2_attention_rows_fwd).
    """
    _require(qkv, torch.bfloat16, "qkv")
    _require(ctx, torch.bfloat16, "ctx")
    if kv_len is not None:
        _require(kv_len, torch.int32, "kv_len")
        if kv_len.numel() != batch:
            raise ValueError("kv_len must have one entry per sequence")
    lib = load_library()
    if q_rows is None:
        status = lib.b2_attention_fwd(
            _ptr(qkv), qkv.shape[-1], q_col, k_col, v_col, batch, seq_len, num_heads, head_dim, _ptr(kv_len),
            1 if causal else 0, float(scale), _ptr(ctx), ctx.shape[-1], _stream_ptr(qkv.device),
        )
        _check(status, "b2_attention_fwd")
        return
    ranges = [tuple(q_rows)] if isinstance(q_rows[0], int) else [tuple(r) for r in q_rows]
    arr = (_i64 * (2 * len(ranges)))(*[int(v) for r in ranges for v in r])
    status = lib.b2_attention_rows_fwd(
        _ptr(qkv), qkv.shape[-1], q_col, k_col, v_col, batch, seq_len, num_heads, head_dim, _ptr(kv_len),
        1 if causal else 0, float(scale), arr, len(ranges), _ptr(ctx), ctx.shape[-1], _stream_ptr(qkv.device),
    )
    _check(status, "b2_attention_rows_fwd")


PAD_WORDS = 32  # kPadChannels x kMaxPeers uint32 flags per rank


def peer_barrier(pads, rank: int, channel: int, device: torch.device) -> None:
    """Enqueues a cross-GPU barrier on the current stream (see b2_peer_barrier).

    `pads` lists every rank's flag-pad device address (ints) as mapped into this process.
    """
    arr = (_vp * len(pads))(*[int(p) for p in pads])
    status = load_library().b2_peer_barrier(arr, len(pads), int(rank), int(channel), _stream_ptr(device))
    _check(status, "b2_peer_barrier")


def linear_rs(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], zero_masked_rows: bool, peer_resid,
              rank: int, rows_per_rank: int, ldo: int, row_mask: Optional[torch.Tensor] = None, tile_n: int = 0) -> None:
    """Residual GEMM whose rows are added into their owner rank's residual (see b2_linear_rs_fwd).

    `peer_resid` lists every rank's residual base address (ints) as mapped into this process.
    """
    _require(a, torch.bfloat16, "a")
    _require(w, torch.bfloat16, "w")
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError("a and w disagree on K")
    if bias is not None:
        _require(bias, torch.bfloat16, "bias")
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    arr = (_vp * len(peer_resid))(*[int(x) for x in peer_resid])
    status = load_library().b2_linear_rs_fwd(
        _ptr(a), _ptr(w), _ptr(bias), m, n, k, 1 if zero_masked_rows else 0, arr, len(peer_resid), int(rank),
        int(rows_per_rank), int(ldo), _ptr(row_mask), int(tile_n), _stream_ptr(a.device),
    )
    _check(status, "b2_linear_rs_fwd")


def layernorm_gather(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float, y_ranks,
                     row_mask: Optional[torch.Tensor] = None) -> None:
    """LayerNorm of fp32 rows x written as bf16 into every rank's buffer (see b2_layernorm_gather_fwd).

    `y_ranks` lists each rank's destination address (ints) for x's first row.
    """
    _require(x, torch.float32, "x")
    _require(gamma, torch.bfloat16, "gamma")
    _require(beta, torch.bfloat16, "beta")
    if row_mask is not None:
        _require(row_mask, torch.uint8, "row_mask")
    d_model = x.shape[-1]
    rows = x.numel() // d_model
    arr = (_vp * len(y_ranks))(*[int(p) for p in y_ranks])
    status = load_library().b2_layernorm_gather_fwd(
        _ptr(x), _ptr(gamma), _ptr(beta), float(eps), arr, len(y_ranks), _ptr(row_mask), rows, d_model,
        _stream_ptr(x.device),
    )
    _check(status, "b2_layernorm_gather_fwd")


def linear_bcast(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], peer_out, rank: int, col_begin: int,
                 ldo: int, tile_n: int = 0) -> None:
    """out = bf16(a @ w.T + bias) into peer_out[rank], columns >= col_begin also into every other
    rank's peer_out (see b2_linear_bcast_fwd). `peer_out` lists device addresses (ints)."""
    _require(a, torch.bfloat16, "a")
    _require(w, torch.bfloat16, "w")
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError("a and w disagree on K")
    if bias is not None:
        _require(bias, torch.bfloat16, "bias")
    arr = (_vp * len(peer_out))(*[int(x) for x in peer_out])
    status = load_library().b2_linear_bcast_fwd(
        _ptr(a), _ptr(w), _ptr(bias), m, n, k, arr, len(peer_out), int(rank), int(col_begin), int(ldo), int(tile_n),
        _stream_ptr(a.device),
    )
    _check(status, "b2_linear_bcast_fwd")
