"""Times one kernel of libb200tx.so in isolation (CUDA events on the launching stream).

    python -m tiktoktechjam2026track3_b200.kernel_bench gemm --m 65536 --n 3072 --k 768 --epi gelu
    python -m tiktoktechjam2026track3_b200.kernel_bench attention --b 4 --s 8192 --h 16 --hd 64 --causal
    python -m tiktoktechjam2026track3_b200.kernel_bench layernorm --rows 400000 --d 1024

Each run does --warmup untimed launches, then --iters timed launches, each preceded by an L2
flush (256 MiB write), and prints one JSON line: average launch time, algorithmic work per launch
(GEMM 2MNK FLOPs; attention 4*hd*H*pairs FLOPs over useful query/key pairs; LayerNorm bytes read
+ written) and the achieved rate. Used for tile sweeps and as the small-case target of ncu captures.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _capi

EPI = {"bias": _capi.EPI_BIAS, "gelu": _capi.EPI_BIAS_GELU, "residual": _capi.EPI_RESIDUAL,
       "residual_zero": _capi.EPI_RESIDUAL_ZERO, "f32": _capi.EPI_STORE_F32}


def _time(fn, warmup: int, iters: int) -> float:
    flush = torch.empty(64 << 20, device="cuda", dtype=torch.float32)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.fill_(0.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="kernel", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, required=True)
    g.add_argument("--n", type=int, required=True)
    g.add_argument("--k", type=int, required=True)
    g.add_argument("--epi", choices=sorted(EPI), default="bias")
    g.add_argument("--tile-n", type=int, default=0)
    a = sub.add_parser("attention")
    a.add_argument("--b", type=int, required=True)
    a.add_argument("--s", type=int, required=True)
    a.add_argument("--h", type=int, required=True)
    a.add_argument("--hd", type=int, default=64)
    a.add_argument("--causal", action="store_true")
    a.add_argument("--min-len", type=int, default=0, help="padding: lengths uniform in [min-len, s]")
    ln = sub.add_parser("layernorm")
    ln.add_argument("--rows", type=int, required=True)
    ln.add_argument("--d", type=int, required=True)
    ln.add_argument("--bf16-in", action="store_true")
    for sp in (g, a, ln):
        sp.add_argument("--warmup", type=int, default=3)
        sp.add_argument("--iters", type=int, default=10)
    args = p.parse_args(argv)
    torch.manual_seed(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    _capi.device_status(clear=True)
    result = {"kernel": args.kernel}

    if args.kernel == "gemm":
        m, n, k = args.m, args.n, args.k
        x = torch.randn(m, k, device=dev).bfloat16()
        w = (torch.randn(n, k, device=dev) / k**0.5).bfloat16()
        bias = torch.randn(n, device=dev).bfloat16()
        epi = EPI[args.epi]
        out = torch.zeros(m, n, device=dev, dtype=torch.bfloat16 if epi in (0, 1) else torch.float32)
        ms = _time(lambda: _capi.linear(x, w, bias, epi, out, tile_n=args.tile_n), args.warmup, args.iters)
        flops = 2.0 * m * n * k
        result.update(shape=[m, n, k], epi=args.epi, tile_n=args.tile_n, ms=ms, tflops=flops / ms / 1e9,
                      bytes_min=(m * k + n * k) * 2 + m * n * out.element_size() * (2 if epi in (2, 3) else 1))
    elif args.kernel == "attention":
        b, s, h, hd = args.b, args.s, args.h, args.hd
        d = h * hd
        qkv = torch.randn(b * s, 3 * d, device=dev).bfloat16()
        ctx = torch.empty(b * s, d, device=dev, dtype=torch.bfloat16)
        kv_len = None
        lens = [s] * b
        if args.min_len > 0:
            kv_len = torch.randint(args.min_len, s + 1, (b,), device=dev, dtype=torch.int32)
            lens = kv_len.tolist()
        ms = _time(lambda: _capi.attention(qkv, b, s, h, hd, 0, d, 2 * d, kv_len, args.causal, hd**-0.5, ctx),
                   args.warmup, args.iters)
        pairs = sum(n * (n + 1) / 2 for n in lens) if args.causal else sum(float(n) * n for n in lens)
        flops = 4.0 * hd * h * pairs
        result.update(shape=[b, s, h, hd], causal=args.causal, ms=ms, tflops=flops / ms / 1e9)
    else:
        rows, d = args.rows, args.d
        x = torch.randn(rows, d, device=dev, dtype=torch.bfloat16 if args.bf16_in else torch.float32)
        gamma = torch.ones(d, device=dev, dtype=torch.bfloat16)
        beta = torch.zeros(d, device=dev, dtype=torch.bfloat16)
        y = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
        resid = torch.empty(rows, d, device=dev) if args.bf16_in else None
        ms = _time(lambda: _capi.layernorm(x, gamma, beta, 1e-5, y, resid_out=resid), args.warmup, args.iters)
        nbytes = rows * d * (x.element_size() + 2 + (4 if args.bf16_in else 0))
        result.update(shape=[rows, d], ms=ms, gbs=nbytes / ms / 1e6, bytes=nbytes)
    torch.cuda.synchronize()
    result["device_status"] = _capi.device_status(clear=True)
    print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
