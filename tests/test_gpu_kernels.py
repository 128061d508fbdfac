"""Kernel-level parity on a B200: each sm_100a kernel, called through the C-ABI, against a plain
PyTorch fp32 computation of the same op on the same inputs."""

import pytest
import torch
import torch.nn.functional as F

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200 import _capi

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tf32_and_clean_status(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    _capi.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == 0, "a kernel pipeline wait timed out"


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


# ---------------------------------------------------------------------------------- LayerNorm
@pytest.mark.parametrize("rows,d", [(1000, 256), (777, 768), (300, 1024), (129, 2048), (50, 96), (64, 4096)])
def test_layernorm_fp32_input(rows, d):
    g = _gen(rows + d)
    x = torch.randn(rows, d, device="cuda", generator=g) * 3 + 0.5
    w = (torch.randn(d, device="cuda", generator=g) * 0.2 + 1).bfloat16()
    b = (torch.randn(d, device="cuda", generator=g) * 0.1).bfloat16()
    y = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    _capi.layernorm(x, w, b, 1e-5, y)
    ref = F.layer_norm(x, (d,), w.float(), b.float(), 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=1e-2, rtol=8e-3)


@pytest.mark.parametrize("d", [256, 1024, 96])
def test_layernorm_bf16_input_writes_residual_and_masks_rows(d):
    rows = 333
    g = _gen(d)
    x = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    w = torch.ones(d, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros(d, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    resid = torch.empty(rows, d, device="cuda", dtype=torch.float32)
    mask = (torch.rand(rows, device="cuda", generator=g) > 0.3).to(torch.uint8)
    _capi.layernorm(x, w, b, 1e-5, y, resid_out=resid, row_mask=mask)
    assert torch.equal(resid, x.float())
    ref = F.layer_norm(x.float(), (d,), None, None, 1e-5)
    keep = mask.bool()
    torch.testing.assert_close(y.float()[keep], ref[keep], atol=1e-2, rtol=8e-3)
    assert torch.all(y[~keep] == 0)


# ---------------------------------------------------------------------------------- GEMM
GEMM_SHAPES = [
    (128, 256, 64),
    (4096, 768, 768),    # C2 out_proj (128x192 tiles)
    (200, 384, 200),     # ragged M and K, N not a multiple of 256
    (4096, 2304, 768),   # C2 packed QKV
    (1000, 3072, 768),   # C2 ffn_in, ragged M
    (513, 768, 3072),    # C2 ffn_out, ragged M
    (2048, 1024, 4096),  # C3 ffn_out
    (64, 32, 8),         # tiny
]


def _gemm_inputs(m, n, k, seed):
    g = _gen(seed)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) / k**0.5).bfloat16()
    bias = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16()
    ref = a.float() @ w.float().T + bias.float()
    return a, w, bias, ref


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_gemm_bias_bf16(m, n, k):
    a, w, bias, ref = _gemm_inputs(m, n, k, 1)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _capi.linear(a, w, bias, _capi.EPI_BIAS, out)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES[:4])
def test_gemm_bias_gelu(m, n, k):
    a, w, bias, ref = _gemm_inputs(m, n, k, 2)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _capi.linear(a, w, bias, _capi.EPI_BIAS_GELU, out)
    expect = F.gelu(ref.bfloat16().float(), approximate="none")
    torch.testing.assert_close(out.float(), expect, atol=2e-2, rtol=1e-2)


def test_gelu_epilogue_against_exact_gelu():
    """GELU on exactly representable GEMM outputs (A @ I) against float64 exact-erf GELU.

    The epilogue evaluates erf with a rational formula (|error| <= 3e-7) in fp32,
    so 0.5 x (1 + erf) keeps fp32's absolute cancellation error (~1e-7 |x|) in the negative tail,
    as ATen's fp32 GELU does; elsewhere the result is the correctly rounded bf16 value or one ulp
    away when the exact value sits next to a rounding boundary."""
    g = _gen(11)
    m, k = 4096, 64
    x = (torch.rand(m, k, generator=g, device="cuda") * 20 - 10).bfloat16()
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-3, -1e-3, 9.9, -9.9, 3.0, -3.0]).bfloat16()
    eye = torch.eye(k, device="cuda").bfloat16()
    out = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
    _capi.linear(x, eye, None, _capi.EPI_BIAS_GELU, out)
    exact = F.gelu(x.double(), approximate="none")
    err = (out.double() - exact).abs()
    tol = exact.abs() * 2.0**-8 + x.double().abs() * 2e-7
    assert bool((err <= tol).all()), float((err - tol).max())
    big = exact.abs() > 1e-3
    mismatch = (out.float() != exact.bfloat16().float()) & big
    assert mismatch.float().sum().item() <= 3e-3 * big.sum().item()  # measured: about 0.1%


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("zero", [False, True])
def test_gemm_residual(m, n, k, zero):
    a, w, bias, ref = _gemm_inputs(m, n, k, 3)
    g = _gen(4)
    resid0 = torch.randn(m, n, device="cuda", generator=g)
    mask = (torch.rand(m, device="cuda", generator=g) > 0.25).to(torch.uint8)
    resid = resid0.clone()
    _capi.linear(a, w, bias, _capi.EPI_RESIDUAL_ZERO if zero else _capi.EPI_RESIDUAL, resid, row_mask=mask)
    keep = mask.bool()[:, None]
    expect = torch.where(keep, resid0 + ref, torch.zeros_like(resid0) if zero else resid0)
    torch.testing.assert_close(resid, expect, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES[:3])
def test_gemm_store_f32_and_tile_choice_agree(m, n, k):
    a, w, bias, ref = _gemm_inputs(m, n, k, 5)
    out128 = torch.empty(m, n, device="cuda")
    _capi.linear(a, w, None, _capi.EPI_STORE_F32, out128, tile_n=128)
    torch.testing.assert_close(out128, ref - bias.float(), atol=2e-3, rtol=1e-4)
    for tile in (192, 256):
        if n % tile == 0:
            other = torch.empty(m, n, device="cuda")
            _capi.linear(a, w, None, _capi.EPI_STORE_F32, other, tile_n=tile)
            assert torch.equal(out128, other), tile


PAIR = 0x10000  # B2_TILE_PAIR


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (4096, 2304, 768), (1000, 3072, 768), (300, 768, 3072),
                                   (4096, 768, 768), (32768, 1024, 1024)])
@pytest.mark.parametrize("epi", ["bias", "gelu", "residual_zero", "f32"])
def test_gemm_pair_tiles_match_fp32(m, n, k, epi):
    """The 2-SM (CTA pair, 256-row tile) variant against fp32, every epilogue, N tiles 256 and 192."""
    a, w, bias, ref = _gemm_inputs(m, n, k, 7)
    for bn in (256, 192):
        if n % bn:
            continue
        if epi in ("bias", "gelu"):
            out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            code = _capi.EPI_BIAS if epi == "bias" else _capi.EPI_BIAS_GELU
            _capi.linear(a, w, bias, code, out, tile_n=PAIR | bn)
            expect = ref if epi == "bias" else F.gelu(ref.bfloat16().float(), approximate="none")
            torch.testing.assert_close(out.float(), expect, atol=2e-2, rtol=1e-2)
        elif epi == "f32":
            out = torch.empty(m, n, device="cuda")
            _capi.linear(a, w, None, _capi.EPI_STORE_F32, out, tile_n=PAIR | bn)
            one = torch.empty(m, n, device="cuda")
            _capi.linear(a, w, None, _capi.EPI_STORE_F32, one, tile_n=128)
            torch.testing.assert_close(out, one, atol=1e-5, rtol=1e-6)
        else:
            g = _gen(8)
            resid0 = torch.randn(m, n, device="cuda", generator=g)
            mask = (torch.rand(m, device="cuda", generator=g) > 0.25).to(torch.uint8)
            resid = resid0.clone()
            _capi.linear(a, w, bias, _capi.EPI_RESIDUAL_ZERO, resid, row_mask=mask, tile_n=PAIR | bn)
            keep = mask.bool()[:, None]
            torch.testing.assert_close(resid, torch.where(keep, resid0 + ref, torch.zeros_like(resid0)),
                                       atol=2e-3, rtol=1e-4)


def test_gemm_is_row_invariant():
    """Each output row depends only on its own input row: a sub-batch gives bit-identical rows."""
    a, w, bias, _ = _gemm_inputs(1536, 1024, 1024, 6)
    full = torch.empty(1536, 1024, device="cuda", dtype=torch.bfloat16)
    part = torch.empty(256, 1024, device="cuda", dtype=torch.bfloat16)
    _capi.linear(a, w, bias, _capi.EPI_BIAS, full)
    _capi.linear(a[640:896].contiguous(), w, bias, _capi.EPI_BIAS, part)
    assert torch.equal(full[640:896], part)


# ---------------------------------------------------------------------------------- attention
ATTN_CASES = [
    # batch, seq, heads, hd, causal, lengths (None = no padding)
    (2, 128, 2, 64, True, None),
    (2, 300, 3, 64, False, [300, 129]),
    (1, 1024, 2, 128, True, None),
    (3, 200, 2, 128, True, [200, 77, 1]),
    (2, 2048, 4, 64, True, None),
    (1, 640, 2, 64, False, None),
    (2, 512, 12, 64, False, [256, 511]),
    (2, 300, 2, 128, False, [300, 129]),
    (1, 4096, 2, 128, True, None),
    (1, 384, 1, 128, False, None),
    # enough CTAs that the tensor-core kernel keeps two query tiles per CTA (the small cases above
    # fit one wave either way and run one tile per CTA): even and odd tile counts
    (8, 1024, 16, 64, True, None),
    (4, 1152, 16, 128, False, [1152, 1000, 640, 129]),
    # C2's shape with its padding lengths, causal with padding and ragged lengths (head_dim 64 and
    # 32), a sequence shorter than one query tile
    (8, 512, 12, 64, False, [256, 511, 384, 300, 512, 257, 449, 320]),
    (3, 500, 5, 64, True, [500, 257, 64]),
    (4, 448, 6, 32, True, [448, 65, 1, 200]),
    (1, 65, 1, 64, True, None),
    # CUDA-core kernel (head dims of the reference's official case matrix)
    (2, 128, 4, 32, True, None),
    (3, 200, 4, 8, False, [200, 77, 1]),
    (2, 128, 4, 256, True, None),
    (1, 1024, 4, 32, True, None),
    (4, 32, 4, 32, True, None),
    (2, 130, 16, 8, True, [130, 65]),
    (2, 96, 2, 16, False, None),
]


@pytest.mark.parametrize("batch,seq,heads,hd,causal,lengths", ATTN_CASES)
def test_attention_matches_fp32_reference(batch, seq, heads, hd, causal, lengths):
    d = heads * hd
    g = _gen(seq + hd)
    qkv = torch.randn(batch * seq, 3 * d, device="cuda", generator=g).bfloat16()
    kv_len = None
    key_mask = None
    if lengths is not None:
        kv_len = torch.tensor(lengths, device="cuda", dtype=torch.int32)
        key_mask = torch.arange(seq, device="cuda")[None, :] < kv_len[:, None]
    ctx = torch.zeros(batch * seq, d, device="cuda", dtype=torch.bfloat16)
    scale = hd**-0.5
    _capi.attention(qkv, batch, seq, heads, hd, 0, d, 2 * d, kv_len, causal, scale, ctx)

    t = qkv.float().view(batch, seq, 3, heads, hd)
    q, k, v = (t[:, :, i].transpose(1, 2) for i in range(3))
    ref = oracle.attention_core(q, k, v, key_mask, causal, scale, query_chunk=512)
    ref = ref.transpose(1, 2).reshape(batch, seq, d)
    got = ctx.float().view(batch, seq, d)
    for b in range(batch):
        n = seq if lengths is None else lengths[b]
        torch.testing.assert_close(got[b, :n], ref[b, :n], atol=2e-2, rtol=2e-2)
    assert torch.isfinite(got).all()


@pytest.mark.parametrize("hd,causal,q_begin,q_count", [(64, True, 256, 384), (64, True, 128, 256), (128, True, 384, 640),
                                                       (64, False, 512, 512), (32, True, 128, 384), (128, True, 0, 256),
                                                       (64, True, 896, 128)])
def test_attention_query_row_range_matches_full(hd, causal, q_begin, q_count):
    """b2_attention_rows_fwd writes exactly the requested query rows, bit-identical to the full run
    (each query tile's arithmetic does not depend on which tiles share its CTA)."""
    batch, seq, heads = 2, 1024, 2
    if q_begin + q_count > seq:
        q_count = seq - q_begin
    d = heads * hd
    g = _gen(7 + hd)
    qkv = torch.randn(batch * seq, 3 * d, device="cuda", generator=g).bfloat16()
    kv_len = torch.tensor([seq, 700], device="cuda", dtype=torch.int32)
    full = torch.zeros(batch * seq, d, device="cuda", dtype=torch.bfloat16)
    part = torch.full((batch * seq, d), 7.0, device="cuda", dtype=torch.bfloat16)
    _capi.attention(qkv, batch, seq, heads, hd, 0, d, 2 * d, kv_len, causal, hd**-0.5, full)
    _capi.attention(qkv, batch, seq, heads, hd, 0, d, 2 * d, kv_len, causal, hd**-0.5, part,
                    q_rows=(q_begin, q_count))
    full, part = full.view(batch, seq, d), part.view(batch, seq, d)
    valid = [seq, 700]
    for b in range(batch):
        n = min(valid[b], q_begin + q_count) - q_begin
        if n > 0:
            assert torch.equal(part[b, q_begin:q_begin + n], full[b, q_begin:q_begin + n])
    assert torch.all(part[:, :q_begin] == 7.0) and torch.all(part[:, q_begin + q_count:] == 7.0)


@pytest.mark.parametrize("hd,heads,n", [(64, 2, 256), (128, 2, 256), (32, 2, 256), (64, 64, 512)])
def test_attention_two_query_ranges_match_full(hd, heads, n):
    """Two ranges in one launch (the context-parallel zigzag chunks) equal the full run on their rows
    (64 heads x 2 x 4 query tiles: enough CTAs for two query tiles per CTA)."""
    batch, seq = 1, 2048
    d = heads * hd
    g = _gen(11 + hd)
    qkv = torch.randn(batch * seq, 3 * d, device="cuda", generator=g).bfloat16()
    full = torch.zeros(seq, d, device="cuda", dtype=torch.bfloat16)
    part = torch.full((seq, d), 7.0, device="cuda", dtype=torch.bfloat16)
    ranges = [(256, n), (1536, n)]
    _capi.attention(qkv, batch, seq, heads, hd, 0, d, 2 * d, None, True, hd**-0.5, full)
    _capi.attention(qkv, batch, seq, heads, hd, 0, d, 2 * d, None, True, hd**-0.5, part, q_rows=ranges)
    for r0, cnt in ranges:
        assert torch.equal(part[r0:r0 + cnt], full[r0:r0 + cnt])
    assert torch.all(part[:256] == 7.0) and torch.all(part[256 + n:1536] == 7.0) and torch.all(part[1536 + n:] == 7.0)


def test_attention_reads_heads_at_column_offsets():
    """Q/K/V blocks at arbitrary 64-aligned column offsets of a wider row (tensor-parallel shards)."""
    batch, seq, heads, hd = 1, 256, 2, 64
    d = heads * hd
    g = _gen(11)
    wide = torch.randn(batch * seq, 5 * d, device="cuda", generator=g).bfloat16()
    ctx = torch.zeros(batch * seq, 2 * d, device="cuda", dtype=torch.bfloat16)
    _capi.attention(wide, batch, seq, heads, hd, 4 * d, d, 2 * d, None, True, hd**-0.5, ctx)
    t = wide.float()
    q = t[:, 4 * d:5 * d].view(batch, seq, heads, hd).transpose(1, 2)
    k = t[:, d:2 * d].view(batch, seq, heads, hd).transpose(1, 2)
    v = t[:, 2 * d:3 * d].view(batch, seq, heads, hd).transpose(1, 2)
    ref = oracle.attention_core(q, k, v, None, True, hd**-0.5).transpose(1, 2).reshape(seq, d)
    torch.testing.assert_close(ctx[:, :d].float(), ref, atol=2e-2, rtol=2e-2)
    assert torch.all(ctx[:, d:] == 0)


# ---------------------------------------------------------------------------------- fused add + LayerNorm
@pytest.mark.parametrize("d", [256, 768, 1024, 2048])
@pytest.mark.parametrize("flags", [0, 1, 3])
def test_add_layernorm(d, flags):
    rows = 517
    g = _gen(d + flags)
    resid0 = torch.randn(rows, d, device="cuda", generator=g)
    delta = torch.randn(rows, d, device="cuda", generator=g)
    bias = (torch.randn(d, device="cuda", generator=g) * 0.1).bfloat16()
    w = (torch.randn(d, device="cuda", generator=g) * 0.2 + 1).bfloat16()
    b = (torch.randn(d, device="cuda", generator=g) * 0.1).bfloat16()
    mask = (torch.rand(rows, device="cuda", generator=g) > 0.3).to(torch.uint8)
    resid = resid0.clone()
    y = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    _capi.add_layernorm(resid, delta, bias, w, b, 1e-5, y, row_mask=mask, flags=flags)
    keep = mask.bool()[:, None]
    other = torch.zeros_like(resid0) if flags & 1 else resid0
    expect_r = torch.where(keep, resid0 + delta + bias.float(), other)
    torch.testing.assert_close(resid, expect_r, atol=1e-5, rtol=1e-6)
    expect_y = F.layer_norm(expect_r, (d,), w.float(), b.float(), 1e-5)
    if flags & 2:
        expect_y = torch.where(keep, expect_y, torch.zeros_like(expect_y))
    torch.testing.assert_close(y.float(), expect_y, atol=1e-2, rtol=8e-3)


# ---------------------------------------------------------------------------------- GEMM + residual + LayerNorm
LN_SHAPES = [  # (m, n, k): clusters of 1, 2, 4 and 8 CTAs, ragged m, n below one tile
    (1000, 768, 768),    # C2 out_proj: 4 x 192
    (4096, 768, 3072),   # C2 ffn_out
    (777, 1024, 1024),   # 4 x 256 (3-deep ring)
    (300, 2048, 512),    # 8 x 256
    (513, 384, 256),     # 2 x 192
    (256, 256, 256),     # one CTA, 256 wide
    (130, 96, 64),       # one 128-wide tile holding 96 columns
    (64, 32, 128),       # 32 columns
]


@pytest.mark.parametrize("m,n,k", LN_SHAPES)
@pytest.mark.parametrize("zero", [False, True])
def test_gemm_residual_layernorm(m, n, k, zero):
    """b2_linear_ln_fwd: the residual is bit-identical to the plain residual GEMM with the same tile;
    the LayerNorm output matches the separate LayerNorm kernel on that residual to within one bf16
    ulp (the row statistics are summed in another order) and fp32 F.layer_norm within the usual
    LayerNorm tolerance."""
    a, w, bias, _ = _gemm_inputs(m, n, k, 7)
    g = _gen(8)
    resid0 = torch.randn(m, n, device="cuda", generator=g) * 2 + 0.3
    mask = (torch.rand(m, device="cuda", generator=g) > 0.25).to(torch.uint8)
    gamma = (torch.randn(n, device="cuda", generator=g) * 0.2 + 1).bfloat16()
    beta = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16()
    tile, cluster, _ = _capi.linear_ln_plan(m, n, k)
    assert 1 <= cluster <= 8 and (cluster == 1 or tile * cluster == n)
    resid = resid0.clone()
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _capi.linear_ln(a, w, bias, resid, gamma, beta, 1e-5, y, zero, row_mask=mask)
    plain = resid0.clone()
    _capi.linear(a, w, bias, _capi.EPI_RESIDUAL_ZERO if zero else _capi.EPI_RESIDUAL, plain, row_mask=mask,
                 tile_n=tile)
    assert torch.equal(resid, plain)
    y_sep = torch.empty_like(y)
    _capi.layernorm(plain, gamma, beta, 1e-5, y_sep)
    diff = (y.float() - y_sep.float()).abs()
    assert bool((diff <= y_sep.float().abs() * 2.0**-7 + 1e-6).all()), float(diff.max())
    assert (diff > 0).float().mean().item() < 0.01
    ref = F.layer_norm(plain, (n,), gamma.float(), beta.float(), 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=1e-2, rtol=8e-3)


def test_gemm_residual_layernorm_is_row_invariant_and_deterministic():
    """A row's output does not depend on how many rows share the launch, and repeats bit for bit."""
    m, n, k = 2048, 1024, 1024
    a, w, bias, _ = _gemm_inputs(m, n, k, 9)
    g = _gen(10)
    resid0 = torch.randn(m, n, device="cuda", generator=g)
    gamma = (torch.randn(n, device="cuda", generator=g) * 0.2 + 1).bfloat16()
    beta = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16()
    outs = []
    for rows in (m, m, 384):
        r = resid0[:rows].clone()
        y = torch.empty(rows, n, device="cuda", dtype=torch.bfloat16)
        _capi.linear_ln(a[:rows].contiguous(), w, bias, r, gamma, beta, 1e-5, y, True)
        outs.append((r, y))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][0][:384], outs[2][0]) and torch.equal(outs[0][1][:384], outs[2][1])


# ---------------------------------------------------------------------------------- cross-GPU epilogues, one GPU
# The tensor/context-parallel entry points take every rank's buffer address; here every "rank's"
# buffer is a local tensor, so the owner split, the extra stores and the masks run on one GPU.
@pytest.mark.parametrize("zero", [False, True])
def test_linear_rs_adds_rows_into_their_owner(zero):
    m, n, k, rpr = 1000, 768, 512, 512
    a, w, bias, ref = _gemm_inputs(m, n, k, 21)
    g = _gen(22)
    r0 = torch.randn(m, n, device="cuda", generator=g)
    r1 = torch.randn(m, n, device="cuda", generator=g)
    mask = (torch.rand(m, device="cuda", generator=g) > 0.25).to(torch.uint8)
    res0, res1 = r0.clone(), r1.clone()
    _capi.linear_rs(a, w, bias, zero, [res0.data_ptr(), res1.data_ptr()], 0, rpr, n, row_mask=mask)
    keep = mask.bool()[:, None]
    exp0, exp1 = r0.clone(), r1.clone()
    exp0[:rpr] = torch.where(keep[:rpr], r0[:rpr] + ref[:rpr], torch.zeros_like(r0[:rpr]) if zero else r0[:rpr])
    exp1[rpr:] = torch.where(keep[rpr:], r1[rpr:] + ref[rpr:], r1[rpr:])  # rank 1 zeroes its own masked rows
    torch.testing.assert_close(res0, exp0, atol=2e-3, rtol=1e-4)
    torch.testing.assert_close(res1, exp1, atol=2e-3, rtol=1e-4)


def test_linear_bcast_stores_kv_columns_into_every_copy():
    m, n, k, col_begin = 700, 768, 256, 256
    a, w, bias, _ = _gemm_inputs(m, n, k, 23)
    out0 = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    out1 = torch.full((m, n), 7.0, device="cuda", dtype=torch.bfloat16)
    _capi.linear_bcast(a, w, bias, [out0.data_ptr(), out1.data_ptr()], 0, col_begin, n)
    plain = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _capi.linear(a, w, bias, _capi.EPI_BIAS, plain)
    assert torch.equal(out0, plain)
    assert torch.equal(out1[:, col_begin:], plain[:, col_begin:])
    assert torch.all(out1[:, :col_begin] == 7.0)


def test_layernorm_gather_writes_every_copy():
    rows, d = 333, 768
    g = _gen(24)
    x = torch.randn(rows, d, device="cuda", generator=g) * 2 + 0.3
    w = (torch.randn(d, device="cuda", generator=g) * 0.2 + 1).bfloat16()
    b = (torch.randn(d, device="cuda", generator=g) * 0.1).bfloat16()
    mask = (torch.rand(rows, device="cuda", generator=g) > 0.3).to(torch.uint8)
    y0 = torch.zeros(rows, d, device="cuda", dtype=torch.bfloat16)
    y1 = torch.full((rows, d), 7.0, device="cuda", dtype=torch.bfloat16)
    _capi.layernorm_gather(x, w, b, 1e-5, [y0.data_ptr(), y1.data_ptr()], row_mask=mask)
    expect = F.layer_norm(x, (d,), w.float(), b.float(), 1e-5)
    expect = torch.where(mask.bool()[:, None], expect, torch.zeros_like(expect))
    assert torch.equal(y0, y1)
    torch.testing.assert_close(y0.float(), expect, atol=1e-2, rtol=8e-3)


# ---------------------------------------------------------------------------------- masks
@pytest.mark.parametrize("batch,seq", [(8, 512), (3, 100), (1, 1), (64, 2048)])
def test_mask_lengths_prefixes_and_non_prefixes(batch, seq):
    g = _gen(batch * 7 + seq)
    lengths = torch.randint(0, seq + 1, (batch,), device="cuda", generator=g)
    mask = torch.arange(seq, device="cuda")[None, :] < lengths[:, None]
    if batch > 2:
        mask[1, seq - 1] = not bool(mask[1, seq - 1])  # row 1 breaks the prefix form unless full
        if bool(mask[2, 0]):
            mask[2, 0] = False  # a hole at the start
    kv = torch.full((batch,), -7, device="cuda", dtype=torch.int32)
    bad = torch.full((batch,), 9, device="cuda", dtype=torch.uint8)
    copy = torch.zeros(batch * seq, device="cuda", dtype=torch.uint8)
    _capi.mask_lengths(mask, kv, bad, copy)
    torch.cuda.synchronize()
    assert torch.equal(kv.long(), mask.sum(1))
    prefix = torch.arange(seq, device="cuda")[None, :] < mask.sum(1)[:, None]
    assert torch.equal(bad.bool(), (mask != prefix).any(1))
    assert torch.equal(copy.view(batch, seq).bool(), mask)
