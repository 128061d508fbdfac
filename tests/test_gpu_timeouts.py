"""The GEMM pipeline's bounded waits, made to run out on purpose without faulting the GPU.

With a short wait limit (b2_set_wait_limit) and the test-only fault selector
(b2_test_set_fault(1): CTA 0's producer neither arms nor loads its first stage, as if a TMA
arrival were lost), the MMA issuer's wait for that stage runs out: the kernel records the status
word (kernel 2 = linear, site 3 = the issuer's stage wait, reason 1 = timeout), every role leaves
its loop, tensor memory is freed and the launch returns. The context stays usable and a clean
GEMM afterwards is exact.
"""

import time

import pytest
import torch

from tiktoktechjam2026track3_b200 import _capi

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    _capi.device_status(clear=True)
    yield
    _capi.test_set_fault(0)
    _capi.set_wait_limit(0)
    torch.cuda.synchronize()
    _capi.device_status(clear=True)


def _gemm_case():
    torch.manual_seed(0)
    a = torch.randn(1024, 256, device="cuda").bfloat16()
    w = (torch.randn(512, 256, device="cuda") * 0.05).bfloat16()
    b = torch.randn(512, device="cuda").bfloat16()
    ref = (a.float() @ w.float().t() + b.float()).bfloat16()
    return a, w, b, ref


def test_gemm_stage_wait_runs_out_and_the_context_survives():
    a, w, b, ref = _gemm_case()
    out = torch.zeros(1024, 512, device="cuda", dtype=torch.bfloat16)
    _capi.set_wait_limit(50_000_000)  # 50 ms
    _capi.test_set_fault(1)
    t0 = time.time()
    _capi.linear(a, w, b, _capi.EPI_BIAS, out, tile_n=128)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    _capi.test_set_fault(0)
    _capi.set_wait_limit(0)
    status = _capi.device_status(clear=True)
    assert status == (2 << 16) | (3 << 8) | 1, hex(status)
    assert elapsed < 5.0
    # the context is usable: a clean launch of the same GEMM is right, and the other CTAs' tiles of
    # the faulted launch (32 tiles of 128 x 128, one per CTA; CTA 0 holds rows 0..127 x columns
    # 0..127) are bit-identical to it
    out2 = torch.zeros_like(out)
    _capi.linear(a, w, b, _capi.EPI_BIAS, out2, tile_n=128)
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == 0
    assert (out2.float() - ref.float()).abs().max().item() <= 2 ** -7 * ref.float().abs().max().item()
    assert torch.equal(out[128:], out2[128:]) and torch.equal(out[:128, 128:], out2[:128, 128:])


def test_wait_limit_arguments():
    with pytest.raises(RuntimeError):
        _capi.set_wait_limit(1000)  # below 1 ms
    with pytest.raises(RuntimeError):
        _capi.test_set_fault(7)
