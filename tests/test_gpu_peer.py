"""The cross-GPU flag barrier (b2_peer_barrier) on one GPU, without a peer kernel.

Two barrier kernels that wait on each other never run on the same GPU here, so the peer's side is
played by the host: it sets or leaves unset the flag the peer would write.
"""

import time

import pytest
import torch

from tiktoktechjam2026track3_b200 import _capi

pytestmark = pytest.mark.gpu

WORDS = _capi.PAD_WORDS
MAX_PEERS = 8


def _slot(channel, src):
    return channel * MAX_PEERS + src


@pytest.fixture(autouse=True)
def _setup(cuda_device):
    _capi.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    _capi.device_status(clear=True)


def test_barrier_consumes_peer_signal_and_signals_peer():
    pads = torch.zeros(2, WORDS, dtype=torch.int32, device="cuda")
    ch = 2
    pads[0, _slot(ch, 1)] = 1  # rank 1 has already signalled rank 0 on channel 2
    _capi.peer_barrier([pads[0].data_ptr(), pads[1].data_ptr()], 0, ch, pads.device)
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == 0
    assert pads[0, _slot(ch, 1)].item() == 0  # consumed
    assert pads[1, _slot(ch, 0)].item() == 1  # rank 0's signal waits in rank 1's pad
    others = pads.clone()
    others[0, _slot(ch, 1)] = 0
    others[1, _slot(ch, 0)] = 0
    assert torch.count_nonzero(others) == 0


def test_barrier_times_out_with_status_when_peer_never_signals():
    pads = torch.zeros(2, WORDS, dtype=torch.int32, device="cuda")
    t0 = time.time()
    _capi.peer_barrier([pads[0].data_ptr(), pads[1].data_ptr()], 0, 0, pads.device)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    status = _capi.device_status(clear=True)
    assert status >> 16 == 4 and status & 0xFF == 1, hex(status)  # peer barrier, timeout
    assert 3.0 < elapsed < 30.0
    assert pads[1, _slot(0, 0)].item() == 1
    # the context is still usable
    assert torch.ones(4, device="cuda").sum().item() == 4


def test_barrier_argument_checks():
    pads = torch.zeros(2, WORDS, dtype=torch.int32, device="cuda")
    ptrs = [pads[0].data_ptr(), pads[1].data_ptr()]
    with pytest.raises(RuntimeError):
        _capi.peer_barrier(ptrs, 2, 0, pads.device)  # rank outside world
    with pytest.raises(RuntimeError):
        _capi.peer_barrier(ptrs, 0, 4, pads.device)  # channel out of range
    with pytest.raises(RuntimeError):
        _capi.peer_barrier(ptrs * 5, 0, 0, pads.device)  # 10 ranks
    _capi.peer_barrier(ptrs[:1], 0, 0, pads.device)  # one rank: no-op
    torch.cuda.synchronize()
    assert torch.count_nonzero(pads) == 0
