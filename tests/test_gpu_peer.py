"""The NVLink exchange's cross-GPU barrier on one GPU: the count it keeps in device memory, and its
bounded wait (a peer that never arrives sets the timeout status bit and the kernel returns; the
context stays usable).  No two waiting kernels run as separate launches on one GPU."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _barrier(lib, signals, peer_ptrs, rank, world):
    arr = (ctypes.c_void_p * world)(*peer_ptrs)
    return lib.ogx_peer_barrier(signals.data_ptr(), arr, rank, world, torch.cuda.current_stream().cuda_stream)


def test_barrier_count_advances(ogx_lib):
    from opengenie_b200 import _lib

    sig = torch.zeros(16, dtype=torch.int32, device="cuda")
    for _ in range(3):
        assert _barrier(ogx_lib, sig, [sig.data_ptr()], 0, 1) == 0
    torch.cuda.synchronize()
    assert sig[8].item() == 3
    assert _lib.device_status(clear=True) == 0


def test_barrier_wait_is_bounded(ogx_lib):
    """Rank 0 of 2 with a peer that never signals: the wait gives up after its limit (about a second),
    records the timeout and returns."""
    from opengenie_b200 import _lib

    sig = torch.zeros(16, dtype=torch.int32, device="cuda")
    absent_peer = torch.zeros(16, dtype=torch.int32, device="cuda")  # stands in for the peer's block
    _lib.device_status(clear=True)
    assert _barrier(ogx_lib, sig, [sig.data_ptr(), absent_peer.data_ptr()], 0, 2) == 0
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & _lib.OGX_ERR_TIMEOUT
    assert absent_peer[0].item() == 1  # the arrival was still published
    assert sig[8].item() == 1
    # the context is usable afterwards
    assert torch.arange(4, device="cuda").sum().item() == 6


def test_barrier_rejects_bad_arguments(ogx_lib):
    sig = torch.zeros(16, dtype=torch.int32, device="cuda")
    assert _barrier(ogx_lib, sig, [sig.data_ptr()] * 2, 2, 2) != 0
    assert _barrier(ogx_lib, sig, [sig.data_ptr()] * 9, 0, 9) != 0
