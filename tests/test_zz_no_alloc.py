"""The allocation-free cross-GPU barrier (ogx_peer_barrier_static) against the barrier that takes a
caller-allocated signal block (ogx_peer_barrier).  Callers that cannot allocate device memory, such
as a runtime that reserves all of its GPUs' memory for its own pool before serving, use the static
variant; it must count barriers exactly as the allocated one does.

This file is named to be collected last: the static signal block lives for the whole process, so
nothing else in the test run touches it before this test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_static_barrier_counts_like_allocated_barrier(ogx_lib):
    from opengenie_b200 import _lib

    stream = torch.cuda.current_stream().cuda_stream
    dev = torch.cuda.current_device()
    _lib.device_status(clear=True)

    # the existing entry point, on a signal block the caller allocated
    sig = torch.zeros(16, dtype=torch.int32, device="cuda")
    peers = (ctypes.c_void_p * 1)(sig.data_ptr())
    allocated = []
    for _ in range(2):
        assert ogx_lib.ogx_peer_barrier(sig.data_ptr(), peers, 0, 1, stream) == 0
        torch.cuda.synchronize()
        allocated.append(int(sig[8].item()))

    # the allocation-free entry point (count_out is an output the caller provides)
    devices = (ctypes.c_int * 1)(dev)
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    static = []
    for _ in range(2):
        assert ogx_lib.ogx_peer_barrier_static(0, 1, devices, count.data_ptr(), stream) == 0, \
            ogx_lib.ogx_last_error()
        torch.cuda.synchronize()
        static.append(int(count.item()))

    assert allocated == [1, 2]
    assert static == allocated
    assert _lib.device_status(clear=True) == 0


def test_static_barrier_rejects_more_ranks_than_its_block_holds(ogx_lib):
    dev = torch.cuda.current_device()
    devices = (ctypes.c_int * 9)(*([dev] * 9))
    stream = torch.cuda.current_stream().cuda_stream
    assert ogx_lib.ogx_peer_barrier_static(0, 9, devices, None, stream) != 0
    assert b"at most 8 ranks" in ogx_lib.ogx_last_error()
    assert ogx_lib.ogx_peer_barrier_static(1, 1, devices, None, stream) != 0


def test_static_barrier_rejects_a_device_named_twice(ogx_lib):
    dev = torch.cuda.current_device()
    devices = (ctypes.c_int * 2)(dev, dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert ogx_lib.ogx_peer_barrier_static(0, 2, devices, None, stream) != 0
    assert b"both name device" in ogx_lib.ogx_last_error()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in this process")
def test_static_barrier_across_two_gpus_of_one_process(ogx_lib):
    """The part the one-GPU case cannot reach: each device's own count looked up on that device, and the
    arrivals crossing between the GPUs through the library's page-locked host slots (no GPU touches the
    other's memory).  Two ranks on GPUs 0 and 1 of this process, each on its own stream, pass two
    barriers together."""
    from opengenie_b200 import _lib

    counts = [torch.zeros(1, dtype=torch.int32, device=f"cuda:{d}") for d in (0, 1)]
    streams = [torch.cuda.Stream(device=d) for d in (0, 1)]
    solo = (ctypes.c_int * 1)()

    def one_rank_barrier(d):
        # a group of one on device d: advances d's count by one and returns it
        solo[0] = d
        with torch.cuda.device(d):
            assert ogx_lib.ogx_peer_barrier_static(0, 1, solo, counts[d].data_ptr(), streams[d].cuda_stream) == 0, \
                ogx_lib.ogx_last_error()
            streams[d].synchronize()
        return int(counts[d].item())

    # the counts live for the whole process: bring both devices to the same barrier number first
    c = [one_rank_barrier(0), one_rank_barrier(1)]
    while c[0] != c[1]:
        lo = 0 if c[0] < c[1] else 1
        c[lo] = one_rank_barrier(lo)
    start = c[0]
    for d in (0, 1):
        with torch.cuda.device(d):
            _lib.device_status(clear=True)

    devices = (ctypes.c_int * 2)(0, 1)
    seen = {0: [], 1: []}
    for _ in range(2):
        for r in (0, 1):
            with torch.cuda.device(r):
                assert ogx_lib.ogx_peer_barrier_static(r, 2, devices, counts[r].data_ptr(),
                                                       streams[r].cuda_stream) == 0, ogx_lib.ogx_last_error()
        for r in (0, 1):
            streams[r].synchronize()
            seen[r].append(int(counts[r].item()))
    assert seen[0] == [start + 1, start + 2]
    assert seen[1] == seen[0]
    for d in (0, 1):
        with torch.cuda.device(d):
            assert _lib.device_status(clear=True) == 0
