"""GPU, one device: the signal-pad barrier of the peer-memory pipeline, its completion and its bounded wait.

A second rank is emulated by a local buffer standing for its signal pad. When that rank's signal is already in this
rank's pad the barrier completes and leaves the error flag 0; when nothing ever signals, the wait runs out after its
time limit and the kernel returns with error 201 (a dead or late peer), the device still usable: no fault, no hang."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def barrier(own, peer_pad, epoch, timeout_ns, err):
    from hffn_b200 import _native as native
    peers = (ctypes.c_uint64 * 2)(0, peer_pad.data_ptr())       # rank 0 (this one) needs no entry
    native.check(native.lib.hffn_peer_barrier(own.data_ptr(), peers, 2, 0, epoch, timeout_ns, err.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream), "hffn_peer_barrier")
    torch.cuda.synchronize()


def test_barrier_completes_when_the_peer_has_signalled():
    own = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer_pad = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    own[1] = 5                                                   # rank 1 reached epoch 5 already
    barrier(own, peer_pad, 5, 2_000_000_000, err)
    assert int(err.item()) == 0
    assert int(peer_pad[0].item()) == 5                          # this rank's signal landed in rank 1's pad


def test_barrier_wait_runs_out_with_an_error_status():
    own = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer_pad = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    start = time.perf_counter()
    barrier(own, peer_pad, 1, 50_000_000, err)                   # nothing ever signals: 50 ms limit
    elapsed = time.perf_counter() - start
    assert int(err.item()) == 201
    assert elapsed < 5.0
    # the context is intact: ordinary work runs and the barrier works again once the peer signals
    assert float(torch.ones(1000, device="cuda").sum()) == 1000.0
    err.zero_()
    own[1] = 2
    barrier(own, peer_pad, 2, 2_000_000_000, err)
    assert int(err.item()) == 0
