"""Failure detection on the GPU without a GPU fault.

The multi-GPU kernels wait on flags that other ranks write (the fused
all-gather's ready and done flags, the reduce-scatter's finish flags).  Every
such wait gives up after a bounded time (2 s of %globaltimer), records
kDevTimeoutPeer (6) in the library's device error word and returns, so a rank
whose peer never arrives gets an error status instead of a hung GPU.  Here the
"peer" is a second flag block on the same GPU that nothing ever writes: the
wait must run out, the host must read the status, and the context must stay
usable.  No kernel waits on another kernel."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_PEER = 6


def _flags(dev):
    from imagine_b200 import _native as N

    mine = torch.zeros(N.PEER_FLAG_WORDS, dtype=torch.int32, device=dev)
    peer = torch.zeros(N.PEER_FLAG_WORDS, dtype=torch.int32, device=dev)
    ptrs = (ctypes.c_void_p * 2)(mine.data_ptr(), peer.data_ptr())
    return mine, peer, ptrs


def _still_usable(dev):
    import imagine_b200 as W

    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(128, 256, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wq, ws = W.quantize_weight(w)
    y = W.int8_linear(x, wq, ws)
    torch.cuda.synchronize(dev)
    assert torch.isfinite(y.float()).all()
    assert W.device_error(dev) == 0


def test_peer_barrier_times_out():
    import imagine_b200 as W
    from imagine_b200 import _native as N
    from imagine_b200.linear import _stream

    dev = torch.device("cuda", 0)
    W.device_error(dev)  # start clean
    mine, peer, ptrs = _flags(dev)
    N.check(N.LIB.w8a8_peer_barrier(ptrs, 0, 2, 1, _stream(dev)))
    torch.cuda.synchronize(dev)
    assert W.device_error(dev) == TIMEOUT_PEER
    # the barrier did signal its own arrival into the peer's ready slot 0
    assert int(peer[0]) == 1 and int(mine[1]) == 0
    _still_usable(dev)


def test_allgather_finish_times_out():
    """The done-wait of the fused all-gather gives up; the unpack that follows
    copies whatever the receive buffer holds (here zeros) and faults nothing."""
    import imagine_b200 as W
    from imagine_b200 import _native as N
    from imagine_b200.linear import _stream

    dev = torch.device("cuda", 0)
    W.device_error(dev)
    mine, peer, ptrs = _flags(dev)
    m, ns = 64, 128
    nbytes = int(N.LIB.w8a8_allgather_recv_bytes(m, ns, N.BF16, 2))
    recv0 = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    recv1 = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    recvs = (ctypes.c_void_p * 2)(recv0.data_ptr(), recv1.data_ptr())
    out = torch.full((m, 2 * ns), 7.0, dtype=torch.bfloat16, device=dev)
    N.check(N.LIB.w8a8_allgather_finish(out.data_ptr(), N.BF16, 2 * ns, m, ns, recvs, ptrs, 0, 2, 1,
                                        _stream(dev)))
    torch.cuda.synchronize(dev)
    assert W.device_error(dev) == TIMEOUT_PEER
    assert bool((out[:, :ns] == 7.0).all())  # this rank's own columns are untouched
    _still_usable(dev)
