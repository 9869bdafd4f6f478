"""The KV-head exchange barrier gives up with an error status, on one GPU.

cxs_exchange_barrier waits (bounded) for a peer's flag. Here the "peer" flag
array is a second local device word that nothing writes, so the wait runs
out: the kernel must record CXS_DEVICE_ERR_READY_TIMEOUT in the error word
and return, leaving the context usable. No GPU fault, trap or unbounded wait
is involved: every address is a valid allocation on this GPU, and the spin
limit is about 10 ms of clock cycles.
"""

import ctypes

import pytest
import torch

from cxlsparse_b200 import _lib

pytestmark = pytest.mark.gpu

COUNTER, FLAGS, PEER_FLAGS, ERROR = 0, 64, 128, 192  # byte offsets in one allocation


class _Words:
    """64 int32 words of a raw device allocation, viewed as a tensor."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = dict(shape=(n,), typestr="<i4", data=(ptr, False),
                                             version=3, strides=None)


def test_exchange_barrier_times_out_with_error_status(cuda):
    lib = _lib.lib()
    ptr = ctypes.c_void_p()
    _lib.check(lib.cxs_device_alloc(256, ctypes.byref(ptr)))
    base = ptr.value
    try:
        words = torch.as_tensor(_Words(base, 64), device=cuda)  # zeroed by the alloc
        peer_flags = (ctypes.c_void_p * 2)(0, base + PEER_FLAGS)
        stream = torch.cuda.current_stream()
        _lib.check(lib.cxs_exchange_barrier(base + COUNTER, peer_flags, base + FLAGS, 0, 2,
                                            20_000_000, base + ERROR, stream.cuda_stream))
        torch.cuda.synchronize()
        assert int(words[ERROR // 4]) & _lib.DEVICE_ERR_READY_TIMEOUT
        assert int(words[COUNTER // 4]) == 1               # step 1 was taken
        assert int(words[PEER_FLAGS // 4]) == 1            # and announced to the "peer"
        # The context is still usable: with the peer's announcement in place the
        # next step passes without an error.
        words[ERROR // 4] = 0
        words[FLAGS // 4 + 1] = 2
        _lib.check(lib.cxs_exchange_barrier(base + COUNTER, peer_flags, base + FLAGS, 0, 2,
                                            20_000_000, base + ERROR, stream.cuda_stream))
        torch.cuda.synchronize()
        assert int(words[ERROR // 4]) == 0 and int(words[COUNTER // 4]) == 2
        assert torch.ones(4, device=cuda).sum().item() == 4
    finally:
        torch.cuda.synchronize()
        _lib.check(lib.cxs_device_free(base))
