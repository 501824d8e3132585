"""Failure detection of the peer-memory exchange without a GPU fault: a dispatch whose second
source never arrives (a flag that nothing sets) gives up after its bounded wait, reports
VQ2_ERR_TIMEOUT through the device status word, and leaves the context usable.

One GPU: the exchange region of this process is listed as both "ranks" of a world of 2, so rank 1's
pushes and flags never happen."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_dispatch_wait_times_out_and_context_survives():
    from vq2_vllm import _lib
    from vq2_vllm import ep
    L = _lib.lib()
    L.vq2_device_status(1)                        # clear
    H, k, N, W = 256, 8, 1, 2
    row_x = H * 2
    off = ep.P2PExchange.layout(W, N, H, k, row_x)
    o = off["bytes"]
    p = ctypes.c_void_p()
    _lib.check(L.vq2_ep_alloc(o, ctypes.byref(p)), "vq2_ep_alloc")
    base = p.value
    try:
        row = [base + off["x"], base + off["ids"], base + off["w"], base + off["comb"], base + off["dflag"],
               base + off["cflag"]]
        peers = torch.tensor([row, row], dtype=torch.int64, device="cuda")
        x = torch.randn(N, H, device="cuda").bfloat16()
        ids = torch.zeros(N, k, dtype=torch.int32, device="cuda")
        w = torch.ones(N, k, device="cuda")
        rc = L.vq2_ep_dispatch(x.data_ptr(), ids.data_ptr(), 0, w.data_ptr(), N, row_x, k, peers.data_ptr(), W, 0,
                               base, off["dflag"], off["epoch"], _lib.stream_ptr())
        assert rc == 0
        torch.cuda.synchronize()                  # returns: the wait is bounded
        assert L.vq2_device_status(1) == 8        # VQ2_ERR_TIMEOUT
        # the context is still usable
        y = (torch.arange(1024, device="cuda") * 2).sum().item()
        assert y == 1023 * 1024
        assert L.vq2_device_status(0) == 0
    finally:
        L.vq2_ep_free(base)
