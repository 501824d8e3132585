"""The allocation-free decode entry point, called through the C ABI.

Some callers cannot allocate device memory when they call into the library (a memory pool that
forbids new allocations, a driver callback, a host runtime without a CUDA allocator), so
vq2_decode_noalloc takes its scratch from a fixed array inside the library. This checks that two
calls in a row, with different inputs, give the same result as the workspace entry point
vq2_decode within the decode tolerance, and that an over-limit request is refused with its own
error code. Collected last on purpose (file name), so a failure here stops nothing else.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-5   # same kernels; only the order of the fp32 output atomics differs


def _call(entry, layer, x, ids, tw):
    from vq2_vllm import _lib, synth
    L = _lib.lib()
    out = torch.empty(x.shape[0], x.shape[1], device="cuda", dtype=torch.float32)
    a = _lib.moe_args(x, ids, tw, *synth.layer_args(layer), out)
    stream = torch.cuda.current_stream().cuda_stream
    if entry == "noalloc":
        rc = L.vq2_decode_noalloc(ctypes.byref(a), stream)
    else:
        nb = L.vq2_decode_workspace_size(a.N, a.topk, a.H, a.I)
        ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
        rc = L.vq2_decode(ctypes.byref(a), ws.data_ptr(), nb, stream)
    torch.cuda.synchronize()
    return rc, out


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def test_noalloc_matches_workspace_entry_twice():
    from vq2_vllm import _lib, synth
    layer = synth.make_layer(32, 4096, 2048, seed=0, device="cuda")
    for call, (N, seed) in enumerate([(1, 11), (8, 12)]):      # 8 tokens x top-8 = the 2 MiB limit
        x = synth.make_tokens(N, 4096, seed=seed, device="cuda")
        ids, tw = synth.route_softmax_topk(x, 32, 8, w_std=0.02, seed=seed + 100)
        rc, got = _call("noalloc", layer, x, ids, tw)
        assert rc == 0, _lib.lib().vq2_strerror(rc)
        rc2, want = _call("workspace", layer, x, ids, tw)
        assert rc2 == 0
        assert _rel(got, want) < TOL, f"call {call}"


def test_noalloc_rejects_over_limit():
    from vq2_vllm import _lib, synth
    layer = synth.make_layer(16, 4096, 2048, seed=1, device="cuda")
    x = synth.make_tokens(9, 4096, seed=3, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 16, 8, w_std=0.02, seed=4)
    rc, _ = _call("noalloc", layer, x, ids, tw)
    assert rc == 10, "expected VQ2_ERR_NOALLOC_LIMIT"
    assert b"VQ2_NOALLOC_SCRATCH_BYTES" in _lib.lib().vq2_strerror(rc)
