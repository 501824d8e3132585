"""There is no CPU fallback: without the library, or with CPU tensors, the product path raises."""
import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "deepseek-v4-flash-2bit-gb10_b200")


def test_missing_library_raises():
    code = """
import torch
from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
try:
    from vq2_vllm import _lib
    _lib.lib()
except RuntimeError as ex:
    print("raised:", ex)
"""
    env = dict(os.environ, VQ2_LIB=os.path.join(REPO, "no_such_dir", "libvq2_b200.so"),
               PYTHONPATH=os.pathsep.join([PKG, REPO]))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "raised:" in r.stdout and "no fallback" in r.stdout


def test_cpu_tensors_are_rejected():
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    from vq2_vllm.kernels.moe_align import moe_align
    from vq2_vllm.kernels.router import router_topk
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    layer = synth.make_layer(4, 128, 64, seed=0)
    x = synth.make_tokens(2, 128, seed=1)
    ids, w = synth.route_softmax_topk(x, 4, 2, w_std=0.02, seed=2)
    for fn in (vq2_moe_fused_10b, vq2_moe_grouped_wmma):
        with pytest.raises(RuntimeError, match="no CPU path"):
            fn(x, ids, w, *synth.layer_args(layer))
    with pytest.raises(RuntimeError, match="no CPU path"):
        moe_align(ids, 4, 64)
    with pytest.raises(RuntimeError, match="no CPU path"):
        router_topk(x, torch.zeros(128, 4, dtype=torch.bfloat16), 2)


def test_packer_rejects_bad_arguments_without_a_gpu():
    """The packer's argument checks run on the host before any launch: the mirror raises on
    unsupported formats and CPU tensors, the C ABI returns its error codes."""
    from vq2_vllm import _lib
    from vq2_vllm.kernels.vq2_kernel import pack_vq2
    with pytest.raises(ValueError):
        pack_vq2(torch.zeros(4, 64), k=2048)
    with pytest.raises(RuntimeError, match="no CPU path"):
        pack_vq2(torch.zeros(4, 64), k=64)
    L = _lib.lib()
    fake = 1 << 20                                   # never dereferenced: every call below fails its checks
    assert L.vq2_pack_assign(fake, 0, 4, 64, fake, 2000, None, None, None, fake, None, None) == 2   # k > 1024
    assert L.vq2_pack_assign(fake, 0, 4, 64, fake + 4, 16, None, None, None, fake, None, None) == 3  # C unaligned
    assert L.vq2_pack_assign(fake, 0, 4, 64, fake, 16, fake, None, None, fake, None, None) == 1   # lo without hi
    assert L.vq2_pack_assign(fake, 7, 4, 64, fake, 16, None, None, None, fake, None, None) == 4   # dtype
    assert L.vq2_kmeans(fake, 10, fake, 16, 3, None, 0, None) == 5                                # workspace
    assert L.vq2_pack_gather(fake, 0, 4, 64, fake, 5, fake + 8, None) == 3                       # out unaligned
    assert L.vq2_kmeans_workspace_size(1025) == 0


def test_shared_expert_rejects_bad_arguments_without_a_gpu():
    from vq2_vllm import _lib
    from vq2_vllm.kernels.shared_expert import shared_expert_fused
    with pytest.raises(RuntimeError, match="no CPU path"):
        shared_expert_fused(torch.zeros(1, 256), torch.zeros(512, 256, dtype=torch.bfloat16),
                            torch.zeros(256, 256, dtype=torch.bfloat16))
    L = _lib.lib()
    fake = 1 << 20
    assert L.vq2_shared_expert(fake, 0, fake, fake, 9, 256, 256, fake, 0, fake, 1 << 20, None) == 2     # N > 8
    assert L.vq2_shared_expert(fake, 0, fake, fake, 1, 320, 256, fake, 0, fake, 1 << 20, None) == 2     # H % 256
    assert L.vq2_shared_expert(fake, 0, fake + 2, fake, 1, 256, 256, fake, 0, fake, 1 << 20, None) == 3  # alignment
    assert L.vq2_shared_expert(fake, 0, fake, fake, 1, 256, 256, fake, 0, None, 0, None) == 5           # workspace
    assert L.vq2_shared_expert(None, 0, fake, fake, 1, 256, 256, fake, 0, fake, 1 << 20, None) == 1     # null


def test_fused_ep_and_coscheduled_entries_reject_bad_arguments_without_a_gpu():
    """vq2_ep_decode and vq2_decode_with_shared return their error codes before any CUDA call."""
    import ctypes
    from vq2_vllm import _lib
    L = _lib.lib()
    fake = 1 << 20
    a = _lib.Vq2MoeArgs()
    a.N, a.H, a.I, a.E, a.topk, a.x_dtype, a.ids_dtype = 1, 4096, 2048, 32, 8, 0, 0
    a.x = a.topk_ids = a.topk_w = a.out = fake
    a.w13_cb = a.w13_lo = a.w13_hi = a.w13_sc = a.w2_cb = a.w2_lo = a.w2_hi = a.w2_sc = fake
    lay = _lib.Vq2EpLayout(0, 256, 512, 768, 1024, 1280, 1536, 1552)
    ref, lref = ctypes.byref(a), ctypes.byref(lay)
    assert L.vq2_ep_decode(None, fake, 2, 0, fake, lref, fake, 1 << 20, None) == 1            # null args
    assert L.vq2_ep_decode(ref, fake, 0, 0, fake, lref, fake, 1 << 20, None) == 2             # world 0
    assert L.vq2_ep_decode(ref, fake, 2, 2, fake, lref, fake, 1 << 20, None) == 2             # rank >= world
    a.N = 2
    assert L.vq2_ep_decode(ref, fake, 64, 0, fake, lref, fake, 1 << 20, None) == 6            # 64*2*8 > 512 pairs
    a.N = 1
    bad = _lib.Vq2EpLayout(0, 256, 512, 768, 1024, 1280, 1536, 1544)
    assert L.vq2_ep_decode(ref, fake, 2, 0, fake, ctypes.byref(bad), fake, 1 << 20, None) == 3  # offset % 16
    a.ids_dtype = 5
    assert L.vq2_ep_decode(ref, fake, 2, 0, fake, lref, fake, 1 << 20, None) == 4             # dtype
    a.ids_dtype = 0
    assert L.vq2_decode_with_shared(None, fake, fake, 2048, 0, fake, 1 << 30, None) == 1     # null args
    a.N = 9
    assert L.vq2_decode_with_shared(ref, fake, fake, 2048, 0, fake, 1 << 30, None) == 2      # shared part N > 8
    a.N = 1
    assert L.vq2_decode_with_shared(ref, fake, fake, 2048, 0, None, 0, None) == 5            # workspace
    assert L.vq2_decode_with_shared(ref, fake + 2, fake, 2048, 0, fake, 1 << 30, None) == 3  # alignment
    assert L.vq2_decode_with_shared_workspace_size(1, 8, 4096, 2048, 2048) >= \
        L.vq2_decode_workspace_size(1, 8, 4096, 2048) + L.vq2_shared_expert_workspace_size(1, 2048)
