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
