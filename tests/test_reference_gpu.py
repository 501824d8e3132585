"""Parity against the reference's own GPU kernels on the same inputs, at the config-1 widths.

Uses an unmodified install of the reference in baseline/_ref (its Triton decode kernels; its
prefill extension built for sm_100a by baseline/build_ref_ext.py); skipped when that install is
absent. Tolerances: decode 1e-2 relative L2 (both paths approximate the fp32 MoE; measured
3.7e-3 apart at full size), fp8 prefill 5e-3 (the same algorithm on both sides; measured 4.9e-4).
"""
import os

import pytest
import torch

from oracle import torch_ref

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HAVE_REF = os.path.isdir(os.path.join(REPO, "baseline", "_ref", "vq2_vllm", "kernels"))


@pytest.fixture(scope="module")
def refs():
    if not HAVE_REF:
        pytest.skip("reference not installed in baseline/_ref")
    from baseline.ref_modules import RefModules
    return RefModules()


@pytest.fixture(scope="module")
def layer():
    from vq2_vllm import synth
    return synth.make_layer(16, 4096, 2048, seed=41, device="cuda")


@pytest.mark.parametrize("N", [1, 3, 16])
def test_decode_vs_reference_triton(refs, layer, N):
    from vq2_vllm import synth
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    x = synth.make_tokens(N, 4096, seed=42 + N, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 16, 8, w_std=0.02, seed=43 + N)
    ours = vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(layer))
    with refs as m:
        theirs = m["vq2_kernel"].vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(layer))
    torch.cuda.synchronize()
    assert torch_ref.rel_l2(ours, theirs) < 1e-2


def test_prefill_fp8_vs_reference_cuda(refs, layer):
    if not refs.has_prefill:
        pytest.skip("reference prefill extension not built for sm_100a")
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    N = 512
    x = synth.make_tokens(N, 4096, seed=44, device="cuda")
    ids, tw = synth.route_zipf(N, 16, 8, seed=45, device="cuda")
    ours = vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(layer), precision="fp8")
    with refs as m:
        theirs = m["ds4_vq2_cuda"].vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(layer))
    torch.cuda.synchronize()
    assert torch_ref.rel_l2(ours, theirs) < 5e-3
