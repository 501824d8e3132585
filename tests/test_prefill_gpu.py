"""K2 prefill (tcgen05 grouped GEMM) parity through the C ABI.

fp16 operands: within 3e-2 relative L2 of the fp32 dequant+matmul oracle (the prefill bar).
fp8 operands: the reference's fp8 algorithm — within 3e-2 of the oracle's fp8 restatement
(oracle/torch_ref.moe_prefill_fp8_ref, pinned to the numpy oracle); its distance to fp32 is the
reference algorithm's own (about 7 % on these weights) and is only bounded loosely here."""
import os

import pytest
import torch

from oracle import torch_ref

pytestmark = pytest.mark.gpu
TOL = 3e-2


def _run(x, ids, tw, layer, prec, **kw):
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    return vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(layer), precision=prec, **kw)


@pytest.fixture(scope="module")
def small():
    from vq2_vllm import synth
    return synth.make_layer(8, 512, 256, seed=0, device="cuda")


@pytest.mark.parametrize("N,K", [(1, 2), (40, 2), (300, 8), (1000, 3)])
def test_small_shapes(small, N, K):
    from vq2_vllm import synth
    x = synth.make_tokens(N, 512, seed=N, device="cuda")
    ids, tw = synth.route_zipf(N, 8, K, seed=N + 1, device="cuda")
    assert torch_ref.rel_l2(_run(x, ids, tw, small, "f16"), torch_ref.moe_ref(x, ids, tw, small)) < TOL
    out8 = _run(x, ids, tw, small, "fp8")
    assert torch_ref.rel_l2(out8, torch_ref.moe_prefill_fp8_ref(x, ids, tw, small)) < TOL
    assert torch_ref.rel_l2(out8, torch_ref.moe_ref(x, ids, tw, small)) < 0.15


@pytest.fixture(scope="module")
def big():
    from vq2_vllm import synth
    return synth.make_layer(32, 4096, 2048, seed=0, device="cuda")


@pytest.mark.parametrize("prec", ["f16", "fp8"])
def test_full_width_zipf(big, prec):
    """Config-2 layer widths (H=4096, I=2048), Zipf-skewed top-8 over 32 resident experts."""
    from vq2_vllm import synth
    N = 1024
    x = synth.make_tokens(N, 4096, seed=7, device="cuda")
    ids, tw = synth.route_zipf(N, 32, 8, seed=8, device="cuda")
    out = _run(x, ids, tw, big, prec)
    ref = torch_ref.moe_ref(x, ids, tw, big) if prec == "f16" else torch_ref.moe_prefill_fp8_ref(x, ids, tw, big)
    assert torch_ref.rel_l2(out, ref) < TOL


def test_expert_window_drops_foreign_pairs(big):
    """Expert parallelism: only ids in [base, base+E) are applied; the rest are dropped."""
    from vq2_vllm import synth
    N = 256
    x = synth.make_tokens(N, 4096, seed=9, device="cuda")
    ids, tw = synth.route_uniform(N, 64, 8, seed=10, device="cuda")
    out = _run(x, ids, tw, big, "f16", expert_base=16)
    ref = torch_ref.moe_ref(x, ids, tw, big, expert_base=16)
    assert torch_ref.rel_l2(out, ref) < TOL


def test_decode_entry_routes_large_batches_to_grouped(small):
    """vq2_moe_fused_10b with more pairs than the decode kernel takes goes to the grouped path."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    N = 600
    x = synth.make_tokens(N, 512, seed=11, device="cuda")
    ids, tw = synth.route_zipf(N, 8, 2, seed=12, device="cuda")
    out = vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(small))      # VQ2_FP8_PREFILL default: fp8
    assert torch_ref.rel_l2(out, torch_ref.moe_prefill_fp8_ref(x, ids, tw, small)) < TOL
    os.environ["VQ2_FP8_PREFILL"] = "0"
    try:
        out16 = vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(small))
    finally:
        del os.environ["VQ2_FP8_PREFILL"]
    assert torch_ref.rel_l2(out16, torch_ref.moe_ref(x, ids, tw, small)) < TOL


def test_prefill_fp8_linear_in_routing_weights():
    """The fp8 prefill output is linear in the routing weights (they scale the down epilogue)."""
    from oracle import torch_ref
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    L = synth.make_layer(16, 4096, 2048, seed=71, device="cuda")
    x = synth.make_tokens(300, 4096, seed=72, device="cuda")
    ids, w1 = synth.route_zipf(300, 16, 8, seed=73, device="cuda")
    w2 = torch.rand_like(w1)
    f = lambda w: vq2_moe_grouped_wmma(x, ids, w, *synth.layer_args(L), precision="fp8")
    assert torch_ref.rel_l2(f(2.0 * w1 + 0.5 * w2), 2.0 * f(w1) + 0.5 * f(w2)) < 1e-5


@pytest.fixture(scope="module")
def config2():
    """The exact config-2 layer and routing: 8,192 tokens, 256 experts, H=4096, I=2048, Zipf(1.1)
    top-8 (65,536 pairs; Pmax 98,304 at 128-slot blocks, 768 blocks)."""
    from vq2_vllm import synth
    L = synth.make_layer(256, 4096, 2048, seed=10, device="cuda")
    x = synth.make_tokens(8192, 4096, seed=300, device="cuda")
    ids, tw = synth.route_zipf(8192, 256, 8, s=1.1, seed=301, device="cuda")
    return L, x, ids, tw


@pytest.mark.parametrize("prec", ["fp8", "f16"])
def test_config2_full_size(config2, prec):
    """The benchmark's prefill configuration end to end: multi-chunk align feeding the GEMMs,
    the heaviest Zipf experts spanning dozens of blocks, every block pair of the grid."""
    L, x, ids, tw = config2
    out = _run(x, ids, tw, L, prec)
    if prec == "fp8":
        ref = torch_ref.moe_prefill_fp8_ref(x, ids, tw, L)
    else:
        ref = torch_ref.moe_ref(x, ids, tw, L)
    assert torch_ref.rel_l2(out, ref) < TOL
    assert torch.isfinite(out).all()
