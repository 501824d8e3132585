"""Shared expert (dense bf16 SiLU-gated MLP, vq2_shared_expert) against the same layer in torch
fp32, its accumulate mode on top of the routed experts' output on the same stream (the two
programmatic-dependent-launch kernels must see the decode's result), and CUDA-graph capture."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _weights(H, Is, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w13 = (torch.randn(2 * Is, H, device="cuda", generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(H, Is, device="cuda", generator=g) * 0.02).bfloat16()
    return w13, w2


def _ref(x, w13, w2):
    Is = w13.shape[0] // 2
    h = x.double() @ w13.double().T
    return (torch.nn.functional.silu(h[:, :Is]) * h[:, Is:]) @ w2.double().T


@pytest.mark.parametrize("N", [1, 3, 8])
@pytest.mark.parametrize("H,Is", [(4096, 2048), (512, 256), (1024, 768)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_shared_expert_matches_torch(N, H, Is, dt):
    from vq2_vllm.kernels.shared_expert import shared_expert_fused
    w13, w2 = _weights(H, Is, N + H)
    x = torch.randn(N, H, device="cuda", generator=torch.Generator(device="cuda").manual_seed(N)).to(dt)
    out = shared_expert_fused(x, w13, w2)
    ref = _ref(x, w13, w2)
    rel = ((out.double() - ref).norm() / ref.norm()).item()
    assert rel < 1e-4, rel


def test_shared_expert_adds_onto_the_routed_output_and_captures():
    from vq2_vllm import synth
    from vq2_vllm.kernels.shared_expert import shared_expert_fused
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    E, H, I, N, k = 8, 512, 256, 3, 2
    layer = {kk: v.cuda() for kk, v in synth.make_layer(E, H, I, seed=0).items()}
    x = synth.make_tokens(N, H, seed=1).cuda()
    ids, w = synth.route_softmax_topk(x, E, k, w_std=1.0, seed=2)
    w13, w2 = _weights(H, 512, 5)
    moe = vq2_moe_fused_10b(x, ids, w, *synth.layer_args(layer)).clone()
    expect = moe.double() + _ref(x, w13, w2)
    for _ in range(3):                                   # back to back on one stream, no sync between
        out = vq2_moe_fused_10b(x, ids, w, *synth.layer_args(layer))
        shared_expert_fused(x, w13, w2, out=out)
    rel = ((out.double() - expect).norm() / expect.norm()).item()
    assert rel < 1e-4, rel
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = vq2_moe_fused_10b(x, ids, w, *synth.layer_args(layer))
        shared_expert_fused(x, w13, w2, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gout = vq2_moe_fused_10b(x, ids, w, *synth.layer_args(layer))
        shared_expert_fused(x, w13, w2, out=gout)
    gout.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert ((gout.double() - expect).norm() / expect.norm()).item() < 1e-4
