"""Shared expert (dense bf16 SiLU-gated MLP, vq2_shared_expert) against the same layer in torch
fp32, its accumulate mode on top of the routed experts' output on the same stream (the two
programmatic-dependent-launch kernels must see the decode's result), CUDA-graph capture, and the
co-scheduled routed + shared call (vq2_decode_with_shared) against the two run in sequence."""
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


@pytest.mark.parametrize("N", [1, 3])
@pytest.mark.parametrize("shared_sms", [0, 8, 40])
def test_routed_plus_shared_coscheduled(N, shared_sms):
    """vq2_decode_with_shared (routed and shared kernels concurrently on disjoint SM partitions)
    equals the routed decode plus the shared expert run one after the other, at config-1 size,
    over consecutive calls and from a captured CUDA graph."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.shared_expert import moe_with_shared_expert, shared_expert_fused
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    E, H, I, k = 256, 4096, 2048, 8
    layer = {kk: v.cuda() for kk, v in synth.make_layer(E, H, I, seed=7).items()}
    w13, w2 = _weights(H, 2048, 11)
    for rep in range(2):
        x = synth.make_tokens(N, H, seed=20 + rep).cuda()
        ids, w = synth.route_softmax_topk(x, E, k, w_std=1.0, seed=30 + rep)
        expect = vq2_moe_fused_10b(x, ids, w, *synth.layer_args(layer))
        shared_expert_fused(x, w13, w2, out=expect)
        out = moe_with_shared_expert(x, ids, w, *synth.layer_args(layer), w13, w2, shared_sms=shared_sms)
        out2 = moe_with_shared_expert(x, ids, w, *synth.layer_args(layer), w13, w2, shared_sms=shared_sms)
        torch.cuda.synchronize()
        for o in (out, out2):
            rel = ((o.double() - expect.double()).norm() / expect.double().norm()).item()
            assert rel < 1e-5, rel
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe_with_shared_expert(x, ids, w, *synth.layer_args(layer), w13, w2, shared_sms=shared_sms)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gout = moe_with_shared_expert(x, ids, w, *synth.layer_args(layer), w13, w2, shared_sms=shared_sms)
    gout.fill_(1e9)
    graph.replay()
    torch.cuda.synchronize()
    assert ((gout.double() - expect.double()).norm() / expect.double().norm()).item() < 1e-5


def test_routed_plus_shared_rejects_bad_partition():
    from vq2_vllm import synth
    from vq2_vllm.kernels.shared_expert import moe_with_shared_expert
    layer = {kk: v.cuda() for kk, v in synth.make_layer(8, 512, 256, seed=0).items()}
    x = synth.make_tokens(1, 512, seed=1).cuda()
    ids, w = synth.route_softmax_topk(x, 8, 2, w_std=1.0, seed=2)
    w13, w2 = _weights(512, 256, 3)
    with pytest.raises(RuntimeError):
        moe_with_shared_expert(x, ids, w, *synth.layer_args(layer), w13, w2, shared_sms=100000)
