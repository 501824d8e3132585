"""Router kernel (top-k of softmax(x @ W_r)) against the same formula in torch fp32 (the routing
of the benchmark configurations). Ids must match except where two probabilities are within 1e-6
(a near-tie may order either way); weights within 1e-5 relative."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _torch_route(x, wr, k):
    p = torch.softmax(x.float() @ wr.float(), -1)
    tw, ti = torch.topk(p, k, dim=-1)
    return ti.to(torch.int32), tw, p


@pytest.mark.parametrize("N,H,E,k", [(1, 4096, 256, 8), (3, 4096, 256, 8), (16, 4096, 256, 8),
                                     (64, 4096, 256, 8), (5, 512, 16, 2), (7, 1024, 1024, 32)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_router_matches_torch(N, H, E, k, dt):
    from vq2_vllm.kernels.router import router_topk
    g = torch.Generator(device="cuda").manual_seed(N * 1000 + E)
    x = torch.randn(N, H, generator=g, device="cuda").to(dt)
    wr = (torch.randn(H, E, generator=g, device="cuda") * 0.02).bfloat16()
    ids, tw = router_topk(x, wr, k)
    ref_ids, ref_tw, p = _torch_route(x, wr, k)
    assert ids.dtype == torch.int32 and ids.shape == (N, k) and tw.shape == (N, k)
    assert torch.allclose(tw, ref_tw, rtol=1e-5, atol=1e-7)
    diff = ids != ref_ids
    if diff.any():              # only near-ties may differ: same probabilities either way
        got = p.gather(1, ids.long())
        assert torch.allclose(got, ref_tw, rtol=0, atol=1e-6)
    # probabilities are descending and ids distinct per token
    assert bool((tw[:, :-1] >= tw[:, 1:]).all())
    assert all(len(set(r.tolist())) == k for r in ids)


def test_router_feeds_decode():
    """Router output drives the decode layer exactly like the torch routing does."""
    from oracle import torch_ref
    from vq2_vllm import synth
    from vq2_vllm.kernels.router import router_topk
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    L = synth.make_layer(32, 4096, 2048, seed=5, device="cuda")
    x = synth.make_tokens(3, 4096, seed=6, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(7)
    wr = (torch.randn(4096, 32, generator=g, device="cuda") * 0.02).bfloat16()
    ids, tw = router_topk(x, wr, 8)
    out = vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(L))
    assert torch_ref.rel_l2(out, torch_ref.moe_ref(x, ids, tw, L)) < 1e-2
