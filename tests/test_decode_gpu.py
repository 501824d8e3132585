"""K1 decode kernel parity (through the C ABI) against the fp32 dequant+matmul oracle.
Tolerance: 1e-2 relative L2 (the decode bar for this path)."""
import pytest
import torch

from gpu_util import args, config0_cuda
from oracle import torch_ref

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _moe():
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    return vq2_moe_fused_10b


def test_config0_golden():
    z, L, x, ids, tw = config0_cuda()
    out = _moe()(x, ids, tw, *args(L))
    torch.cuda.synchronize()
    ref = torch.from_numpy(z["ref_dense"]).cuda()
    assert out.dtype == torch.float32 and out.shape == ref.shape
    assert torch_ref.rel_l2(out, ref) < TOL
    # and close to the reference's own bf16 decode kernel output
    assert torch_ref.rel_l2(out, torch.from_numpy(z["ref_decode"]).cuda()) < TOL


def test_int64_ids_and_repeat_calls():
    z, L, x, ids, tw = config0_cuda()
    a = _moe()(x, ids.long(), tw, *args(L))
    b = _moe()(x, ids, tw, *args(L))
    ref = torch.from_numpy(z["ref_dense"]).cuda()
    assert torch_ref.rel_l2(a, ref) < TOL and torch_ref.rel_l2(b, ref) < TOL


@pytest.fixture(scope="module")
def big_layer():
    from vq2_vllm import synth
    return synth.make_layer(256, 4096, 2048, seed=0, device="cuda")


@pytest.mark.parametrize("N", [1, 3, 16])
def test_config1_full_size(big_layer, N):
    from vq2_vllm import synth
    x = synth.make_tokens(N, 4096, seed=1, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=2)
    out = _moe()(x, ids, tw, *synth.layer_args(big_layer))
    ref = torch_ref.moe_ref(x, ids, tw, big_layer)
    assert torch_ref.rel_l2(out, ref) < TOL


def test_shared_experts_many_tokens(big_layer):
    """Many tokens on the same few experts (units of more than one token group)."""
    from vq2_vllm import synth
    N = 24
    x = synth.make_tokens(N, 4096, seed=5, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(7)
    ids = torch.stack([torch.randperm(12, generator=g, device="cuda")[:8] for _ in range(N)]).int()
    tw = torch.rand(N, 8, device="cuda", generator=g)
    out = _moe()(x, ids, tw, *synth.layer_args(big_layer))
    assert torch_ref.rel_l2(out, torch_ref.moe_ref(x, ids, tw, big_layer)) < TOL


def test_max_pairs_and_expert_base(big_layer):
    """N*k = 512 (the decode limit) with a local expert window (expert parallelism)."""
    from vq2_vllm import synth
    N = 64
    x = synth.make_tokens(N, 4096, seed=3, device="cuda")
    ids, tw = synth.route_uniform(N, 256, 8, seed=4, device="cuda")
    sub = {k: (v[64:128] if v.dim() == 3 else v) for k, v in big_layer.items()}
    out = _moe()(x, ids, tw, *synth.layer_args(sub), expert_base=64)
    ref = torch_ref.moe_ref(x, ids, tw, sub, expert_base=64)
    assert torch_ref.rel_l2(out, ref) < TOL
    none = _moe()(x, ids * 0 + 255, tw, *synth.layer_args(sub), expert_base=64)
    assert torch.count_nonzero(none) == 0


@pytest.mark.parametrize("H,I", [(1024, 4096), (4096, 4096), (2048, 1024)])
def test_shapes_k_slices(H, I):
    """One and two K-slices on either side (I = 4096 runs 16-row down stages)."""
    from vq2_vllm import synth
    L = synth.make_layer(16, H, I, seed=11, device="cuda")
    x = synth.make_tokens(3, H, seed=12, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 16, 8, w_std=0.02, seed=13)
    out = _moe()(x, ids, tw, *synth.layer_args(L))
    assert torch_ref.rel_l2(out, torch_ref.moe_ref(x, ids, tw, L)) < TOL


def test_many_calls_back_to_back(big_layer):
    """Back-to-back calls on one stream (the chained kernel pair, queued ahead of the GPU)."""
    from vq2_vllm import synth
    x = synth.make_tokens(2, 4096, seed=21, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=22)
    ref = torch_ref.moe_ref(x, ids, tw, big_layer)
    outs = [_moe()(x, ids, tw, *synth.layer_args(big_layer)) for _ in range(50)]
    torch.cuda.synchronize()
    for o in outs[::7]:
        assert torch_ref.rel_l2(o, ref) < TOL


def test_properties_full_size(big_layer):
    """Size-independent properties at the full config-1 layer: the output is linear in the
    routing weights and invariant to the order of a token's top-k slots."""
    from vq2_vllm import synth
    N = 3
    x = synth.make_tokens(N, 4096, seed=61, device="cuda")
    ids, w1 = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=62)
    w2 = torch.rand(N, 8, device="cuda", generator=torch.Generator(device="cuda").manual_seed(63))
    f = lambda i, w: _moe()(x, i, w, *synth.layer_args(big_layer))
    lhs = f(ids, 0.7 * w1 - 1.3 * w2)
    rhs = 0.7 * f(ids, w1) - 1.3 * f(ids, w2)
    assert torch_ref.rel_l2(lhs, rhs) < 1e-5
    perm = torch.stack([torch.randperm(8, generator=torch.Generator().manual_seed(64 + n)) for n in range(N)]).cuda()
    got = f(ids.gather(1, perm), w1.gather(1, perm))
    assert torch_ref.rel_l2(got, f(ids, w1)) < 1e-5


def _wide_range_layer(E, seed):
    """A config-1 layer with real-model dynamic range: a heavy-tailed codebook (2 % of the entries
    x25, max |C| about 60x the typical entry) and group scales spanning 2^-8 .. 2^4."""
    from vq2_vllm import synth
    L = synth.make_layer(E, 4096, 2048, seed=seed, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    for key in ("w13_cb", "w2_cb"):
        cb = L[key].float()
        tail = torch.rand(cb.shape, generator=g, device="cuda") < 0.02
        L[key] = torch.where(tail, cb * 25.0, cb).half()
    for key in ("w13_sc", "w2_sc"):
        ex = torch.randint(-8, 5, L[key].shape, generator=g, device="cuda").float()
        L[key] = (torch.exp2(ex) * (0.75 + 0.5 * torch.rand(L[key].shape, generator=g, device="cuda"))).half()
    return L


@pytest.mark.parametrize("N,outlier", [(1, 50.0), (3, 100.0), (8, 100.0)])
def test_wide_dynamic_range(N, outlier):
    """Outlier activation channels (a few at 50-100 sigma, as real DS4 activations have), a
    heavy-tailed codebook and scales over 2^-8..2^4 at the full config-1 width. The decode keeps
    group partial sums in fp16 (power-of-two group scaling); it must stay within 1e-2 of the
    fp32 oracle and no further from it than the reference's own decode algorithm (bf16
    activations and intermediate, oracle/torch_ref.moe_decode_bf16_ref)."""
    from vq2_vllm import synth
    L = _wide_range_layer(64, seed=40 + N)
    g = torch.Generator(device="cuda").manual_seed(50 + N)
    x = torch.randn(N, 4096, generator=g, device="cuda")
    ch = torch.randperm(4096, generator=g, device="cuda")[:6]
    sign = torch.where(torch.rand(N, 6, generator=g, device="cuda") < 0.5, -1.0, 1.0)
    x[:, ch] = sign * outlier * (0.5 + 0.5 * torch.rand(N, 6, generator=g, device="cuda"))
    x = x.bfloat16()
    ids, tw = synth.route_softmax_topk(x, 64, 8, w_std=0.02, seed=60 + N)
    out = _moe()(x, ids, tw, *synth.layer_args(L))
    ref = torch_ref.moe_ref(x, ids, tw, L)
    ours = torch_ref.rel_l2(out, ref)
    theirs = torch_ref.rel_l2(torch_ref.moe_decode_bf16_ref(x, ids, tw, L), ref)
    assert ours < TOL, f"rel-L2 {ours:.3e} against fp32"
    assert ours <= theirs * 1.05 + 1e-5, f"ours {ours:.3e} vs the reference algorithm's {theirs:.3e}"


@pytest.mark.parametrize("N,ids64", [(1, False), (3, True)])
def test_host_buffer_entry_matches_device_entry(big_layer, N, ids64):
    """vq2_decode_host (inputs and result in page-locked host memory, one library call per step)
    gives the device entry's result; two steps in a row reuse the same device staging."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b_host
    for step in range(2):
        x = synth.make_tokens(N, 4096, seed=80 + step, device="cuda")
        ids, tw = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=90 + step)
        if ids64:
            ids = ids.long()
        want = _moe()(x, ids, tw, *synth.layer_args(big_layer))
        xh, ih, wh = x.cpu().pin_memory(), ids.cpu().pin_memory(), tw.cpu().pin_memory()
        got = vq2_moe_fused_10b_host(xh, ih, wh, *synth.layer_args(big_layer))
        torch.cuda.synchronize()
        assert not got.is_cuda and got.dtype == torch.float32
        assert torch_ref.rel_l2(got, want.cpu()) < 1e-5


def test_host_decode_session_matches_device_entry(big_layer):
    """HostDecodeSession (per step one library call: upload on a copy stream, the decode kernels,
    download on a second copy stream) gives the device entry's result, over more steps than it has
    slots (slot reuse is ordered by the slot's events)."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.vq2_kernel import HostDecodeSession
    sess = HostDecodeSession(*synth.layer_args(big_layer), N=2, k=8, slots=2)
    outs = []
    for step in range(5):
        x = synth.make_tokens(2, 4096, seed=300 + step, device="cuda")
        ids, tw = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=310 + step)
        want = _moe()(x, ids, tw, *synth.layer_args(big_layer)).cpu()
        sl, got = sess.step(x.cpu(), ids.cpu(), tw.cpu())
        sess.synchronize()
        assert sess.done(sl)
        assert torch_ref.rel_l2(got, want) < 1e-5, step
        outs.append(got.clone())
    assert not torch.equal(outs[0], outs[1])
