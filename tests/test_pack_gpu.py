"""VQ packer on the GPU (vq2_pack_gather / vq2_kmeans / vq2_pack_assign through the mirrored
pack_vq2 API): bit-exact against the oracle on the reference's own fixtures and sample, the
mirror's shapes and dtypes, size-independent properties at a full expert-tensor size, and a
pack -> decode round trip that runs the packed planes through the decode kernels."""
import numpy as np
import pytest
import torch

from golden_io import load_pack
from oracle import vq2_oracle as O

pytestmark = pytest.mark.gpu


def _pack(W, si, init, iters):
    from vq2_vllm.kernels.vq2_pack import pack_from_sample
    r = pack_from_sample(torch.from_numpy(W).cuda(), torch.from_numpy(si).cuda(), torch.from_numpy(init).cuda(),
                         iters, planes=True, ids=True, dq=True)
    return {k: v.cpu().numpy() for k, v in r.items()}


@pytest.mark.parametrize("case", ["a", "b"])
def test_pack_bit_exact_vs_oracle_on_reference_sample(case):
    z = load_pack()
    it = int(z[f"{case}_meta"][1])
    W = z["a_W"].reshape(-1, 256) if case == "a" else z["b_W"]
    r = _pack(W, z[f"{case}_si"], z[f"{case}_init"], it)
    C, idx, s, dq = O.pack_from_sample(W, z[f"{case}_si"], z[f"{case}_init"], it)
    assert np.array_equal(r["C"], C)
    assert np.array_equal(r["idx"].astype(np.int64), idx)
    assert np.array_equal(r["scale"], s)
    lo, hi = O.pack10(idx)
    assert np.array_equal(r["lo"], lo) and np.array_equal(r["hi"], hi)
    assert np.array_equal(r["dq"], dq)
    ref_idx = O.unpack10(z["a_lo"], z["a_hi"]).reshape(idx.shape) if case == "a" else z["b_idx"]
    assert np.array_equal(r["idx"].astype(np.int64), ref_idx.astype(np.int64))   # the reference's own ids


def test_pack_bf16_input_matches_f32():
    z = load_pack()
    W = torch.from_numpy(z["b_W"]).cuda()
    from vq2_vllm.kernels.vq2_pack import pack_from_sample
    si, init = torch.from_numpy(z["b_si"]).cuda(), torch.from_numpy(z["b_init"]).cuda()
    a = pack_from_sample(W, si, init, 6)
    b = pack_from_sample(W.to(torch.bfloat16), si, init, 6)      # b_W holds bf16 values exactly
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_pack_api_mirror_shapes():
    from vq2_vllm.kernels.vq2_kernel import pack_vq2, pack_vq2_experts, pack_vq2_experts_10b
    g = torch.Generator(device="cuda").manual_seed(5)
    W = torch.randn(24, 200, device="cuda", generator=g)
    C, idx, sc, dq, inn, pad = pack_vq2(W, k=256, iters=3)
    assert C.shape == (256, 4) and idx.dtype == torch.uint8 and idx.shape == (24, 64)
    assert sc.shape == (24, 4) and dq.shape == (24, 200) and (inn, pad) == (200, 56)
    W3 = torch.randn(3, 32, 128, device="cuda", generator=g)
    C, idx, sc, dq = pack_vq2_experts(W3, k=1024, iters=3)
    assert idx.dtype == torch.int16 and idx.shape == (3, 32, 32) and sc.shape == (3, 32, 2) and dq.shape == W3.shape
    C2, lo, hi, sc2, dq2 = pack_vq2_experts_10b(W3, k=1024, iters=3)    # same seed-0 draw -> same result
    lo_r, hi_r = O.pack10(idx.cpu().numpy())
    assert torch.equal(C, C2) and torch.equal(sc, sc2) and torch.equal(dq, dq2)
    assert np.array_equal(lo.cpu().numpy(), lo_r) and np.array_equal(hi.cpu().numpy(), hi_r)
    with pytest.raises(ValueError):
        pack_vq2(W, vdim=8)


def test_pack_properties_full_size():
    """An 8-expert gate/up tensor at the benchmark's shape (8 x 4096 x 4096 bf16): every sampled
    sub-vector's id is its nearest centroid (float64 check), dq is (C[id] * s) through the group
    Hadamard, the planes encode the ids, k-means lowered the sample objective, and the
    reconstruction error is that of a 2-bit code."""
    from vq2_vllm.kernels.vq2_pack import draw_sample, pack_from_sample
    g = torch.Generator(device="cuda").manual_seed(7)
    W = (torch.randn(8 * 4096, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    rows, D = W.shape
    nvec = rows * D // 4
    si, init = draw_sample(nvec, 1024, W.device)
    r = pack_from_sample(W, si, init, 12)
    C, idx, s = r["C"].double(), r["idx"].long().reshape(-1), r["scale"].reshape(-1)
    # the ids against the planes
    lo, hi = r["lo"].reshape(-1).long(), r["hi"].reshape(-1).long()
    pos = torch.randint(0, nvec, (1 << 14,), device="cuda", generator=g)
    assert torch.equal(idx[pos], lo[pos] | (((hi[pos >> 2] >> ((pos & 3) * 2)) & 3) << 8))
    # nearest centroid, from the rotated and normalised sub-vectors recomputed in float64
    H = torch.from_numpy(O.hadamard(64)).double().cuda()
    gid = pos >> 4
    grp = W.view(-1, 64)[gid].double() @ H
    sg = grp.abs().amax(1).clamp_min(1e-8)
    j = (pos & 15)
    vec = (grp / sg[:, None]).view(-1, 16, 4)[torch.arange(pos.numel(), device="cuda"), j]
    d = ((vec[:, None, :] - C[None]) ** 2).sum(-1)
    chosen = d.gather(1, idx[pos][:, None])[:, 0]
    assert torch.all(chosen <= d.min(1).values + 1e-6)
    assert torch.allclose(s[gid].double(), sg, rtol=1e-6)
    # dq = (C[id] * s) @ H per group
    rows_chk = torch.randint(0, rows, (256,), device="cuda", generator=g)
    ids_r = r["idx"][rows_chk].long()
    rec = (C[ids_r].reshape(256, -1, 64) * r["scale"][rows_chk].double()[..., None]) @ H
    assert torch.allclose(r["dq"][rows_chk].double(), rec.reshape(256, -1), atol=1e-6)
    # k-means lowered the objective on its sample
    samp = torch.empty(si.numel(), 4, device="cuda")
    from vq2_vllm import _lib
    _lib.check(_lib.lib().vq2_pack_gather(W.data_ptr(), 0, rows, D, si.data_ptr(), si.numel(), samp.data_ptr(),
                                          _lib.stream_ptr()), "gather")
    def obj(cb):
        return sum(((samp[i:i + 8192].double()[:, None, :] - cb[None]) ** 2).sum(-1).min(1).values.sum().item()
                   for i in range(0, samp.shape[0], 8192))
    assert obj(C) < 0.99 * obj(samp.double()[init])          # Lloyd iterations never raise it
    rel = ((r["dq"] - W.float()).norm() / W.float().norm()).item()
    assert 0.08 < rel < 0.35, rel


def test_pack_then_decode_round_trip():
    """Weights packed by the GPU packer, run through the decode kernels, reproduce the dense MoE on
    the packer's own reconstruction (dq) to the fp16 rounding of codebook and scales."""
    from vq2_vllm.kernels.vq2_kernel import pack_vq2_experts_10b, vq2_moe_fused_10b
    E, H, I, N, k = 4, 512, 256, 3, 2
    g = torch.Generator(device="cuda").manual_seed(9)
    W13 = torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.05
    W2 = torch.randn(E, H, I, device="cuda", generator=g) * 0.05
    Cg, lg, hg, sg, dq13 = pack_vq2_experts_10b(W13, iters=6)
    Cd, ld, hd, sd, dq2 = pack_vq2_experts_10b(W2, iters=6)
    x = torch.randn(N, H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(N)]).int()
    w = torch.rand(N, k, device="cuda", generator=g)
    out = vq2_moe_fused_10b(x, ids, w, Cg, lg, hg, sg, Cd, ld, hd, sd)
    ref = torch.zeros(N, H, device="cuda", dtype=torch.float64)
    for n in range(N):
        for j in range(k):
            e = int(ids[n, j])
            gu = dq13[e].double() @ x[n].double()
            a = torch.nn.functional.silu(gu[:I]) * gu[I:]
            ref[n] += float(w[n, j]) * (dq2[e].double() @ a)
    rel = ((out.double() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel
