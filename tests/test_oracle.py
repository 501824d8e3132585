"""The CPU oracle pinned against the reference's own outputs (golden fixtures)."""
import numpy as np
import torch

from golden_io import load_align, load_config0
from oracle import vq2_oracle as O


def _w(layer, p):
    return tuple(layer[f"{p}_{s}"] for s in ("cb", "lo", "hi", "sc"))


def test_pack10_matches_reference():
    z, _, _ = load_config0()
    lo, hi = O.pack10(z["pack_idx"])
    assert np.array_equal(lo, z["pack_lo"]) and np.array_equal(hi, z["pack_hi"])
    assert np.array_equal(O.unpack10(lo, hi), z["pack_idx"])


def test_hadamard_matches_reference():
    z, _, x = load_config0()
    np.testing.assert_allclose(O.had_act_batch(x), z["ref_had"], rtol=0, atol=1e-5)
    h = O.hadamard(64)
    np.testing.assert_allclose(h @ h, np.eye(64), atol=1e-6)


def test_dense_moe_matches_reference():
    z, layer, x = load_config0()
    out = O.moe_ref(x, z["topk_ids"], z["topk_w"], _w(layer, "w13"), _w(layer, "w2"))
    assert O.rel_l2(out, z["ref_dense"]) < 1e-5
    # the reference's own bf16 Triton decode path sits within the decode tolerance of it
    assert O.rel_l2(z["ref_decode"], out) < 1e-2


def test_align_matches_reference_torch_and_fast():
    z, _, _ = load_config0()
    st, ss, val, be, nb = O.moe_align(z["topk_ids"], 8, 4)
    for pre in ("align", "fast"):
        assert np.array_equal(st, z[f"{pre}_st"]) and np.array_equal(ss, z[f"{pre}_ss"])
        assert np.array_equal(val, z[f"{pre}_val"]) and np.array_equal(be, z[f"{pre}_be"])
    for ids, E, BM, nblk, rst, rss, rval, rbe in load_align():
        st, ss, val, be, nb = O.moe_align(ids, E, BM)
        assert nb == nblk
        assert np.array_equal(st, rst) and np.array_equal(ss, rss)
        assert np.array_equal(val, rval) and np.array_equal(be, rbe)


def test_e4m3_rounding_matches_torch():
    g = torch.Generator().manual_seed(0)
    v = torch.cat([torch.randn(200000, generator=g) * s for s in (1e-3, 1e-2, 1.0, 60.0)]).clamp(-448, 448)
    v = torch.cat([v, torch.tensor([0.0, -0.0, 448.0, -448.0, 2 ** -9, 2 ** -10, 3 * 2 ** -11, 0.0146484375])])
    ref = v.to(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(O.to_e4m3(v.numpy()), ref)


def test_quant_fp8_rows_matches_reference():
    z, _, _ = load_config0()
    q, inv = O.quant_fp8_rows(z["ref_had"])
    np.testing.assert_array_equal(inv, z["ref_fp8_inv"])
    # The fixture comes from Triton's CPU interpreter, whose fp32->e4m3 cast loses the carry when
    # rounding up crosses into the next binade (e.g. 125.5 -> 64 instead of 128). Every other
    # element must match bit-exactly; the carry cases must be exactly that defect.
    ref = z["ref_fp8"]
    bad = q != ref
    assert bad.mean() < 0.05
    np.testing.assert_array_equal(ref[bad] * 2, q[bad])
    m = np.abs(q[bad])
    assert np.all(np.log2(m) == np.round(np.log2(m)))


def test_fp8_prefill_emulation_sane():
    z, layer, x = load_config0()
    ref = O.moe_ref(x, z["topk_ids"], z["topk_w"], _w(layer, "w13"), _w(layer, "w2"))
    f8 = O.moe_prefill_fp8_ref(x, z["topk_ids"], z["topk_w"], _w(layer, "w13"), _w(layer, "w2"))
    # the reference's fp8 algorithm is a few percent away from fp32 on these weights
    assert 1e-3 < O.rel_l2(f8, ref) < 0.15


def test_torch_ref_matches_numpy_oracle():
    from oracle import torch_ref
    z, layer, x = load_config0()
    tl = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in layer.items()}
    out = torch_ref.moe_ref(torch.from_numpy(x), torch.from_numpy(z["topk_ids"]), torch.from_numpy(z["topk_w"]), tl)
    assert O.rel_l2(out.numpy(), z["ref_dense"]) < 1e-5


def test_torch_fp8_prefill_matches_numpy_oracle():
    from oracle import torch_ref
    z, layer, x = load_config0()
    tl = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in layer.items()}
    a = torch_ref.moe_prefill_fp8_ref(torch.from_numpy(x), torch.from_numpy(z["topk_ids"]),
                                      torch.from_numpy(z["topk_w"]), tl)
    b = O.moe_prefill_fp8_ref(x, z["topk_ids"], z["topk_w"], _w(layer, "w13"), _w(layer, "w2"))
    assert O.rel_l2(a.numpy(), b) < 2e-3


def test_packer_matches_reference():
    """The oracle's packer restatement (exact-order butterfly rotation, fixed-point centroid sums)
    against the reference's pack_vq2_experts_10b / pack_vq2 run on the same weights and sample:
    identical assignments; codebook, scales and reconstruction equal to fp32 rounding."""
    from golden_io import load_pack
    z = load_pack()
    W = z["a_W"].reshape(-1, 256)
    C, idx, s, dq = O.pack_from_sample(W, z["a_si"], z["a_init"], int(z["a_meta"][1]))
    assert np.array_equal(idx, O.unpack10(z["a_lo"], z["a_hi"]).reshape(idx.shape))
    assert np.abs(C - z["a_C"]).max() <= 2e-6
    assert np.abs(s - z["a_sc"].reshape(s.shape)).max() <= 2e-6 * np.abs(s).max()
    assert O.rel_l2(dq, z["a_dq"].reshape(W.shape)) <= 1e-5
    k, it, inn, pad = (int(v) for v in z["b_meta"])
    C2, idx2, s2, dq2 = O.pack_from_sample(z["b_W"], z["b_si"], z["b_init"], it)
    assert (inn, pad) == (200, 56) and C2.shape == (k, 4) and dq2.shape == (40, 200)
    assert np.array_equal(idx2, z["b_idx"].astype(np.int64))
    assert np.abs(C2 - z["b_C"]).max() <= 2e-6
    assert np.abs(s2 - z["b_sc"]).max() <= 2e-6 * np.abs(s2).max()
    assert O.rel_l2(dq2, z["b_dq"]) <= 1e-5


def test_packer_butterfly_is_the_hadamard():
    x = np.random.default_rng(0).standard_normal((9, 64)).astype(np.float32)
    assert np.allclose(O.fwht64_f32(x), x @ O.hadamard(64), atol=2e-6)
    assert np.allclose(O.fwht64_f32(O.fwht64_f32(x)), x, atol=2e-6)
