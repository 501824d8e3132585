"""Generate the golden fixtures by running the REFERENCE's own Python code on the CPU.

Run where a checkout of the reference is available and name it:
``python tests/golden/make_golden.py <reference checkout>`` (or set ``VQ2_REFERENCE``); the
fixtures it writes (``tests/golden/*.npz``) are committed so the tests never need the reference at
run time.

The reference modules are imported from ``vq2_vllm/kernels`` with two shims:
  * ``vq2_kernel.py:129`` allocates a 384 MB flush buffer on "cuda" at import; that one
    allocation is redirected to the meta device during import;
  * its Triton kernels run under ``TRITON_INTERPRET=1``; ``@triton.autotune`` needs a driver, so
    each autotuned kernel is called through its ``.fn`` with one fixed config from its own list.

Fixtures:
  config0.npz   the tiny config-0 layer + routing + reference outputs (decode Triton path,
                fp32 dequant+matmul MoE, Hadamard, moe_align (torch + fast), fp8 row quant)
  align.npz     moe_align outputs of the reference for several (N, k, E, BM) cases
  pack.npz      the reference's k-means packer (pack_vq2_experts_10b, pack_vq2 with padding and
                k <= 256) on small weights, with the sample it drew (its own torch.manual_seed(0)
                draw, repeated here on the same CPU generator)

Extra arguments after the checkout name the fixtures to write (config0, align, pack); default all.
"""
import os
import sys

import numpy as np
import torch

os.environ["TRITON_INTERPRET"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VQ2_REFERENCE", "")
if not os.path.isdir(os.path.join(REF, "vq2_vllm", "kernels")):
    sys.exit("usage: make_golden.py <reference checkout> (or VQ2_REFERENCE=<checkout>)")
sys.path.insert(0, os.path.join(REF, "vq2_vllm", "kernels"))
sys.path.insert(0, os.path.join(REPO, "deepseek-v4-flash-2bit-gb10_b200"))

_real_empty = torch.empty


def _empty(*a, **kw):
    if str(kw.get("device", "")).startswith("cuda"):
        kw["device"] = "meta"
    return _real_empty(*a, **kw)


torch.empty = _empty
import vq2_kernel as rk  # noqa: E402  (reference module)
torch.empty = _real_empty
rk.DEV = "cpu"
import moe_align as rma  # noqa: E402  (reference module)
import ds4_vq2_cuda as rds  # noqa: E402  (reference module)

from vq2_vllm import synth  # noqa: E402


class _Fixed:
    """Calls an autotuned Triton kernel with one fixed config (interpreter has no autotune)."""

    def __init__(self, tuner, **cfg):
        self.fn, self.cfg = tuner.fn, cfg

    def __getitem__(self, grid):
        def run(*args, **kw):
            g = grid(self.cfg) if callable(grid) else grid
            return self.fn[g](*args, **kw, **self.cfg)
        return run


rk._vq2_gateup_silu_10b = _Fixed(rk._vq2_gateup_silu_10b, BLOCK_O=16, NG_BLK=4)
rk._vq2_down_scatter_10b = _Fixed(rk._vq2_down_scatter_10b, BLOCK_O=32, NG_BLK=2, SPLIT_K=1)


def ref_dense_moe(x, ids, w, layer):
    """The reference's fp32 dequant-plus-matmul MoE (vq2_kernel.py:63-64 dequant, :720-727 MoE)."""
    H = rk._hadamard(64)

    def dq(cb, lo, hi, sc):
        lo32, hi32 = lo.int(), hi.int()
        s = torch.arange(lo.shape[-1])
        idx = lo32 | (((hi32[..., s >> 2] >> ((s & 3) * 2)) & 3) << 8)
        R, nsub = idx.shape
        rr = cb.float()[idx.long()].reshape(R, nsub // 16, 64) * sc.float()[..., None]
        return (rr @ H.t()).reshape(R, -1)

    N, _ = x.shape
    I = layer["w13_lo"].shape[1] // 2
    out = torch.zeros(N, x.shape[1])
    for n in range(N):
        for j in range(ids.shape[1]):
            e = int(ids[n, j])
            g = dq(layer["w13_cb"], layer["w13_lo"][e], layer["w13_hi"][e], layer["w13_sc"][e]) @ x[n].float()
            a = torch.nn.functional.silu(g[:I]) * g[I:]
            out[n] += float(w[n, j]) * (dq(layer["w2_cb"], layer["w2_lo"][e], layer["w2_hi"][e], layer["w2_sc"][e]) @ a)
    return out


def draw_sample(nvec, k):
    """The reference's sample draw (vq2_kernel.py:50-52) on the CPU generator."""
    torch.manual_seed(0)
    si = torch.randint(0, nvec, (min(nvec, 200000),))
    return si, torch.randperm(si.shape[0])[:k]


def main_pack():
    g = torch.Generator().manual_seed(11)
    W3 = torch.randn(2, 48, 256, generator=g) * 0.02
    W3[:, :, 5] *= 8.0                                    # an outlier column, as trained weights have
    C, lo, hi, sc, dq = rk.pack_vq2_experts_10b(W3, k=1024, iters=12)
    si, init = draw_sample(2 * 48 * 4 * 16, 1024)
    W2 = torch.randn(40, 200, generator=g).to(torch.bfloat16)
    C2, idx2, sc2, dq2, inn2, pad2 = rk.pack_vq2(W2, k=256, iters=6)
    si2, init2 = draw_sample(40 * 4 * 16, 256)
    print(f"pack: 10b case rel-L2 {((dq - W3).norm() / W3.norm()).item():.3f}, padded case "
          f"{((dq2 - W2.float()).norm() / W2.float().norm()).item():.3f} (inn {inn2}, pad {pad2}, idx {idx2.dtype})")
    np.savez_compressed(
        os.path.join(HERE, "pack.npz"),
        a_W=W3.numpy(), a_C=C.numpy(), a_lo=lo.numpy(), a_hi=hi.numpy(), a_sc=sc.numpy(), a_dq=dq.numpy(),
        a_si=si.numpy(), a_init=init.numpy(), a_meta=np.array([1024, 12]),
        b_W_bf16_bits=W2.view(torch.int16).numpy(), b_C=C2.numpy(), b_idx=idx2.numpy(), b_sc=sc2.numpy(),
        b_dq=dq2.numpy(), b_si=si2.numpy(), b_init=init2.numpy(), b_meta=np.array([256, 6, inn2, pad2]))
    print("wrote", os.path.join(HERE, "pack.npz"))


def main():
    which = set(sys.argv[2:]) or {"config0", "align", "pack"}
    if "pack" in which:
        main_pack()
    if not which & {"config0", "align"}:
        return
    E, H, I, N, K = 8, 512, 256, 4, 2
    layer = synth.make_layer(E, H, I, seed=0)
    x = synth.make_tokens(N, H, seed=1)
    ids, tw = synth.route_softmax_topk(x, E, K, w_std=1.0, seed=2)
    # the packer must equal the reference's _pack10 on the same indices
    gen = torch.Generator().manual_seed(3)
    idx = torch.randint(0, 1024, (16, 64), generator=gen)
    lo_r, hi_r = rk._pack10(idx.int())
    lo_s, hi_s = synth.pack10(idx)
    assert torch.equal(lo_r, lo_s) and torch.equal(hi_r, hi_s)
    args = synth.layer_args(layer)
    dec = rk.vq2_moe_fused_10b(x, ids, tw, *args, group=64)
    dense = ref_dense_moe(x, ids, tw, layer)
    had = rk.had_act_batch(x.float(), 64)
    st, ss, val, be, nb = rma._moe_align_torch(ids, E, 4)
    fst, fss, fval, fbe, fnb = rma.moe_align_fast(ids, E, 4)
    xq, inv = rds.quant_fp8_rows(had.contiguous())
    rel = ((dec - dense).norm() / dense.norm()).item()
    print(f"config0: reference decode (bf16 Triton) vs reference fp32 dense MoE rel-L2 = {rel:.3e}")
    np.savez_compressed(
        os.path.join(HERE, "config0.npz"),
        x_bf16_bits=x.view(torch.int16).numpy(), topk_ids=ids.numpy(), topk_w=tw.numpy(),
        **{k: (v.view(torch.int16).numpy() if v.dtype == torch.float16 else v.numpy()) for k, v in layer.items()},
        pack_idx=idx.numpy(), pack_lo=lo_r.numpy(), pack_hi=hi_r.numpy(),
        ref_decode=dec.numpy(), ref_dense=dense.numpy(), ref_had=had.numpy(),
        ref_fp8=xq.float().numpy(), ref_fp8_inv=inv.numpy(),
        align_st=st.numpy(), align_ss=ss.numpy(), align_val=val.numpy(), align_be=be.numpy(),
        fast_st=fst.numpy(), fast_ss=fss.numpy(), fast_val=fval.numpy(), fast_be=fbe.numpy())

    cases = {}
    for ci, (n, k, e, bm, kind) in enumerate([(5, 3, 8, 4, "topk"), (4, 2, 8, 64, "topk"), (37, 8, 256, 64, "zipf"),
                                              (300, 8, 64, 64, "zipf"), (1, 8, 256, 64, "topk"),
                                              (129, 6, 16, 16, "uniform"), (1000, 8, 256, 128, "zipf")]):
        torch.manual_seed(ci)
        if kind == "topk":
            tid = torch.topk(torch.randn(n, e), k, 1).indices.int()
        elif kind == "zipf":
            tid, _ = synth.route_zipf(n, e, k, seed=ci)
        else:
            tid, _ = synth.route_uniform(n, e, k, seed=ci)
        out = rma._moe_align_torch(tid, e, bm)
        cases[f"c{ci}_ids"] = tid.numpy()
        cases[f"c{ci}_meta"] = np.array([e, bm, out[4]])
        for nm, t in zip(("st", "ss", "val", "be"), out[:4]):
            cases[f"c{ci}_{nm}"] = t.numpy()
    np.savez_compressed(os.path.join(HERE, "align.npz"), **cases)
    print("wrote", os.path.join(HERE, "config0.npz"), os.path.join(HERE, "align.npz"))


if __name__ == "__main__":
    main()
