"""fp32 torch restatement of the oracle's dense MoE (TEST INFRASTRUCTURE ONLY).

Same maths as ``oracle.vq2_oracle.moe_ref`` (reference vq2_vllm/kernels/vq2_kernel.py:63-64
dequant, :720-727 MoE), written with torch so the full-size (config 1) parity tests can run it on
the GPU box. It is cross-checked against the numpy oracle on the CPU (tests/test_oracle.py).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use it.
"""
from __future__ import annotations

import torch


def _had(n, device):
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / n ** 0.5).float().to(device)


def had_rows(x):
    *b, n = x.shape
    return (x.float().reshape(*b, n // 64, 64) @ _had(64, x.device)).reshape(*b, n)


def dequant_rot(cb, lo, hi, sc):
    """recon_rot = C[id] * scale per 64-group (reference vq2_kernel.py:63); lo [R,nsub]."""
    lo32 = lo.int()
    s = torch.arange(lo.shape[-1], device=lo.device)
    hb = hi.int()[..., s >> 2]
    ids = lo32 | (((hb >> ((s & 3) * 2)) & 3) << 8)
    w = cb.float()[ids.long()]                                   # [R, nsub, 4]
    R, nsub = ids.shape
    return (w.reshape(R, nsub // 16, 64) * sc.float()[..., None]).reshape(R, nsub * 4)


def moe_ref(x, topk_ids, topk_w, layer, expert_base=0, E=None):
    """fp32 dense MoE over the experts [expert_base, expert_base+E) held in ``layer``."""
    x = x.float()
    N, H = x.shape
    E = layer["w13_lo"].shape[0] if E is None else E
    I = layer["w13_lo"].shape[1] // 2
    ids = topk_ids.long() - expert_base
    out = torch.zeros(N, H, device=x.device)
    xh = had_rows(x)
    for e in torch.unique(ids).tolist():
        if e < 0 or e >= E:
            continue
        n_idx, j_idx = torch.nonzero(ids == e, as_tuple=True)
        wgu = dequant_rot(layer["w13_cb"], layer["w13_lo"][e], layer["w13_hi"][e], layer["w13_sc"][e])
        wdn = dequant_rot(layer["w2_cb"], layer["w2_lo"][e], layer["w2_hi"][e], layer["w2_sc"][e])
        g = xh[n_idx] @ wgu.T
        a = torch.nn.functional.silu(g[:, :I]) * g[:, I:]
        d = had_rows(a) @ wdn.T
        out.index_add_(0, n_idx, d * topk_w.float()[n_idx, j_idx, None])
    return out


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def quant_fp8_rows(x):
    """s = 448 / max(amax, 1e-6); q = e4m3(x * s); inv = 1 / s per row
    (reference vq2_vllm/kernels/ds4_vq2_cuda.py:8-23). Returns (q as fp32 values, inv)."""
    amax = x.abs().amax(-1)
    s = 448.0 / amax.clamp_min(1e-6)
    q = (x * s[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    return q, 1.0 / s


def moe_prefill_fp8_ref(x, topk_ids, topk_w, layer, expert_base=0, E=None):
    """The reference's fp8 prefill algorithm (vq2_vllm/kernels/ds4_vq2_cuda.py:72-111): per-token
    fp8 activations, weights decoded as e4m3(sat(C[id] * sc)) (vq2_grouped.cu:434-446),
    silu(g*inv)*(u*inv) (vq2_grouped.cu:255-264), per-row fp8 of had(inter), down weighted by
    w * inv_vb. fp32 sums. Same maths as oracle.vq2_oracle.moe_prefill_fp8_ref."""
    x = x.float()
    N, H = x.shape
    E = layer["w13_lo"].shape[0] if E is None else E
    I = layer["w13_lo"].shape[1] // 2
    ids = topk_ids.long() - expert_base
    xq, inv_x = quant_fp8_rows(had_rows(x))
    out = torch.zeros(N, H, device=x.device)
    q8 = lambda w: w.clamp(-448, 448).to(torch.float8_e4m3fn).float()
    for e in torch.unique(ids).tolist():
        if e < 0 or e >= E:
            continue
        n_idx, j_idx = torch.nonzero(ids == e, as_tuple=True)
        bgu = q8(dequant_rot(layer["w13_cb"], layer["w13_lo"][e], layer["w13_hi"][e], layer["w13_sc"][e]))
        bdn = q8(dequant_rot(layer["w2_cb"], layer["w2_lo"][e], layer["w2_hi"][e], layer["w2_sc"][e]))
        gu = (xq[n_idx] @ bgu.T) * inv_x[n_idx, None]
        a = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        vq, inv_v = quant_fp8_rows(had_rows(a))
        d = (vq @ bdn.T) * (topk_w.float()[n_idx, j_idx] * inv_v)[:, None]
        out.index_add_(0, n_idx, d)
    return out


def moe_decode_bf16_ref(x, topk_ids, topk_w, layer, expert_base=0, E=None):
    """The reference's own decode algorithm (vq2_vllm/kernels/vq2_kernel.py:569-594 with its
    defaults VQ2_BF16_ACT=1, VQ2_BF16_INTER=1): the Hadamard-rotated activation xh rounded to bf16
    (:584), fp32 dot products, inter = silu(g) * u rounded to bf16 (:585-588), vb = had(inter)
    rounded to bf16 (:589), fp32 down products weighted by w (:590-593). Dense dequantised
    weights as in moe_ref; used to bound the decode kernel's error by the reference's own."""
    x = x.float()
    N, H = x.shape
    E = layer["w13_lo"].shape[0] if E is None else E
    I = layer["w13_lo"].shape[1] // 2
    ids = topk_ids.long() - expert_base
    out = torch.zeros(N, H, device=x.device)
    bf = lambda t: t.bfloat16().float()
    xh = bf(had_rows(bf(x)))
    for e in torch.unique(ids).tolist():
        if e < 0 or e >= E:
            continue
        n_idx, j_idx = torch.nonzero(ids == e, as_tuple=True)
        wgu = dequant_rot(layer["w13_cb"], layer["w13_lo"][e], layer["w13_hi"][e], layer["w13_sc"][e])
        wdn = dequant_rot(layer["w2_cb"], layer["w2_lo"][e], layer["w2_hi"][e], layer["w2_sc"][e])
        g = xh[n_idx] @ wgu.T
        a = bf(torch.nn.functional.silu(g[:, :I]) * g[:, I:])
        d = bf(had_rows(a)) @ wdn.T
        out.index_add_(0, n_idx, d * topk_w.float()[n_idx, j_idx, None])
    return out
