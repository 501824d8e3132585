"""Seeded synthetic vq2 layers and inputs in the reference's exact tensor layout.

Layout follows ``Vq2MoEMethod.create_weights`` (vq2_vllm/__init__.py:164-173):
  w13_lo [E,2I,H/4] u8, w13_hi [E,2I,H/16] u8, w13_sc [E,2I,H/64] f16,
  w2_lo  [E,H,I/4]  u8, w2_hi  [E,H,I/16]  u8, w2_sc  [E,H,I/64]  f16,
  w13_cb / w2_cb [1024,4] f16.
Codebook entries are drawn N(0, 0.02) in bf16 and stored as fp16; indices are uniform 10-bit;
scales are U(0.5, 1.5) fp16 (the format needs them; the benchmark spec leaves them open).
"""
from __future__ import annotations

import torch

KEYS = ("w13_cb", "w13_lo", "w13_hi", "w13_sc", "w2_cb", "w2_lo", "w2_hi", "w2_sc")


def pack10(idx: torch.Tensor):
    """10-bit index -> (lo u8, hi u8 with four 2-bit fields per byte), the reference's ``_pack10``
    format (vq2_vllm/kernels/vq2_kernel.py:491-498)."""
    lo = (idx & 0xFF).to(torch.uint8)
    h = ((idx >> 8) & 0x3).to(torch.uint8)
    h = h.reshape(*h.shape[:-1], h.shape[-1] // 4, 4)
    hp = (h[..., 0] | (h[..., 1] << 2) | (h[..., 2] << 4) | (h[..., 3] << 6)).to(torch.uint8)
    return lo.contiguous(), hp.contiguous()


def _planes(E, R, K, gen, device):
    """Random 10-bit planes generated directly as bytes (uniform lo byte + uniform 2-bit fields)."""
    lo = torch.randint(0, 256, (E, R, K // 4), generator=gen, dtype=torch.uint8, device=device)
    hi = torch.randint(0, 256, (E, R, K // 16), generator=gen, dtype=torch.uint8, device=device)
    sc = (torch.rand((E, R, K // 64), generator=gen, device=device) + 0.5).half()
    return lo, hi, sc


def make_layer(E: int, H: int, I: int, seed: int = 0, device="cpu"):
    """One seeded vq2 expert layer as a dict keyed like the reference's safetensors file
    (vq2_vllm/__init__.py:233-235)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    cb13 = (torch.randn((1024, 4), generator=gen, device=device) * 0.02).bfloat16().half()
    cb2 = (torch.randn((1024, 4), generator=gen, device=device) * 0.02).bfloat16().half()
    l13, h13, s13 = _planes(E, 2 * I, H, gen, device)
    l2, h2, s2 = _planes(E, H, I, gen, device)
    return {"w13_cb": cb13, "w13_lo": l13, "w13_hi": h13, "w13_sc": s13,
            "w2_cb": cb2, "w2_lo": l2, "w2_hi": h2, "w2_sc": s2}


def layer_args(layer):
    """(Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn) in the kernel-entry argument order
    (vq2_vllm/kernels/vq2_kernel.py:569)."""
    return tuple(layer[k] for k in KEYS)


def make_tokens(N: int, H: int, seed: int = 1, device="cpu"):
    gen = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((N, H), generator=gen, device=device).bfloat16()


def route_softmax_topk(x: torch.Tensor, E: int, k: int, w_std: float, seed: int = 2):
    """Router of the benchmark configs: softmax(x @ W_r) over E experts, then top-k
    (weights are the selected softmax probabilities, not renormalised)."""
    gen = torch.Generator(device=x.device).manual_seed(seed)
    wr = (torch.randn((x.shape[1], E), generator=gen, device=x.device) * w_std).bfloat16()
    p = torch.softmax((x.float() @ wr.float()), -1)
    tw, ti = torch.topk(p, k, dim=-1)
    return ti.to(torch.int32), tw.float()


def route_zipf(N: int, E: int, k: int, s: float = 1.1, seed: int = 2, device="cpu", draw_seed=None):
    """Zipf(s)-skewed top-k routing with distinct experts per token: p_e ~ 1/rank_e^s over a
    seeded permutation of ranks; weights = softmax of N(0,1) over the k picks. ``draw_seed``
    (optional) seeds the token draws separately from the popularity permutation, so several
    sources (expert-parallel ranks) share one expert popularity but draw different tokens."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    ranks = torch.randperm(E, generator=gen).double() + 1.0
    if draw_seed is not None:
        gen = torch.Generator(device="cpu").manual_seed(draw_seed)
    p = ranks.pow(-s)
    p = (p / p.sum()).float()
    ids = torch.multinomial(p.expand(N, E), k, replacement=False, generator=gen).to(torch.int32)
    tw = torch.softmax(torch.randn((N, k), generator=gen), -1).float()
    return ids.to(device), tw.to(device)


def route_uniform(N: int, E: int, k: int, seed: int = 2, device="cpu"):
    """Uniformly random distinct top-k experts per token; weights softmax of N(0,1)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.argsort(torch.rand((N, E), generator=gen), dim=-1)[:, :k].to(torch.int32)
    tw = torch.softmax(torch.randn((N, k), generator=gen), -1).float()
    return ids.to(device), tw.to(device)
