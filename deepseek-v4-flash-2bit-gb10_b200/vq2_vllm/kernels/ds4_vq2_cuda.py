"""vq2 prefill entry points on the B200 C-ABI extension (mirrors reference
vq2_vllm/kernels/ds4_vq2_cuda.py): ``quant_fp8_rows`` and ``vq2_moe_grouped_wmma``."""
from __future__ import annotations

import os

import torch

from .. import _lib
from .vq2_kernel import _prep


def quant_fp8_rows(x):
    """x [M,N] fp32 -> (fp8 e4m3 [M,N], inv [M] fp32): s = 448/max(amax,1e-6) per row
    (reference ds4_vq2_cuda.py:8-32)."""
    _lib.require_cuda(x)
    x = x.float().contiguous()
    M, N = x.shape
    o = torch.empty(M, N, device=x.device, dtype=torch.float8_e4m3fn)
    inv = torch.empty(M, device=x.device, dtype=torch.float32)
    _lib.check(_lib.lib().vq2_quant_fp8_rows(x.data_ptr(), M, N, o.data_ptr(), inv.data_ptr(),
                                             _lib.stream_ptr(x.device)), "quant_fp8_rows")
    return o, inv


def vq2_moe_grouped_wmma(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, group=64, NN=2, BKC=64, NW=8,
                         expert_base=0, precision=None):
    """Prefill (grouped GEMM) MoE -> fp32 [N, H] (reference ds4_vq2_cuda.py:72-111).
    NN/BKC/NW are the reference's mma.sync tiling hints, accepted and ignored. ``precision``:
    "fp8" (the reference's fp8 e4m3 algorithm, default, like VQ2_FP8_PREFILL=1) or "f16"
    (fp16 operands with power-of-two activation scaling, fp32 accumulation; VQ2_FP8_PREFILL=0)."""
    if group != 64:
        raise ValueError("vq2: only group=64 is supported")
    if precision is None:
        precision = "fp8" if os.environ.get("VQ2_FP8_PREFILL", "1") == "1" else "f16"
    if x.is_cuda and x.get_device() != torch.cuda.current_device():   # the library launches on the current device
        with torch.cuda.device(x.device):
            return vq2_moe_grouped_wmma(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, group=group,
                                        expert_base=expert_base, precision=precision)
    t = _prep(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn)
    N = x.shape[0]
    out = torch.empty(N, x.shape[1], device=x.device, dtype=torch.float32)
    L = _lib.lib()
    a = _lib.moe_args(*t, out, expert_base=expert_base)
    p = _lib.PREC[precision]
    nb = L.vq2_prefill_workspace_size(a.N, a.topk, a.E, a.H, a.I, p)
    ws = _lib.workspace(nb, x.device)
    _lib.check(L.vq2_prefill(a, p, ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device)), "vq2_moe_grouped_wmma")
    return out
