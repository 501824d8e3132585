"""Shared expert of the decode step on the B200 library (dense bf16 SiLU-gated MLP).

In the served model vLLM runs the shared expert beside the MoE method (the reference plugin's
``apply`` receives ``shared_experts`` and leaves it alone, vq2_vllm/__init__.py:197-198). This
entry computes the same layer with two HBM-streaming kernels chained by programmatic dependent
launch, and can add its result onto the routed experts' output on the same stream.
"""
from __future__ import annotations

import torch

from .. import _lib

_WS = {}


def shared_expert_fused(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, out: torch.Tensor | None = None):
    """x [N, H] (bf16 / fp16 / fp32, N <= 8), w13 bf16 [2*Is, H] (gate rows then up rows), w2 bf16
    [H, Is] -> fp32 [N, H] = w2 @ (silu(x @ Wg^T) * (x @ Wu^T)). With ``out`` (fp32 [N, H], e.g. the
    routed output of vq2_moe_fused_10b) the result is added into it and ``out`` is returned."""
    _lib.require_cuda(x, w13, w2, *(() if out is None else (out,)), device=x.get_device() if x.is_cuda else -1)
    if w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
        raise ValueError("vq2 shared expert: bf16 weights expected")
    N, H = x.shape
    Is = w13.shape[0] // 2
    if w13.shape != (2 * Is, H) or w2.shape != (H, Is):
        raise ValueError("vq2 shared expert: w13 [2*Is, H] and w2 [H, Is] expected")
    with torch.cuda.device(x.device):
        x = x.contiguous() if x.dtype in _lib.DT else x.float().contiguous()
        w13, w2 = w13.contiguous(), w2.contiguous()
        acc = out is not None
        if acc:
            if out.dtype != torch.float32 or out.shape != (N, H) or not out.is_contiguous():
                raise ValueError("vq2 shared expert: out must be contiguous fp32 [N, H]")
        else:
            out = torch.empty(N, H, dtype=torch.float32, device=x.device)
        L = _lib.lib()
        need = L.vq2_shared_expert_workspace_size(N, Is)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        key = (x.device.index, stream)
        ws = _WS.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1 << 16), dtype=torch.uint8, device=x.device)
            _WS[key] = ws
        _lib.check(L.vq2_shared_expert(x.data_ptr(), _lib.DT[x.dtype], w13.data_ptr(), w2.data_ptr(), N, H, Is,
                                       out.data_ptr(), int(acc), ws.data_ptr(), ws.numel(), stream),
                   "vq2_shared_expert")
        return out


def moe_with_shared_expert(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, w13, w2, shared_sms: int = 0,
                           expert_base: int = 0):
    """Routed decode (as ``vq2_moe_fused_10b``) plus the shared expert (as ``shared_expert_fused``)
    for the same tokens in one call -> fp32 [N, H] (N <= 8, N * k within the decode pair limit).
    The shared expert's kernels run concurrently with the routed ones on ``shared_sms`` SMs (0: the
    library default) on a second stream of the library, forked and joined with events on the
    current stream; both add into the output with fp32 atomics."""
    from .vq2_kernel import _prep
    if w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
        raise ValueError("vq2 shared expert: bf16 weights expected")
    N, H = x.shape
    Is = w13.shape[0] // 2
    if w13.shape != (2 * Is, H) or w2.shape != (H, Is):
        raise ValueError("vq2 shared expert: w13 [2*Is, H] and w2 [H, Is] expected")
    if N * topk_ids.shape[1] > _lib.DECODE_MAX_PAIRS:
        raise ValueError("vq2 routed + shared: N * k above the decode pair limit")
    with torch.cuda.device(x.device):
        t = _prep(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn)
        w13, w2 = w13.contiguous(), w2.contiguous()
        _lib.require_cuda(w13, w2, device=x.get_device())
        out = torch.empty(N, H, dtype=torch.float32, device=x.device)
        L = _lib.lib()
        a = _lib.moe_args(*t, out, expert_base=expert_base)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        ws = _lib.workspace(L.vq2_decode_with_shared_workspace_size(N, topk_ids.shape[1], H, a.I, Is), x.device, stream)
        _lib.check(L.vq2_decode_with_shared(a, w13.data_ptr(), w2.data_ptr(), Is, int(shared_sms), ws.data_ptr(),
                                            ws.numel(), stream), "vq2_decode_with_shared")
        return out
