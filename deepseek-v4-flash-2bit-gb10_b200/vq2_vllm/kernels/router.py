"""Router of the routed experts on the B200 library: top-k of softmax(x @ W_r).

This is the routing the benchmark configurations specify (softmax over the E experts, top-k, the
selected probabilities as weights, not renormalised). In vLLM the router runs just before the MoE
method, whose `apply` receives its topk_weights / topk_ids; this kernel produces the same two
tensors in two chained launches instead of a GEMM, a softmax and a top-k.
"""
from __future__ import annotations

import torch

from .. import _lib

_WS = {}


def router_topk(x: torch.Tensor, w_r: torch.Tensor, k: int):
    """x [N, H] (bf16 / fp16 / fp32), w_r [H, E] bf16 -> (topk_ids int32 [N, k], topk_w fp32 [N, k]).
    Ids by probability descending (lower index first on ties)."""
    _lib.require_cuda(x, w_r, device=x.get_device() if x.is_cuda else -1)
    if w_r.dtype != torch.bfloat16 or w_r.dim() != 2 or x.dim() != 2 or x.shape[1] != w_r.shape[0]:
        raise ValueError("vq2 router: x [N, H] and bf16 w_r [H, E] expected")
    x = x.contiguous()
    w_r = w_r.contiguous()
    N, H = x.shape
    E = w_r.shape[1]
    ids = torch.empty(N, k, dtype=torch.int32, device=x.device)
    wts = torch.empty(N, k, dtype=torch.float32, device=x.device)
    L = _lib.lib()
    need = L.vq2_router_workspace_size(N, H, E)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    key = (x.device.index, stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=x.device)
        _WS[key] = ws
    _lib.check(L.vq2_router_topk(x.data_ptr(), _lib.DT[x.dtype], w_r.data_ptr(), N, H, E, k, ids.data_ptr(),
                                 wts.data_ptr(), ws.data_ptr(), ws.numel(), stream), "vq2_router_topk")
    return ids, wts
