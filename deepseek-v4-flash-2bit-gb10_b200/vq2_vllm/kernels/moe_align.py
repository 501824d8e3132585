"""moe_align on the B200 C-ABI extension (mirrors reference vq2_vllm/kernels/moe_align.py).

``moe_align(topk_ids, E, BM)`` -> (sorted_tok i32[Pmax], sorted_slot i32[Pmax], valid bool[Pmax],
block_e i32[nblk], nblk) with Pmax = M + min(M, E) * BM. Output is bit-identical to the
reference's deterministic ``_moe_align_torch`` (moe_align.py:56-86): pairs keep their order
within an expert. ``moe_align_fast`` is the same kernel (the reference's atomic version is a
non-deterministic permutation of this output). Graph-safe: fixed host-computable sizes, no sync.
"""
from __future__ import annotations

import torch

from .. import _lib


def moe_align(topk_ids, E, BM):
    _lib.require_cuda(topk_ids)
    ids = topk_ids if topk_ids.dtype in _lib.ID else topk_ids.to(torch.int32)
    ids = ids.contiguous()
    N, k = ids.shape
    M = N * k
    Pmax = M + min(M, E) * BM
    nblk = Pmax // BM
    dev = ids.device
    st = torch.empty(Pmax, dtype=torch.int32, device=dev)
    ss = torch.empty(Pmax, dtype=torch.int32, device=dev)
    val = torch.empty(Pmax, dtype=torch.bool, device=dev)
    be = torch.empty(nblk, dtype=torch.int32, device=dev)
    L = _lib.lib()
    nb = L.vq2_align_workspace_size(N, k, E)
    ws = _lib.workspace(nb, dev)
    _lib.check(L.vq2_align(ids.data_ptr(), _lib.ID[ids.dtype], N, k, E, BM, st.data_ptr(), ss.data_ptr(),
                           val.data_ptr(), be.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev)),
               "moe_align")
    return st, ss, val, be, nblk


moe_align_fast = moe_align
