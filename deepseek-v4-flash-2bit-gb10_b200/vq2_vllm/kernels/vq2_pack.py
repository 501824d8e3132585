"""VQ packer on the B200 library: quantise weights into the vq2 format (offline, not serving).

Mirrors the reference packer in ``vq2_vllm/kernels/vq2_kernel.py``: ``pack_vq2`` (:37-72),
``pack_vq2_experts`` (:160-167) and ``pack_vq2_experts_10b`` (:501-505): same names, arguments and
return values. The sample of sub-vectors and the initial codebook are drawn exactly as the
reference draws them (``torch.manual_seed(0)``, ``torch.randint`` then ``torch.randperm`` on the
weight's device), so on the same GPU both start from the same sample. Rotation, k-means and the
final assignment run in libvq2_b200.so (``vq2_pack_gather``, ``vq2_kmeans``, ``vq2_pack_assign``);
their arithmetic is fixed operation by operation, so results are reproducible bit for bit (the
reference's torch.cdist rounds differently, so near-ties can resolve differently there).
Supported: vdim=4, group=64, k <= 1024 (the vq2 format); anything else raises.
"""
from __future__ import annotations

import torch

from .. import _lib

SAMPLE = 200000      # k-means sample size (reference vq2_kernel.py:51)


def _check(vdim, k, group):
    if vdim != 4 or group != 64 or not (1 <= k <= 1024):
        raise ValueError("vq2 packer: vdim=4, group=64 and 1 <= k <= 1024 only (the vq2 format)")


def draw_sample(nvec: int, k: int, device):
    """(sample sub-vector indices int64 [min(nvec, 200000)], initial-codebook positions into the
    sample [<= k]) drawn as the reference does (vq2_kernel.py:50-52)."""
    torch.manual_seed(0)
    si = torch.randint(0, nvec, (min(nvec, SAMPLE),), device=device)
    init = torch.randperm(si.shape[0], device=device)[:k]
    return si, init


def _w_arg(W):
    if W.dtype not in _lib.DT:
        W = W.float()
    return W.contiguous()


def pack_from_sample(W, si, init, iters=12, planes=True, ids=True, dq=True):
    """Pack W [rows, D] with a given sample (``si``: sub-vector indices, ``init``: positions of the
    initial codebook in the sample). Returns a dict with C f32 [k', 4] (k' = len(init)), scale f32
    [rows, ng], and as asked lo/hi (10-bit planes), idx int16 [rows, ng*16], dq f32 [rows, D]."""
    _lib.require_cuda(W, si, init, device=W.get_device() if W.is_cuda else -1)
    if W.dim() != 2:
        raise ValueError("vq2 packer: W must be 2-D [out, in]")
    with torch.cuda.device(W.device):
        W = _w_arg(W)
        rows, D = W.shape
        ng = (D + 63) // 64
        dev = W.device
        L = _lib.lib()
        st = _lib.stream_ptr(dev)
        dt = _lib.DT[W.dtype]
        si = si.to(torch.int64).contiguous()
        nvec = rows * ng * 16
        if si.numel() and (int(si.min()) < 0 or int(si.max()) >= nvec):
            raise ValueError(f"vq2 packer: sample indices must lie in [0, {nvec})")
        if init.numel() == 0 or int(init.min()) < 0 or int(init.max()) >= si.shape[0]:
            raise ValueError(f"vq2 packer: init positions must lie in [0, {si.shape[0]})")
        samp = torch.empty(si.shape[0], 4, dtype=torch.float32, device=dev)
        _lib.check(L.vq2_pack_gather(W.data_ptr(), dt, rows, D, si.data_ptr(), si.shape[0], samp.data_ptr(), st),
                   "vq2_pack_gather")
        C = samp.index_select(0, init.to(torch.int64)).contiguous()
        k = C.shape[0]
        ws = torch.empty(L.vq2_kmeans_workspace_size(k), dtype=torch.uint8, device=dev)
        _lib.check(L.vq2_kmeans(samp.data_ptr(), samp.shape[0], C.data_ptr(), k, iters, ws.data_ptr(), ws.numel(), st),
                   "vq2_kmeans")
        out = {"C": C, "scale": torch.empty(rows, ng, dtype=torch.float32, device=dev)}
        nsub = ng * 16
        if planes:
            out["lo"] = torch.empty(rows, nsub, dtype=torch.uint8, device=dev)
            out["hi"] = torch.empty(rows, nsub // 4, dtype=torch.uint8, device=dev)
        if ids:
            out["idx"] = torch.empty(rows, nsub, dtype=torch.int16, device=dev)
        if dq:
            out["dq"] = torch.empty(rows, D, dtype=torch.float32, device=dev)
        ptr = lambda name: out[name].data_ptr() if name in out else None  # noqa: E731
        _lib.check(L.vq2_pack_assign(W.data_ptr(), dt, rows, D, C.data_ptr(), k, ptr("lo"), ptr("hi"), ptr("idx"),
                                     out["scale"].data_ptr(), ptr("dq"), st), "vq2_pack_assign")
        return out


def _pack(W, k, iters, planes, ids):
    _lib.require_cuda(W)
    rows, D = W.shape
    nvec = rows * ((D + 63) // 64) * 16
    si, init = draw_sample(nvec, k, W.device)
    return pack_from_sample(W, si, init, iters, planes=planes, ids=ids, dq=True)


def pack_vq2(W, vdim=4, k=1024, group=64, iters=12):
    """W [out, in] -> (C [k, 4] f32, idx [out, nsub] (uint8 for k <= 256, else int16), scale
    [out, ng] f32, dq [out, in] f32, in, pad) (reference vq2_kernel.py:37-72)."""
    _check(vdim, k, group)
    r = _pack(W, k, iters, planes=False, ids=True)
    inn = W.shape[1]
    idx = r["idx"].to(torch.uint8) if k <= 256 else r["idx"]
    return r["C"], idx, r["scale"], r["dq"], inn, (-inn) % group


def pack_vq2_experts(W3, vdim=4, k=1024, group=64, iters=12):
    """W3 [E, R, D] with ONE codebook over all experts -> (C, idx [E, R, nsub], scale [E, R, ng],
    dq [E, R, D]) (reference vq2_kernel.py:160-167)."""
    E, R, D = W3.shape
    C, idx, scale, dq, _, _ = pack_vq2(W3.reshape(E * R, D), vdim, k, group, iters)
    return C, idx.reshape(E, R, -1), scale.reshape(E, R, -1), dq.reshape(E, R, D)


def pack_vq2_experts_10b(W3, vdim=4, k=1024, group=64, iters=12):
    """Like pack_vq2_experts with the 10-bit planes: (C, lo [E, R, nsub], hi [E, R, nsub/4],
    scale, dq) (reference vq2_kernel.py:501-505). The planes come straight from the kernel."""
    _check(vdim, k, group)
    E, R, D = W3.shape
    r = _pack(W3.reshape(E * R, D), k, iters, planes=True, ids=False)
    return (r["C"], r["lo"].reshape(E, R, -1), r["hi"].reshape(E, R, -1), r["scale"].reshape(E, R, -1),
            r["dq"].reshape(E, R, D))
