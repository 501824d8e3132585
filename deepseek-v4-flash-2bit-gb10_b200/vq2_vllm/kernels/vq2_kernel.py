"""vq2 decode entry points on the B200 C-ABI extension.

Mirrors the reference module ``vq2_vllm/kernels/vq2_kernel.py`` for the routed-expert path: same
function names, argument order and meaning, same return types. The arithmetic runs in
libvq2_b200.so (sm_100a); there is no Triton and no CPU path.
"""
from __future__ import annotations

import torch

from .. import _lib

DEV = "cuda"


def _hadamard(n):
    """Sylvester Hadamard / sqrt(n) (reference vq2_kernel.py:18-22). Host helper for tests and
    weight tooling; the kernels apply the transform in-register."""
    h = torch.ones(1, 1)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / (n ** 0.5)


def _pack10(idx):
    """10-bit index -> (lo u8, hi u8 with four 2-bit fields per byte) (reference vq2_kernel.py:491-498)."""
    from ..synth import pack10
    return pack10(idx)


def had_act_batch(X, group=64):
    """Hadamard per 64-group over the last dim: X[..., in] -> [..., in_pad], same dtype
    (reference vq2_kernel.py:188-195). Runs the extension's shuffle-FWHT kernel."""
    if group != 64:
        raise ValueError("vq2: only group=64 is supported")
    _lib.require_cuda(X)
    *b, n = X.shape
    pad = (-n) % group
    if pad:
        X = torch.cat([X, torch.zeros(*b, pad, device=X.device, dtype=X.dtype)], -1)
    X = X.contiguous()
    Y = torch.empty_like(X)
    rows = X.numel() // X.shape[-1]
    _lib.check(_lib.lib().vq2_hadamard_rows(X.data_ptr(), _lib.DT[X.dtype], Y.data_ptr(), _lib.DT[Y.dtype],
                                            rows, X.shape[-1], _lib.stream_ptr(X.device)), "had_act_batch")
    return Y


def had_act(x, group=64):
    """x [in] -> x' [in_pad] (reference vq2_kernel.py:75-82)."""
    return had_act_batch(x[None], group)[0]


_F16, _U8, _F32, _I32, _I64 = torch.float16, torch.uint8, torch.float32, torch.int32, torch.int64


def _ok(t, dtype):
    return t.dtype is dtype and t.is_contiguous()


def _prep(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn):
    """Normalise dtypes / contiguity (copies only when needed) and require CUDA tensors."""
    if not x.is_cuda:
        _lib.require_cuda(x)
    if x.dtype not in _lib.DT:
        x = x.to(torch.bfloat16)
    if not x.is_contiguous():
        x = x.contiguous()
    if topk_ids.dtype is not _I32 and topk_ids.dtype is not _I64:
        topk_ids = topk_ids.to(_I32)
    if not topk_ids.is_contiguous():
        topk_ids = topk_ids.contiguous()
    if not _ok(topk_w, _F32):
        topk_w = topk_w.float().contiguous()
    ws = [Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn]
    want = (_F16, _U8, _U8, _F16, _F16, _U8, _U8, _F16)
    for i, (t, d) in enumerate(zip(ws, want)):
        if not _ok(t, d):
            ws[i] = t.to(d).contiguous()
    _lib.require_cuda(topk_ids, topk_w, *ws, device=x.get_device())
    return [x, topk_ids, topk_w] + ws


def vq2_moe_fused_10b(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, group=64, expert_base=0):
    """Decode MoE over 10-bit byte-plane VQ experts -> fp32 [N, H]
    (reference vq2_kernel.py:569-594). ``expert_base`` (extension, default 0): ids are global and
    only experts [expert_base, expert_base + E) held in these tensors are applied (expert
    parallelism). Batches above the decode kernel's pair limit go to the grouped GEMM path, in the
    precision VQ2_FP8_PREFILL selects (fp8 by default, as the plugin's prefill dispatch)."""
    if group != 64:
        raise ValueError("vq2: only group=64 is supported")
    if x.is_cuda and x.get_device() != torch.cuda.current_device():   # the library launches on the current device
        with torch.cuda.device(x.device):
            return vq2_moe_fused_10b(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, group, expert_base)
    N = x.shape[0]
    k = topk_ids.shape[1]
    if N * k > _lib.DECODE_MAX_PAIRS:
        from .ds4_vq2_cuda import vq2_moe_grouped_wmma
        return vq2_moe_grouped_wmma(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, group=group,
                                    expert_base=expert_base)   # VQ2_FP8_PREFILL selects fp8 (default) / f16
    t = _prep(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn)
    out = torch.empty(N, x.shape[1], device=x.device, dtype=torch.float32)
    L = _lib.lib()
    a = _lib.moe_args(*t, out, expert_base=expert_base)
    nb = L.vq2_decode_workspace_size(N, k, a.H, a.I)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    ws = _lib.workspace(nb, x.device, stream)
    rc = L.vq2_decode(a, ws.data_ptr(), ws.numel(), stream)
    if rc:
        _lib.check(rc, "vq2_moe_fused_10b")
    return out


_HOST = {}


def vq2_moe_fused_10b_host(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, out=None, group=64,
                           expert_base=0):
    """Decode step with HOST inputs and result (extension; the reference's callers hold device
    tensors): ``x`` [N, H] bf16/fp16/fp32, ``topk_ids`` [N, k] int32/int64 and ``topk_w`` [N, k] fp32
    are CPU tensors (page-locked for asynchronous copies), the weights are the layer's CUDA tensors.
    One library call queues the input copies, the decode kernels and the copy of the fp32 result
    into ``out`` (a CPU [N, H] fp32 tensor, allocated page-locked when not given) on the current
    stream of the weights' device; ``out`` is valid once that stream is synchronised. The weights
    are validated on their first use."""
    if group != 64:
        raise ValueError("vq2: only group=64 is supported")
    dev = lgu.device
    N, H = x.shape
    k = topk_ids.shape[1]
    if x.is_cuda or topk_ids.is_cuda or topk_w.is_cuda:
        raise ValueError("vq2_moe_fused_10b_host: x, topk_ids and topk_w must be host tensors")
    if (x.dtype not in _lib.DT or topk_ids.dtype not in _lib.ID or topk_w.dtype is not _F32 or not x.is_contiguous()
            or not topk_ids.is_contiguous() or not topk_w.is_contiguous()):
        raise ValueError("vq2_moe_fused_10b_host: contiguous x (bf16/fp16/fp32), ids (int32/int64), w (fp32) expected")
    if N * k > _lib.DECODE_MAX_PAIRS:
        raise ValueError(f"vq2_moe_fused_10b_host: N*k = {N * k} above the decode limit {_lib.DECODE_MAX_PAIRS}")
    if out is None:
        out = torch.empty(N, H, dtype=_F32, pin_memory=True)
    stream = torch.cuda.current_stream(dev).cuda_stream
    wkey = (lgu.data_ptr(), ld.data_ptr(), id(dev))
    if wkey not in _HOST:
        ws = [Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn]
        want = (_F16, _U8, _U8, _F16, _F16, _U8, _U8, _F16)
        for t, d in zip(ws, want):
            if not _ok(t, d):
                raise ValueError("vq2_moe_fused_10b_host: weights must be contiguous fp16 codebooks/scales and u8 planes")
        _lib.require_cuda(*ws, device=lgu.get_device())
        if len(_HOST) > 1024:
            _HOST.clear()
        _HOST[wkey] = True
    L = _lib.lib()
    a = _lib.moe_args(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, out, expert_base=expert_base)
    nst = L.vq2_decode_host_stage_size(N, k, H, a.x_dtype, a.ids_dtype)
    nws = L.vq2_decode_workspace_size(N, k, H, a.I)
    buf = _lib.workspace(nst + nws + 256, dev, stream)
    base = buf.data_ptr()
    rc = L.vq2_decode_host(a, x.data_ptr(), topk_ids.data_ptr(), topk_w.data_ptr(), out.data_ptr(), base, nst,
                           base + nst, buf.numel() - nst, stream)
    if rc:
        _lib.check(rc, "vq2_moe_fused_10b_host")
    return out


class HostDecodeSession:
    """Decode steps of one layer at a fixed batch shape whose inputs and result live in host
    memory (extension; the reference's callers hold device tensors) — the shape of a serving loop
    that receives token rows from the host and returns results to it.

    ``slots`` staging slots each own page-locked host buffers (packed inputs x | topk_ids | topk_w,
    and the fp32 result), device buffers and three events. A step is one library call
    (vq2_decode_host_async): the upload runs on a copy stream, the decode kernels on the current
    stream of the weights' device, the download on a second copy stream, so the copies of
    neighbouring steps overlap this step's kernels. ``step`` first waits until the slot's previous
    upload has read its host buffer; the returned host tensor is valid once ``done(slot)`` is true
    (and stays valid until the slot is reused, ``slots`` steps later)."""

    def __init__(self, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, N, k, x_dtype=torch.bfloat16, ids_dtype=torch.int32,
                 slots=4, expert_base=0):
        import ctypes
        self._ctypes = ctypes
        ws = [Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn]
        want = (_F16, _U8, _U8, _F16, _F16, _U8, _U8, _F16)
        for t, d in zip(ws, want):
            if not _ok(t, d):
                raise ValueError("HostDecodeSession: weights must be contiguous fp16 codebooks/scales and u8 planes")
        _lib.require_cuda(*ws, device=lgu.get_device())
        if x_dtype not in _lib.DT or ids_dtype not in _lib.ID:
            raise ValueError("HostDecodeSession: x bf16/fp16/fp32, ids int32/int64")
        if N * k > _lib.DECODE_MAX_PAIRS:
            raise ValueError(f"HostDecodeSession: N*k = {N * k} above the decode limit {_lib.DECODE_MAX_PAIRS}")
        dev = lgu.device
        H = lgu.shape[2] * 4
        I = lgu.shape[1] // 2
        self.N, self.k, self.H, self.slots, self.dev = N, k, H, slots, dev
        L = self._L = _lib.lib()
        oi, ow, nin = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        L.vq2_decode_host_offsets(N, k, H, _lib.DT[x_dtype], _lib.ID[ids_dtype], ctypes.byref(oi), ctypes.byref(ow),
                                  ctypes.byref(nin))
        self.off_i, self.off_w, self.nin = oi.value, ow.value, nin.value
        xe, ie = torch.empty(0, dtype=x_dtype).element_size(), torch.empty(0, dtype=ids_dtype).element_size()
        self.xb, self.ib, self.wb = N * H * xe, N * k * ie, N * k * 4
        self.nws = L.vq2_decode_workspace_size(N, k, H, I)
        up = lambda v: (v + 255) & ~255
        self.h_in = torch.empty(slots, up(self.nin), dtype=torch.uint8, pin_memory=True)
        self.h_out = torch.empty(slots, N, H, dtype=_F32, pin_memory=True)
        self.d_in = torch.empty(slots, up(self.nin), dtype=torch.uint8, device=dev)
        self.d_out = torch.empty(slots, N, H, dtype=_F32, device=dev)
        self.d_ws = torch.empty(slots, self.nws, dtype=torch.uint8, device=dev)
        self.s_in, self.s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.ev = [[torch.cuda.Event() for _ in range(3)] for _ in range(slots)]   # in, done, out
        with torch.cuda.device(dev):
            for sl in range(slots):            # every event exists (recorded once) before first use
                for e in self.ev[sl]:
                    e.record()
        torch.cuda.synchronize(dev)
        a = self._args = _lib.Vq2MoeArgs()
        a.N, a.H, a.I, a.E, a.topk = N, H, I, lgu.shape[0], k
        a.x_dtype, a.ids_dtype, a.expert_base = _lib.DT[x_dtype], _lib.ID[ids_dtype], expert_base
        a.w13_cb, a.w13_lo, a.w13_hi, a.w13_sc = Cgu.data_ptr(), lgu.data_ptr(), hgu.data_ptr(), sgu.data_ptr()
        a.w2_cb, a.w2_lo, a.w2_hi, a.w2_sc = Cd.data_ptr(), ld.data_ptr(), hd.data_ptr(), sdn.data_ptr()
        self._aref = ctypes.byref(a)
        self._ptr = [(self.h_in[sl].data_ptr(), self.h_out[sl].data_ptr(), self.d_in[sl].data_ptr(),
                      self.d_out[sl].data_ptr(), self.d_ws[sl].data_ptr()) + tuple(e.cuda_event for e in self.ev[sl])
                     for sl in range(slots)]
        self._streams = (self.s_in.cuda_stream, self.s_out.cuda_stream)
        self.i = 0

    def step(self, x, topk_ids, topk_w):
        """Queue one step on host tensors x [N, H], topk_ids [N, k], topk_w [N, k] (fp32);
        returns (slot, the slot's host result tensor)."""
        sl = self.i % self.slots
        self.i += 1
        hin, hout, din, dout, dws, e_in, e_done, e_out = self._ptr[sl]
        self.ev[sl][0].synchronize()             # the slot's previous upload has read h_in
        mm = self._ctypes.memmove
        mm(hin, x.data_ptr(), self.xb)
        mm(hin + self.off_i, topk_ids.data_ptr(), self.ib)
        mm(hin + self.off_w, topk_w.data_ptr(), self.wb)
        rc = self._L.vq2_decode_host_async(self._aref, hin, hout, din, dout, dws, self.nws,
                                           torch.cuda.current_stream(self.dev).cuda_stream, self._streams[0],
                                           self._streams[1], e_in, e_done, e_out)
        if rc:
            _lib.check(rc, "HostDecodeSession")
        return sl, self.h_out[sl]

    def done(self, slot) -> bool:
        return self.ev[slot][2].query()

    def synchronize(self):
        """Wait for every queued step's download."""
        for sl in range(self.slots):
            self.ev[sl][2].synchronize()


# The packer lives beside the decode entry in the reference module (vq2_kernel.py:37-72, :160-167,
# :501-505); its implementation here is kernels/vq2_pack.py.
from .vq2_pack import pack_vq2, pack_vq2_experts, pack_vq2_experts_10b  # noqa: E402,F401
