"""ctypes binding of libvq2_b200.so (the C ABI declared in include/vq2_b200.h).

The library is loaded from the package tree (built in-tree by ``build_lib.py``). There is no
fallback: if the library is missing every kernel entry raises, naming the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("VQ2_LIB") or os.path.join(os.path.dirname(_HERE), "libvq2_b200.so")

DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
ID = {torch.int32: 0, torch.int64: 1}
PREC = {"fp8": 0, "f16": 1}
DECODE_MAX_PAIRS = 512


class Vq2MoeArgs(ctypes.Structure):
    _fields_ = [("N", ctypes.c_int), ("H", ctypes.c_int), ("I", ctypes.c_int), ("E", ctypes.c_int),
                ("topk", ctypes.c_int), ("x_dtype", ctypes.c_int), ("ids_dtype", ctypes.c_int),
                ("expert_base", ctypes.c_int),
                ("x", ctypes.c_void_p), ("topk_ids", ctypes.c_void_p), ("topk_w", ctypes.c_void_p),
                ("w13_cb", ctypes.c_void_p), ("w13_lo", ctypes.c_void_p), ("w13_hi", ctypes.c_void_p),
                ("w13_sc", ctypes.c_void_p),
                ("w2_cb", ctypes.c_void_p), ("w2_lo", ctypes.c_void_p), ("w2_hi", ctypes.c_void_p),
                ("w2_sc", ctypes.c_void_p), ("out", ctypes.c_void_p)]



class Vq2EpLayout(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in ("off_x", "off_ids", "off_w", "off_comb", "off_dflag", "off_cflag",
                                               "off_epoch", "off_count")]


_SIGS = {
    "vq2_decode_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 4),
    "vq2_decode": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_decode_host_stage_size": (ctypes.c_size_t, [ctypes.c_int] * 5),
    "vq2_decode_host": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                       ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_decode_host_offsets": (None, [ctypes.c_int] * 5 + [ctypes.POINTER(ctypes.c_size_t)] * 3),
    "vq2_decode_host_async": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs)] + [ctypes.c_void_p] * 5 + [ctypes.c_size_t]
                              + [ctypes.c_void_p] * 6),
    "vq2_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_void_p]),
    "vq2_prefill_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 6),
    "vq2_prefill": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.c_void_p]),
    "vq2_align_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 3),
    "vq2_align": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_quant_fp8_rows": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p]),
    "vq2_hadamard_rows": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                         ctypes.c_long, ctypes.c_int, ctypes.c_void_p]),
    "vq2_ep_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "vq2_ep_free": (ctypes.c_int, [ctypes.c_void_p]),
    "vq2_ipc_get_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "vq2_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "vq2_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "vq2_ep_dispatch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_ep_combine": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                      ctypes.c_void_p, ctypes.c_void_p]),
    "vq2_ep_decode_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 5),
    "vq2_ep_decode": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_void_p, ctypes.POINTER(Vq2EpLayout), ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_void_p]),
    "vq2_router_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 3),
    "vq2_router_topk": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_pack_gather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]),
    "vq2_kmeans_workspace_size": (ctypes.c_size_t, [ctypes.c_int]),
    "vq2_kmeans": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_pack_assign": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "vq2_shared_expert_workspace_size": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    "vq2_shared_expert": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_decode_with_shared_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 5),
    "vq2_decode_with_shared": (ctypes.c_int, [ctypes.POINTER(Vq2MoeArgs), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "vq2_device_status": (ctypes.c_int, [ctypes.c_int]),
    "vq2_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "vq2_version": (ctypes.c_int, []),
}

_LIB = None


def lib():
    """Load (once) and return the C-ABI library; raises if it is not built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"vq2: {LIB_PATH} is not built; run python build_lib.py "
                               "(or __graft_entry__.build()) — there is no fallback path")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name, None)
            if f is None:
                continue
            f.restype, f.argtypes = res, args
        _LIB = L
    return _LIB


def check(code: int, what: str = "vq2"):
    if code != 0:
        msg = lib().vq2_strerror(code).decode()
        raise RuntimeError(f"{what}: {msg} (code {code})")


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


def require_cuda(*ts, device: int = -1):
    """Every tensor is a CUDA tensor (there is no CPU path) and, with ``device`` >= 0, on that
    device (a tensor on another GPU would hand the kernels a foreign pointer)."""
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("vq2: all tensors must be CUDA tensors (no CPU path)")
        if device >= 0 and t.get_device() != device:
            raise RuntimeError(f"vq2: tensors on cuda:{t.get_device()} and cuda:{device}; all must share one device")


_WS = {}


def workspace(nbytes: int, device, stream=None) -> torch.Tensor:
    """Cached per-(device, stream) byte workspace, grown on demand (graph-safe once sized)."""
    if stream is None:
        stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index if isinstance(device, torch.device) else device, stream)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


_TLS = threading.local()


def moe_args(x, topk_ids, topk_w, Cgu, lgu, hgu, sgu, Cd, ld, hd, sdn, out, expert_base=0, E=None):
    """The vq2_moe_args struct for one call. The weight part is cached per layer (keyed by the
    weight pointers and shapes) and per host thread, so a call only rewrites the per-call fields
    and two threads calling the same layer never share (and race on) one struct. The struct is
    read by the library during the call only."""
    wkey = (Cgu.data_ptr(), lgu.data_ptr(), hgu.data_ptr(), sgu.data_ptr(), Cd.data_ptr(), ld.data_ptr(),
            hd.data_ptr(), sdn.data_ptr(), lgu.shape, E)
    _ARGS = getattr(_TLS, "args", None)
    if _ARGS is None:
        _ARGS = _TLS.args = {}
    a = _ARGS.get(wkey)
    if a is None:
        a = Vq2MoeArgs()
        a.I = lgu.shape[1] // 2
        a.E = lgu.shape[0] if E is None else E
        a.w13_cb, a.w13_lo, a.w13_hi, a.w13_sc = wkey[0], wkey[1], wkey[2], wkey[3]
        a.w2_cb, a.w2_lo, a.w2_hi, a.w2_sc = wkey[4], wkey[5], wkey[6], wkey[7]
        if len(_ARGS) > 4096:
            _ARGS.clear()
        _ARGS[wkey] = a
    N, H = x.shape
    a.N, a.H = N, H
    a.topk = topk_ids.shape[1]
    a.x_dtype, a.ids_dtype, a.expert_base = DT[x.dtype], ID[topk_ids.dtype], expert_base
    a.x, a.topk_ids, a.topk_w, a.out = x.data_ptr(), topk_ids.data_ptr(), topk_w.data_ptr(), out.data_ptr()
    return a
