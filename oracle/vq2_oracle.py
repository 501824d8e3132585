"""CPU oracle for the vq2 routed-expert MoE path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import it. The product path (the CUDA extension)
never routes through it.

It restates, in numpy (fp32, plus a bit-exact software e4m3 rounding), the algorithm of the
reference plugin ``vq2_vllm`` (iggerask/deepseek-v4-flash-2bit-gb10). Every function cites the
reference ``file:line`` it follows; paths are relative to the reference project root.

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference's own Python modules
(Triton kernels run under ``TRITON_INTERPRET=1``) and records their outputs in
``tests/golden/*.npz``; ``tests/test_oracle.py`` checks this module against those fixtures.
"""
from __future__ import annotations

import numpy as np

VDIM = 4          # codebook vector width            (vq2_vllm/__init__.py:331 default vdim=4)
KCB = 1024        # codebook entries (10-bit index)  (vq2_vllm/__init__.py:332 default k=1024)
GROUP = 64        # Hadamard / scale group           (vq2_vllm/__init__.py:333 default group=64)
SPG = GROUP // VDIM


# ----------------------------------------------------------------------------- format
def hadamard(n: int) -> np.ndarray:
    """Sylvester Hadamard normalised by 1/sqrt(n) (vq2_vllm/kernels/vq2_kernel.py:18-22)."""
    h = np.ones((1, 1), dtype=np.float64)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return (h / np.sqrt(n)).astype(np.float32)


def had_act_batch(x: np.ndarray, group: int = GROUP) -> np.ndarray:
    """x' = x @ H per contiguous group of the last dim, zero-padded to a group multiple
    (vq2_vllm/kernels/vq2_kernel.py:188-195). fp32 in, fp32 out."""
    x = np.asarray(x, dtype=np.float32)
    *b, n = x.shape
    pad = (-n) % group
    if pad:
        x = np.concatenate([x, np.zeros((*b, pad), np.float32)], -1)
    h = hadamard(group)
    return (x.reshape(*b, -1, group) @ h).reshape(*b, -1).astype(np.float32)


def pack10(idx: np.ndarray):
    """10-bit index -> (lo u8 plane, hi plane with four 2-bit fields per byte, little-end first)
    (vq2_vllm/kernels/vq2_kernel.py:491-498)."""
    idx = np.asarray(idx).astype(np.int64)
    lo = (idx & 0xFF).astype(np.uint8)
    h = ((idx >> 8) & 0x3).astype(np.uint8)
    h = h.reshape(*h.shape[:-1], h.shape[-1] // 4, 4)
    hp = (h[..., 0] | (h[..., 1] << 2) | (h[..., 2] << 4) | (h[..., 3] << 6)).astype(np.uint8)
    return np.ascontiguousarray(lo), np.ascontiguousarray(hp)


def unpack10(lo: np.ndarray, hi: np.ndarray) -> np.ndarray:
    """Inverse of pack10: id = lo[s] | ((hi[s>>2] >> 2*(s&3)) & 3) << 8
    (in-kernel unpack, vq2_vllm/kernels/vq2_kernel.py:534-535; vq2_grouped.cu:437-438)."""
    lo = np.asarray(lo).astype(np.int32)
    hi = np.asarray(hi).astype(np.int32)
    s = np.arange(lo.shape[-1])
    hb = np.take(hi, s >> 2, axis=-1)
    return lo | (((hb >> ((s & 3) * 2)) & 3) << 8)


def dequant_rot(cb, lo, hi, sc) -> np.ndarray:
    """Weights in the rotated space: recon_rot = C[id] * scale per group
    (vq2_vllm/kernels/vq2_kernel.py:63). cb [1024,4] f16, lo [...,R,nsub], sc [...,R,ng] f16."""
    ids = unpack10(lo, hi)
    c = np.asarray(cb, dtype=np.float32)
    w = c[ids]                                            # [..., R, nsub, 4]
    *b, r, nsub, _ = w.shape
    w = w.reshape(*b, r, nsub // SPG, GROUP)
    w = w * np.asarray(sc, dtype=np.float32)[..., None]
    return w.reshape(*b, r, nsub * VDIM).astype(np.float32)


def dequant(cb, lo, hi, sc) -> np.ndarray:
    """Dense dequantised weight W = recon_rot @ H^T per group (vq2_vllm/kernels/vq2_kernel.py:63-64)."""
    wr = dequant_rot(cb, lo, hi, sc)
    *b, r, k = wr.shape
    h = hadamard(GROUP)
    return (wr.reshape(*b, r, k // GROUP, GROUP) @ h.T).reshape(*b, r, k).astype(np.float32)


def silu(v):
    return v / (1.0 + np.exp(-v))


# ----------------------------------------------------------------------------- MoE (fp32)
def moe_ref(x, topk_ids, topk_w, w13, w2):
    """fp32 dequant-plus-matmul MoE reference (vq2_vllm/kernels/vq2_kernel.py:720-727):
    per (token n, slot j): g = W_gu[e] @ x[n]; a = silu(g[:I]) * g[I:]; out[n] += w * W_dn[e] @ a.
    ``w13``/``w2`` are (cb, lo, hi, sc) tuples in the reference layout (__init__.py:164-173).
    Computed in the rotated space (identical maths: W x = recon_rot @ (H^T x))."""
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(topk_ids).astype(np.int64)
    tw = np.asarray(topk_w, dtype=np.float32)
    N, H = x.shape
    I = w13[1].shape[1] // 2
    out = np.zeros((N, H), np.float32)
    xh = had_act_batch(x)
    cache = {}
    for e in np.unique(ids):
        cache[int(e)] = (dequant_rot(w13[0], w13[1][e], w13[2][e], w13[3][e]),
                         dequant_rot(w2[0], w2[1][e], w2[2][e], w2[3][e]))
    for n in range(N):
        for j in range(ids.shape[1]):
            wgu, wdn = cache[int(ids[n, j])]
            g = wgu @ xh[n]
            a = silu(g[:I]) * g[I:]
            out[n] += tw[n, j] * (wdn @ had_act_batch(a[None])[0])
    return out


# ----------------------------------------------------------------------------- moe_align
def moe_align(topk_ids, E: int, BM: int):
    """Stable sort of (token, slot) pairs by expert, each expert's run padded to a BM multiple
    (vq2_vllm/kernels/moe_align.py:56-86, ``_moe_align_torch``). Returns
    (sorted_tok i32[Pmax], sorted_slot i32[Pmax], valid bool[Pmax], block_e i32[nblk], nblk)
    with Pmax = M + min(M, E) * BM (moe_align.py:75)."""
    ids = np.asarray(topk_ids).astype(np.int64)
    N, k = ids.shape
    flat = ids.reshape(-1)
    M = flat.size
    cnt = np.bincount(flat, minlength=E).astype(np.int64)
    padded = ((cnt + BM - 1) // BM) * BM
    eoff = np.cumsum(padded) - padded
    rank = np.zeros(M, np.int64)
    seen = np.zeros(E, np.int64)
    for p in range(M):                                    # stable: rank = order of appearance
        rank[p] = seen[flat[p]]
        seen[flat[p]] += 1
    dest = eoff[flat] + rank
    Pmax = M + min(M, E) * BM
    nblk = Pmax // BM
    st = np.zeros(Pmax, np.int32)
    ss = np.zeros(Pmax, np.int32)
    val = np.zeros(Pmax, bool)
    ar = np.arange(M)
    st[dest] = ar // k
    ss[dest] = ar % k
    val[dest] = True
    block_start = eoff // BM
    blk = np.arange(nblk)
    be = np.clip(np.searchsorted(block_start, blk, side="right") - 1, 0, None).astype(np.int32)
    return st, ss, val, be, nblk


# ----------------------------------------------------------------------------- fp8 e4m3
def to_e4m3(v) -> np.ndarray:
    """Round fp32 -> float8 e4m3fn (bias 7, 3 mantissa bits, max 448, no inf) with
    round-to-nearest-even, returned as the fp32 value it represents. Finite inputs are expected
    in [-448, 448] (the callers saturate, as vq2_grouped.cu:440-443 does); NaN stays NaN."""
    v = np.asarray(v, dtype=np.float32).astype(np.float64)
    a = np.abs(v)
    # exponent of the representable binade; subnormal spacing is 2^-9 below 2^-6
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    step = np.exp2(e - 3.0)
    q = np.round(a / step) * step                          # np.round = half-to-even
    q = np.minimum(q, 448.0)
    return (np.sign(v) * q).astype(np.float32)


def quant_fp8_rows(x):
    """Per-row absmax fp8 quant: s = 448 / max(amax, 1e-6); q = e4m3(x * s); inv = 1/s
    (vq2_vllm/kernels/ds4_vq2_cuda.py:8-23). Returns (q as fp32 values, inv fp32)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(-1)
    s = (np.float32(448.0) / np.maximum(amax, np.float32(1e-6))).astype(np.float32)
    q = to_e4m3((x * s[:, None]).astype(np.float32))
    inv = (np.float32(1.0) / s).astype(np.float32)
    return q, inv


def decode_fp8_weights(cb, lo, hi, sc) -> np.ndarray:
    """Prefill weight decode: e4m3(sat(C[id] * sc)) per element in the rotated space
    (vq2_vllm/kernels/vq2_grouped.cu:434-446)."""
    wr = dequant_rot(cb, lo, hi, sc)
    return to_e4m3(np.clip(wr, -448.0, 448.0))


def moe_prefill_fp8_ref(x, topk_ids, topk_w, w13, w2):
    """The reference's fp8 prefill algorithm (vq2_vllm/kernels/ds4_vq2_cuda.py:72-111):
    xh = had(x) -> per-token fp8 quant (:94) -> gate_up with fp8-decoded weights (:104,
    vq2_grouped.cu:383-480) -> silu(g*inv)*(u*inv) (vq2_grouped.cu:255-264) -> had(inter) -> per-row
    fp8 quant (:106) -> down with weight w*inv_vb (:108-110, vq2_grouped.cu:483-581). fp32 sums."""
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(topk_ids).astype(np.int64)
    tw = np.asarray(topk_w, dtype=np.float32)
    N, H = x.shape
    I = w13[1].shape[1] // 2
    xq, inv_x = quant_fp8_rows(had_act_batch(x))
    out = np.zeros((N, H), np.float32)
    for e in np.unique(ids):
        e = int(e)
        n_idx, j_idx = np.nonzero(ids == e)
        bgu = decode_fp8_weights(w13[0], w13[1][e], w13[2][e], w13[3][e])
        bdn = decode_fp8_weights(w2[0], w2[1][e], w2[2][e], w2[3][e])
        gu = (xq[n_idx] @ bgu.T) * inv_x[n_idx, None]
        inter = silu(gu[:, :I]) * gu[:, I:]
        vq, inv_v = quant_fp8_rows(had_act_batch(inter))
        contrib = (vq @ bdn.T) * (tw[n_idx, j_idx] * inv_v)[:, None]
        np.add.at(out, n_idx, contrib)
    return out


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ----------------------------------------------------------------------------- VQ packer
# Restates the k-means packer of the reference, vq2_kernel.pack_vq2
# (vq2_vllm/kernels/vq2_kernel.py:37-72), with every fp32 operation in the order the B200 kernels
# use, so results compare bit for bit: the group rotation is the 64-point butterfly (strides
# 32, 16, ..., 1, then x 1/8) rather than a matmul; distances are ((d0^2+d1^2)+d2^2)+d3^2; member
# sums are int64 fixed point (x 2^40, rounded to nearest even), means (double)sum * 2^-40 / count.
PACK_FIX = 2.0 ** 40


def fwht64_f32(x: np.ndarray) -> np.ndarray:
    """Rows of 64 fp32 values -> x @ H64 by the butterfly (pair i with i + len, len = 32 .. 1:
    (lo + hi, lo - hi)), then x 1/8; each step rounded to fp32 (vq2_kernel.py:46 rotates with
    W @ H, the same transform)."""
    x = np.asarray(x, np.float32).reshape(-1, 64).copy()
    n = x.shape[0]
    ln = 32
    while ln >= 1:
        r = x.reshape(n, 64 // (2 * ln), 2, ln)
        lo, hi = r[:, :, 0, :].copy(), r[:, :, 1, :].copy()
        r[:, :, 0, :] = lo + hi
        r[:, :, 1, :] = lo - hi
        x = r.reshape(n, 64)
        ln //= 2
    return (x * np.float32(0.125)).astype(np.float32)


def pack_rotate(W: np.ndarray):
    """W [rows, D] -> (Wn [rows*ng, 64] normalised rotated groups, scale f32 [rows*ng]);
    zero-padded to a group multiple; s = max(|group|, 1e-8) (vq2_kernel.py:41-49)."""
    W = np.asarray(W, np.float32)
    rows, D = W.shape
    pad = (-D) % GROUP
    if pad:
        W = np.concatenate([W, np.zeros((rows, pad), np.float32)], 1)
    g = fwht64_f32(W.reshape(-1, GROUP))
    s = np.maximum(np.abs(g).max(1), np.float32(1e-8)).astype(np.float32)
    return (g / s[:, None]).astype(np.float32), s


def pack_dist(x: np.ndarray, C: np.ndarray) -> np.ndarray:
    """[n, 4] x [k, 4] -> [n, k] squared distances in the kernels' fp32 order."""
    d = (x[:, None, :] - C[None, :, :]).astype(np.float32)
    q = (d * d).astype(np.float32)
    return ((q[..., 0] + q[..., 1]) + q[..., 2]) + q[..., 3]


def pack_nearest(x: np.ndarray, C: np.ndarray, chunk: int = 4096) -> np.ndarray:
    """Nearest centroid, lowest index on ties (vq2_kernel.py:54 and :62, argmin of distances)."""
    out = np.empty(x.shape[0], np.int64)
    for i in range(0, x.shape[0], chunk):
        out[i:i + chunk] = pack_dist(x[i:i + chunk], C).argmin(1)
    return out


def pack_kmeans(samp: np.ndarray, C: np.ndarray, iters: int) -> np.ndarray:
    """Lloyd iterations: assign, then each centroid with members = their mean, others kept
    (vq2_kernel.py:53-58)."""
    C = np.asarray(C, np.float32).copy()
    k = C.shape[0]
    q = np.rint(samp.astype(np.float64) * PACK_FIX).astype(np.int64)
    for _ in range(iters):
        a = pack_nearest(samp, C)
        sums = np.zeros((k, 4), np.int64)
        np.add.at(sums, a, q)
        cnt = np.bincount(a, minlength=k)
        nz = cnt > 0
        C[nz] = ((sums[nz].astype(np.float64) * 2.0 ** -40) / cnt[nz, None]).astype(np.float32)
    return C


def pack_from_sample(W: np.ndarray, si: np.ndarray, init: np.ndarray, iters: int):
    """The whole packer for a given sample (sub-vector indices si, initial codebook = sample rows
    init): returns (C, idx [rows, nsub], scale [rows, ng], dq [rows, D]) (vq2_kernel.py:37-65)."""
    rows, D = np.asarray(W).shape
    wn, s = pack_rotate(W)
    vec = wn.reshape(-1, VDIM)
    samp = vec[np.asarray(si)]
    C = pack_kmeans(samp, samp[np.asarray(init)], iters)
    idx = pack_nearest(vec, C)
    recon = (C[idx].reshape(-1, GROUP) * s[:, None]).astype(np.float32)
    ng = wn.shape[0] // rows
    dq = fwht64_f32(recon).reshape(rows, ng * GROUP)[:, :D]
    return C, idx.reshape(rows, -1), s.reshape(rows, ng), dq
