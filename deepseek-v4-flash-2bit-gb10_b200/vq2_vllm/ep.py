"""Expert parallelism for the vq2 MoE layer: experts partitioned over ranks, NCCL all-to-all
dispatch and combine.

The reference runs on one device and has no parallel code; this module adds the one strategy the
B200 build needs. Rank r of W owns experts [r*E/W, (r+1)*E/W) and holds only their index planes
and scales (codebooks are replicated). One layer call:

  1. every rank decides, per token, the set of destination ranks that own at least one of its
     top-k experts; a token goes to each such rank once (not once per expert);
  2. per-destination counts are exchanged (all_to_all of int64 [W]);
  3. dispatch: all_to_all of the token rows (activation dtype), their global expert ids and
     routing weights, with those split sizes;
  4. each rank runs the local MoE (the CUDA decode or prefill path) on what it received, with its
     expert window, so pairs owned elsewhere are skipped;
  5. combine: all_to_all of the fp32 partial outputs back to the source ranks, which add them
     into their tokens' rows.

Split sizes are read on the host (one device-to-host read of W counts per call), so a call is
not capturable in a CUDA graph.

Decode-sized batches use ``ep_moe_gather`` instead: one all_gather of every rank's packed
(x, ids, w) rows and one reduce_scatter of the fp32 partial outputs — two collectives, no host
read, every rank applies only its expert window to all gathered tokens.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def owner_mask(topk_ids: torch.Tensor, E: int, world: int) -> torch.Tensor:
    """[N, W] bool: token n has at least one expert owned by rank d (contiguous partition)."""
    per = E // world
    dest = (topk_ids.long() // per).clamp_(0, world - 1)
    mask = torch.zeros(topk_ids.shape[0], world, dtype=torch.bool, device=topk_ids.device)
    mask.scatter_(1, dest, True)
    return mask


def dispatch_plan(topk_ids: torch.Tensor, E: int, world: int):
    """Send order (token index per sent row, grouped by destination rank) and per-rank counts."""
    mask = owner_mask(topk_ids, E, world)
    d_idx, n_idx = torch.nonzero(mask.t(), as_tuple=True)       # sorted by destination, then token
    counts = mask.sum(0).to(torch.int64)
    return n_idx, counts


def _a2a(out_t, in_t, out_splits, in_splits, group):
    dist.all_to_all_single(out_t, in_t, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


def ep_moe(x, topk_ids, topk_w, expert_fn, E: int, group=None, combine_dtype=torch.float32):
    """Expert-parallel MoE layer call. ``expert_fn(x, ids, w, expert_base, E_local) -> fp32 [n, H]``
    computes this rank's experts on the received rows. Returns fp32 [N, H] for the local tokens."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if E % world:
        raise ValueError(f"vq2 ep: {E} experts do not split evenly over {world} ranks")
    per = E // world
    N, H = x.shape
    k = topk_ids.shape[1]
    n_idx, counts = dispatch_plan(topk_ids, E, world)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    send_splits = counts.tolist()
    recv_splits = recv_counts.tolist()
    n_recv = int(sum(recv_splits))

    xs = x.index_select(0, n_idx).contiguous()
    ids_s = topk_ids.index_select(0, n_idx).to(torch.int32).contiguous()
    w_s = topk_w.float().index_select(0, n_idx).contiguous()
    xr = torch.empty(n_recv, H, dtype=x.dtype, device=x.device)
    idr = torch.empty(n_recv, k, dtype=torch.int32, device=x.device)
    wr = torch.empty(n_recv, k, dtype=torch.float32, device=x.device)
    _a2a(xr, xs, recv_splits, send_splits, group)
    _a2a(idr, ids_s, recv_splits, send_splits, group)
    _a2a(wr, w_s, recv_splits, send_splits, group)

    if n_recv:
        part = expert_fn(xr, idr, wr, rank * per, per).to(combine_dtype).contiguous()
    else:
        part = torch.empty(0, H, dtype=combine_dtype, device=x.device)
    back = torch.empty(n_idx.numel(), H, dtype=combine_dtype, device=x.device)
    _a2a(back, part, send_splits, recv_splits, group)
    out = torch.zeros(N, H, dtype=torch.float32, device=x.device)
    out.index_add_(0, n_idx, back.float())
    return out


def ep_moe_gather(x, topk_ids, topk_w, expert_fn, E: int, group=None):
    """Expert-parallel MoE for small per-rank batches (every rank the same N): all_gather of the
    packed token rows, local experts applied to all of them, reduce_scatter of the partial sums."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if E % world:
        raise ValueError(f"vq2 ep: {E} experts do not split evenly over {world} ranks")
    per = E // world
    N, H = x.shape
    k = topk_ids.shape[1]
    xb = H * x.element_size()
    row = torch.cat([x.contiguous().view(torch.uint8).view(N, xb),
                     topk_ids.to(torch.int32).contiguous().view(torch.uint8).view(N, 4 * k),
                     topk_w.float().contiguous().view(torch.uint8).view(N, 4 * k)], 1)
    allrows = torch.empty(world * N, row.shape[1], dtype=torch.uint8, device=x.device)
    dist.all_gather_into_tensor(allrows, row, group=group)
    xa = allrows[:, :xb].contiguous().view(x.dtype).view(world * N, H)
    ia = allrows[:, xb:xb + 4 * k].contiguous().view(torch.int32).view(world * N, k)
    wa = allrows[:, xb + 4 * k:].contiguous().view(torch.float32).view(world * N, k)
    part = expert_fn(xa, ia, wa, rank * per, per).float().contiguous()
    out = torch.empty(N, H, dtype=torch.float32, device=x.device)
    if dist.get_backend(group) == "gloo":        # gloo has no reduce_scatter
        dist.all_reduce(part, group=group)
        out.copy_(part[rank * N:(rank + 1) * N])
    else:
        dist.reduce_scatter_tensor(out, part, group=group)
    return out


EP_CTAS = 8          # VQ2_EP_CTAS of the C ABI: flags per source rank


class _DevBuf:
    """A raw device allocation exposed to torch (no ownership) through __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def _up256(v: int) -> int:
    return (v + 255) & ~255


class P2PUnavailable(RuntimeError):
    """Peer mapping failed on some rank; every rank raises it together."""


class P2PExchange:
    """Token exchange of decode-sized expert-parallel steps over NVLink peer memory (the C ABI's
    vq2_ep_dispatch / vq2_ep_combine). Each rank allocates one exchange region, shares it through a
    CUDA IPC handle (exchanged with all_gather_object) and maps every peer's region; a step is one
    dispatch kernel (rows pushed to every rank, a flag per source) and one combine kernel (partial
    outputs pushed to the owning rank, summed there in source order). Every rank must call the
    same sequence with the same N (<= n_max). No host synchronisation: a step can be captured in
    a CUDA graph."""

    def __init__(self, n_max: int, H: int, k: int, x_dtype=torch.bfloat16, group=None):
        import ctypes
        from . import _lib
        self._lib = _lib
        L = _lib.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_max, self.H, self.k, self.x_dtype = n_max, H, k, x_dtype
        self.row_x = H * torch.tensor([], dtype=x_dtype).element_size()
        if self.row_x % 16:
            raise ValueError("vq2 ep: token rows must be a multiple of 16 bytes")
        W = self.world
        lay = self.layout(W, n_max, H, k, self.row_x)
        self.off_x, self.off_ids, self.off_w, self.off_comb = lay["x"], lay["ids"], lay["w"], lay["comb"]
        self.off_dflag, self.off_cflag, self.off_epoch = lay["dflag"], lay["cflag"], lay["epoch"]
        self.off_count = lay["count"]
        self.nbytes = lay["bytes"]
        dev = torch.device("cuda", torch.cuda.current_device())
        p = ctypes.c_void_p()
        _lib.check(L.vq2_ep_alloc(self.nbytes, ctypes.byref(p)), "vq2_ep_alloc")
        self.base = p.value
        self.region = torch.as_tensor(_DevBuf(self.base, self.nbytes), device=dev)
        h = (ctypes.c_char * 64)()
        _lib.check(L.vq2_ipc_get_handle(self.base, h), "vq2_ipc_get_handle")
        handles = [None] * W
        dist.all_gather_object(handles, bytes(h), group=group)
        self._opened = []
        rows = []
        ok = 1
        for r in range(W):
            if r == self.rank:
                b = self.base
            else:
                q = ctypes.c_void_p()
                if L.vq2_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(q)) != 0:
                    ok, b = 0, 0
                else:
                    b = q.value
                    self._opened.append(b)
            rows.append([b + self.off_x, b + self.off_ids, b + self.off_w, b + self.off_comb,
                         b + self.off_dflag, b + self.off_cflag])
        # every rank learns whether every rank mapped every peer (so all fall back together)
        flag = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        if flag.item() == 0:
            self.close()
            raise P2PUnavailable("vq2 ep: a rank could not map a peer's exchange region (CUDA IPC)")
        self.peers = torch.tensor(rows, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group=group)            # every region is zeroed and mapped before any push

    @staticmethod
    def layout(world: int, n_max: int, H: int, k: int, row_x: int) -> dict:
        """Byte offsets of the exchange region's fields (the layout of include/vq2_b200.h), each
        256-byte aligned, and the region size."""
        sizes = (("x", world * n_max * row_x), ("ids", world * n_max * k * 4), ("w", world * n_max * k * 4),
                 ("comb", world * n_max * H * 4), ("dflag", world * EP_CTAS * 4), ("cflag", world * EP_CTAS * 4),
                 ("epoch", 16), ("count", 16))
        out, o = {}, 0
        for name, size in sizes:
            out[name] = o
            o = _up256(o + size)
        out["bytes"] = o
        return out

    def gathered(self, N: int):
        """Views of the gathered rows in source-rank order: x [W*N, H], ids i32 [W*N, k], w f32 [W*N, k]."""
        W, r = self.world, self.region
        xa = r[self.off_x:self.off_x + W * N * self.row_x].view(self.x_dtype).view(W * N, self.H)
        ia = r[self.off_ids:self.off_ids + W * N * self.k * 4].view(torch.int32).view(W * N, self.k)
        wa = r[self.off_w:self.off_w + W * N * self.k * 4].view(torch.float32).view(W * N, self.k)
        return xa, ia, wa

    @staticmethod
    def _aligned(t):
        t = t.contiguous()
        return t if t.data_ptr() % 16 == 0 else t.clone()

    def dispatch(self, x, topk_ids, topk_w):
        N = x.shape[0]
        if N > self.n_max or x.dtype != self.x_dtype or x.shape[1] != self.H or topk_ids.shape[1] != self.k:
            raise ValueError("vq2 ep: step does not fit the exchange region")
        x = self._aligned(x)
        if topk_ids.dtype not in (torch.int32, torch.int64):
            topk_ids = topk_ids.to(torch.int32)
        ids = self._aligned(topk_ids)               # i64 ids are narrowed by the dispatch kernel
        w = self._aligned(topk_w.float())
        self._lib.check(self._lib.lib().vq2_ep_dispatch(
            x.data_ptr(), ids.data_ptr(), 1 if ids.dtype == torch.int64 else 0, w.data_ptr(), N, self.row_x, self.k,
            self.peers.data_ptr(), self.world,
            self.rank, self.base, self.off_dflag, self.off_epoch, self._lib.stream_ptr()), "vq2_ep_dispatch")
        return self.gathered(N)

    def combine(self, part, N: int):
        part = self._aligned(part.float())
        out = torch.empty(N, self.H, dtype=torch.float32, device=part.device)
        self._lib.check(self._lib.lib().vq2_ep_combine(
            part.data_ptr(), N, self.H, self.peers.data_ptr(), self.world, self.rank, self.base, self.off_comb,
            self.off_cflag, self.off_epoch, out.data_ptr(), self._lib.stream_ptr()), "vq2_ep_combine")
        return out

    def decode(self, x, topk_ids, topk_w, local: dict, E: int):
        """One decode step with the exchange fused into the decode kernels (vq2_ep_decode): this
        rank's rows go to every rank, this rank's experts (``local``, experts
        [rank*E/W, (rank+1)*E/W) of an E-expert layer) run on all ranks' rows, and every result
        is added into its owner's output over NVLink. Returns fp32 [N, H] for this rank's tokens."""
        from . import synth
        from .kernels.vq2_kernel import _prep
        L = self._lib.lib()
        N, k = x.shape[0], topk_ids.shape[1]
        if N > self.n_max or x.dtype != self.x_dtype or x.shape[1] != self.H or k != self.k:
            raise ValueError("vq2 ep: step does not fit the exchange region")
        if E % self.world:
            raise ValueError(f"vq2 ep: {E} experts do not split evenly over {self.world} ranks")
        per = E // self.world
        t = _prep(x, topk_ids, topk_w, *synth.layer_args(local))
        t[0] = self._aligned(t[0])
        out = torch.empty(N, self.H, dtype=torch.float32, device=x.device)
        a = self._lib.moe_args(*t, out, expert_base=self.rank * per, E=per)
        if not hasattr(self, "_lay"):
            self._lay = self._lib.Vq2EpLayout(self.off_x, self.off_ids, self.off_w, self.off_comb, self.off_dflag,
                                              self.off_cflag, self.off_epoch, self.off_count)
        stream = self._lib.stream_ptr()
        nb = L.vq2_ep_decode_workspace_size(self.world, N, k, a.H, a.I)
        ws = self._lib.workspace(nb, x.device, stream)
        self._lib.check(L.vq2_ep_decode(a, self.peers.data_ptr(), self.world, self.rank, self.base, self._lay,
                                        ws.data_ptr(), ws.numel(), stream), "vq2_ep_decode")
        return out

    def close(self):
        torch.cuda.synchronize()
        L = self._lib.lib()
        for b in self._opened:
            L.vq2_ipc_close(b)
        self._opened = []
        if self.base:
            L.vq2_ep_free(self.base)
            self.base = 0


def ep_moe_p2p(x, topk_ids, topk_w, expert_fn, E: int, exch: P2PExchange):
    """ep_moe_gather over NVLink peer memory: the gathered rows land in the exchange region (no
    packing copies), this rank's experts run on them, and the partial outputs return to their
    owners through the same region."""
    world, rank = exch.world, exch.rank
    if E % world:
        raise ValueError(f"vq2 ep: {E} experts do not split evenly over {world} ranks")
    per = E // world
    N = x.shape[0]
    xa, ia, wa = exch.dispatch(x, topk_ids, topk_w)
    part = expert_fn(xa, ia, wa, rank * per, per)
    return exch.combine(part, N)


def ep_moe_p2p_fused(x, topk_ids, topk_w, local: dict, E: int, exch: P2PExchange):
    """ep_moe_p2p with the exchange inside the decode kernels (P2PExchange.decode)."""
    return exch.decode(x, topk_ids, topk_w, local, E)


def balanced_placement(load: torch.Tensor, world: int):
    """Expert placement from per-expert loads (e.g. routed-pair counts of a calibration batch):
    returns ``(order, virt)``, int64 [E] each. ``order[v]`` is the global expert held in virtual
    slot v, ranks holding the contiguous virtual slots [r*E/W, (r+1)*E/W) as before, and
    ``virt[e]`` its inverse. Greedy longest-processing-time: experts by load, heaviest first, each
    to the rank with the least load that still has room, so every rank holds E/W experts and the
    per-rank loads are as even as that greedy makes them. Relabel a step's ids with ``virt[ids]``
    and give rank r the experts ``order[r*E/W:(r+1)*E/W]`` (``local_layer_placed``); the exchange
    and the kernels are unchanged."""
    E = load.numel()
    if E % world:
        raise ValueError(f"vq2 ep: {E} experts do not split evenly over {world} ranks")
    per = E // world
    lsum = [0.0] * world
    slots = [[] for _ in range(world)]
    for e in torch.argsort(load.double().cpu(), descending=True, stable=True).tolist():
        r = min((r for r in range(world) if len(slots[r]) < per), key=lambda r: (lsum[r], r))
        slots[r].append(e)
        lsum[r] += float(load[e])
    order = torch.tensor([e for r in range(world) for e in sorted(slots[r])], dtype=torch.int64)
    virt = torch.empty_like(order)
    virt[order] = torch.arange(E, dtype=torch.int64)
    return order, virt


def local_layer_placed(layer: dict, order: torch.Tensor, rank: int, world: int) -> dict:
    """This rank's experts under a placement (``balanced_placement``): the experts
    ``order[rank*E/W:(rank+1)*E/W]`` of a full layer dict, in that order."""
    E = order.numel()
    per = E // world
    sel = order[rank * per:(rank + 1) * per]
    return {k: (v.index_select(0, sel.to(v.device)) if v.dim() == 3 else v) for k, v in layer.items()}


def local_layer(layer: dict, rank: int, world: int) -> dict:
    """This rank's slice of a full layer dict (experts [rank*E/W, (rank+1)*E/W))."""
    E = layer["w13_lo"].shape[0]
    per = E // world
    return {k: (v[rank * per:(rank + 1) * per] if v.dim() == 3 else v) for k, v in layer.items()}


def load_local_layer(path: str, rank: int, world: int, device="cpu") -> dict:
    """This rank's experts of one ``experts_fused_layer_{L}.safetensors`` file, read as slices of
    the file (the other ranks' experts are never read)."""
    from safetensors import safe_open
    from .plugin import read_fused_layer
    with safe_open(path, "pt") as f:
        E = f.get_slice("w13_lo").get_shape()[0]
    if E % world:
        raise ValueError(f"vq2 ep: {E} experts do not split evenly over {world} ranks")
    per = E // world
    return read_fused_layer(path, device=device, expert_range=(rank * per, (rank + 1) * per))


def cuda_expert_fn(local: dict):
    """expert_fn running the B200 kernels on a rank's local expert slice (decode for small
    batches, the tcgen05 grouped GEMM above the decode pair limit)."""
    from . import synth
    from .kernels.vq2_kernel import vq2_moe_fused_10b

    def fn(x, ids, w, expert_base, E_local):
        return vq2_moe_fused_10b(x, ids, w, *synth.layer_args(local), expert_base=expert_base)

    return fn


# ----------------------------------------------------------------------------- benchmark (N > 1)
def bench_ep(args, rank, world, metric, clocks_cls=None, peaks_fn=None):
    """Weak-scaling expert-parallel decode: every rank contributes `per_rank` decode tokens per
    step (1 = the config-1 batch per rank); the 256 experts are split over the ranks. Device time
    with CUDA events, the max over ranks. `clocks_cls` samples the GPU clocks during the timed
    steps (rank 0's GPU); `peaks_fn` gives the measured HBM peak for the roofline figure."""
    import json
    import os
    import time

    from . import synth
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl", device_id=dev)
    H, I, E, K = 4096, 2048, 256, 8
    per = E // world
    nlayers = 4
    layers = []
    for l in range(nlayers):   # each rank materialises only its experts (seeded per rank and layer)
        full = synth.make_layer(per, H, I, seed=1000 * l + rank, device=dev)
        layers.append(full)
    fns = [cuda_expert_fn(L) for L in layers]

    graphs_used = {}
    use_p2p = os.environ.get("VQ2_EP_P2P", "1") != "0"
    exchanges = {}
    # the headline steps use the stand-alone peer-memory exchange (dispatch / decode / combine),
    # measured faster on the device than the exchange fused into the decode kernels
    # (vq2_ep_decode); VQ2_EP_FUSED=1 makes the fused step the headline. The fused step is timed
    # beside it either way.
    use_fused = use_p2p and os.environ.get("VQ2_EP_FUSED", "0") != "0"
    fexchanges = {}
    fused_used = {}
    idx_bytes_per_expert = 3 * H * I // 4 + 3 * H * I // 16      # lo + hi planes, gate/up/down

    def local_distinct(per_rank):
        """Mean over the 8 input sets of the distinct experts this rank serves per step (every
        rank's routing is rebuilt from its seed, so no communication is needed)."""
        tot = 0
        for j in range(8):
            ids = torch.cat([synth.route_uniform(per_rank, E, K, seed=500 + 97 * r + j, device=dev)[0]
                             for r in range(world)]).long()
            mine = ids[(ids >= rank * per) & (ids < (rank + 1) * per)]
            tot += torch.unique(mine).numel()
        return tot / 8

    def run(per_rank, steps, warmup, collective_only=False, fused=None):
        fused = use_fused if fused is None else fused
        xs = [synth.make_tokens(per_rank, H, seed=50 + 97 * rank + j, device=dev) for j in range(8)]
        rs = [synth.route_uniform(per_rank, E, K, seed=500 + 97 * rank + j, device=dev) for j in range(8)]
        gather = per_rank * world <= 512
        moe = ep_moe_gather if gather else ep_moe
        if gather and use_p2p:               # NVLink peer-memory exchange (one region per size)
            if per_rank not in exchanges:
                try:
                    exchanges[per_rank] = P2PExchange(per_rank, H, K)
                except P2PUnavailable:
                    exchanges[per_rank] = None      # all ranks fall back to NCCL together
            exch = exchanges[per_rank]
            if exch is not None:
                moe = lambda x, ids, w, fn, E_: ep_moe_p2p(x, ids, w, fn, E_, exch)
        fexch = None
        if fused and not collective_only and per_rank * world * K <= 512 and exchanges.get(per_rank):
            if per_rank not in fexchanges:
                fexchanges[per_rank] = P2PExchange(per_rank, H, K)
            fexch = fexchanges[per_rank]
            if fused == use_fused:
                fused_used[per_rank] = True
        if fexch is not None:
            step = lambda i: fexch.decode(xs[i % 8], rs[i % 8][0], rs[i % 8][1], layers[i % nlayers], E)
        elif collective_only:      # the same exchange with an expert function that does no work
            zero = lambda x, ids, w, base, El: torch.zeros(x.shape[0], H, device=x.device)
            step = lambda i: moe(xs[i % 8], rs[i % 8][0], rs[i % 8][1], zero, E)
        else:
            step = lambda i: moe(xs[i % 8], rs[i % 8][0], rs[i % 8][1], fns[i % nlayers], E)
        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        block = 1                              # steps per launch unit
        if gather:
            # the gather-mode step has no host read: the timed steps are captured as one CUDA
            # graph of consecutive steps (input sets and layers in turn, as a model's decode graph
            # holds its layers), so the kernels keep their programmatic-launch overlap across step
            # boundaries. A graph holds `steps` steps (up to 64) or the largest divisor of `steps`
            # in [8, 64], replayed steps / block times; without one, eight one-step graphs (one per
            # input set and layer) replayed in turn. Exactly `steps` steps are timed.
            try:
                block = steps if steps <= 64 else max([b for b in range(8, 65) if steps % b == 0], default=1)
                torch.cuda.synchronize()
                gks = []
                for gi in range(1 if block > 1 else 8):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        for j in range(block):
                            step(gi + j)
                    gks.append(g)
                torch.cuda.synchronize()
                for g in gks:
                    g.replay()                 # untimed: each graph's first launch
                torch.cuda.synchronize()
                dist.barrier()
                step = lambda i: gks[i % len(gks)].replay()
                if not collective_only:
                    graphs_used[per_rank] = (f"one graph of {block} steps" if block > 1
                                             else "one graph per step, 8 cycled")
            except Exception as ex:            # fall back to eager launches
                block = 1
                if not collective_only:
                    graphs_used[per_rank] = f"eager ({type(ex).__name__})"
                torch.cuda.synchronize()
        nunits = steps // block
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda._sleep(5_000_000)          # every rank queues its steps ahead of its GPU, so the
        s.record()                            # timed region sees device time, not launch gaps
        for i in range(nunits):
            step(i)
        e.record()
        e.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / (nunits * block)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        return ms.item()

    def run_stack(tokens_total=65536, nl=8, reps=2):
        """Config 4: a stack of `nl` seeded layers over `tokens_total` tokens (tokens_total / W per
        rank), Zipf(1.1) top-8 per layer (one expert popularity per layer, shared by the ranks),
        x = x + moe(x) in bf16, NCCL all-to-all dispatch and combine, each rank's experts on the
        grouped GEMM (fp8). Timed twice: experts placed contiguously, and placed by
        `balanced_placement` from the per-expert loads of a separate calibration draw of the same
        popularity (ids relabelled; every rank derives the same placement from the summed
        counts). Whole-stack time on the device, max over ranks."""
        n = tokens_total // world
        Ls = [synth.make_layer(per, H, I, seed=5000 + 100 * l + rank, device=dev) for l in range(nl)]
        sfns = [cuda_expert_fn(L) for L in Ls]
        x0 = synth.make_tokens(n, H, seed=6000 + rank, device=dev)
        routes = [synth.route_zipf(n, E, K, s=1.1, seed=7000 + l, device=dev, draw_seed=7100 + 100 * l + rank)
                  for l in range(nl)]
        placed = []
        for l in range(nl):             # calibration: the same popularity, another draw
            cal, _ = synth.route_zipf(n, E, K, s=1.1, seed=7000 + l, device=dev, draw_seed=9100 + 100 * l + rank)
            cnt = torch.bincount(cal.flatten().long(), minlength=E).double()
            dist.all_reduce(cnt)
            _, virt = balanced_placement(cnt, world)
            placed.append((virt.to(dev)[routes[l][0].long()].to(torch.int32), routes[l][1]))

        def imbalance(rts):             # pairs per owning rank, summed over the ranks
            out = []
            for ids, _ in rts:
                cnt = torch.bincount((ids.long() // per).flatten(), minlength=world).float()
                dist.all_reduce(cnt)
                out.append(round((cnt.max() / cnt.mean()).item(), 3))
            return out

        def timed(rts):
            def stack_step():
                x = x0
                for l in range(nl):
                    x = x + ep_moe(x, *rts[l], sfns[l], E).to(x.dtype)
                return x

            stack_step()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            for _ in range(reps):
                stack_step()
            e.record()
            e.synchronize()
            ms = torch.tensor([s.elapsed_time(e) / reps], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            return ms.item()

        ms_c = timed(routes)
        ms = timed(placed)
        flops = nl * (2.0 * tokens_total * K * H * 2 * I + 2.0 * tokens_total * K * I * H)
        bf16 = peaks_fn()[1] if peaks_fn is not None else 1590.0
        del Ls, sfns
        torch.cuda.empty_cache()
        return {"workload": f"config4: {nl} layers, {tokens_total} tokens ({n} per rank), Zipf(1.1) top-8, fp8, "
                            f"residual, ep{world} (NCCL all-to-all), load-balanced expert placement",
                "ms_per_stack": ms, "tok_per_s": tokens_total / (ms * 1e-3),
                "tensor_frac_per_gpu": flops / world / (ms * 1e-3) / 1e12 / (2 * bf16),
                "expert_load_max_over_mean_per_layer": imbalance(placed),
                "contiguous_placement": {"ms_per_stack": ms_c, "tok_per_s": tokens_total / (ms_c * 1e-3),
                                         "expert_load_max_over_mean_per_layer": imbalance(routes)},
                "reps": reps}

    def detail(per_rank, ms):
        """Per-GPU HBM rate on the index bytes of this rank's distinct experts (mean over ranks)
        and the exchange alone."""
        u = torch.tensor([local_distinct(per_rank)], device=dev)
        dist.all_reduce(u)
        u = u.item() / world
        coll = run(per_rank, max(3, args.steps // 4), 3, collective_only=True)
        return {"local_distinct_experts_per_rank": u,
                "local_idx_GBps_per_gpu": u * idx_bytes_per_expert / (ms * 1e-3) / 1e9,
                "exchange_only_us": coll * 1e3}

    if clocks_cls is not None and rank == 0:
        with clocks_cls(dev.index) as ck:
            ms1 = run(1, args.steps, max(args.warmup, 3))
        clocks = ck.summary()
    else:
        ms1 = run(1, args.steps, max(args.warmup, 3))
        clocks = None
    d1 = detail(1, ms1)
    if use_p2p and exchanges.get(1) is not None:    # the other exchange variant of the same step
        d1["fused_exchange_ms_per_step" if not use_fused else "standalone_exchange_ms_per_step"] = run(
            1, args.steps, max(args.warmup, 3), fused=not use_fused)

    # e2e: the public call (ep_moe_p2p / ep_moe_gather) with this rank's token row, ids and
    # weights copied in from pinned host memory and its output copied back, every step
    xh = [synth.make_tokens(1, H, seed=50 + 97 * rank + j).pin_memory() for j in range(8)]
    rh = [tuple(t.cpu().pin_memory() for t in synth.route_uniform(1, E, K, seed=500 + 97 * rank + j, device=dev))
          for j in range(8)]
    outh = torch.empty(1, H, dtype=torch.float32).pin_memory()
    exch1 = exchanges.get(1)
    fexch1 = fexchanges.get(1) if use_fused else None

    def e2e_step(i):
        x = xh[i % 8].to(dev, non_blocking=True)
        ids = rh[i % 8][0].to(dev, non_blocking=True)
        w = rh[i % 8][1].to(dev, non_blocking=True)
        if fexch1 is not None:
            out = fexch1.decode(x, ids, w, layers[i % nlayers], E)
        elif exch1 is not None:
            out = ep_moe_p2p(x, ids, w, fns[i % nlayers], E, exch1)
        else:
            out = ep_moe_gather(x, ids, w, fns[i % nlayers], E)
        outh.copy_(out, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for i in range(args.steps):
        e2e_step(i)
    e.record()
    e.synchronize()
    e2e_ms = torch.tensor([s.elapsed_time(e) / args.steps], device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()
    extra = {}
    for total in (64, 256):
        if total % world == 0:
            m = run(total // world, max(3, args.steps // 4), 3)
            extra[f"config3_{total}_tokens"] = {"ms_per_step": m, "us_per_token": m * 1e3 / total,
                                                **detail(total // world, m)}
    stack = run_stack() if os.environ.get("VQ2_BENCH_STACK", "1") == "1" else None
    p2p_used = use_p2p and all(v is not None for v in exchanges.values())
    hbm, src = (peaks_fn()[0], peaks_fn()[2]) if peaks_fn is not None else (None, None)
    achieved = d1["local_idx_GBps_per_gpu"]
    if rank == 0:
        line = {"metric": metric, "value": ms1 * 1e3 / world, "unit": "us/token", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms1,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16x2+f32 (10-bit VQ indices, fp16 codebook/scales)",
                "data": "synthetic (seeded per-rank expert shards, uniform top-8 routing)",
                "config": {"workload": "expert-parallel decode, 1 token per rank per step",
                           "H": H, "I": I, "E": E, "topk": K, "experts_per_rank": per,
                           "parallelism": f"ep{world}", "l2": f"{nlayers} layers cycled"},
                "e2e": {"value": e2e_ms * 1e3 / world, "unit": "us/token", "h2d_bytes_per_step": H * 2 + K * 8 + K * 4,
                        "d2h_bytes_per_step": H * 4, "per": "rank (every rank copies its own token in and out)"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": (achieved / hbm) if hbm else None, "traffic": None,
                             "kernel": "decode layer step per GPU (index bytes of its distinct local experts)",
                             "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src},
                "clocks": clocks,
                "ep": {"one_token_per_rank": d1, **extra,
                       "exchange": ("nvlink peer memory, fused into the decode kernels (vq2_ep_decode)"
                                    if fused_used.get(1) else
                                    "nvlink peer memory (vq2_ep_dispatch / vq2_ep_combine)" if p2p_used
                                    else "nccl all_gather + reduce_scatter"),
                       "exchange_only_us_is": "the stand-alone dispatch + combine with no expert work"},
                "cuda_graphs": {str(k): v for k, v in graphs_used.items()},
                "stack": stack,
                # this package's kernels per timed step: the two decode kernels, plus the push
                # kernel (fused exchange) or dispatch and combine (stand-alone peer-memory
                # exchange); NCCL kernels are not counted
                "gpu_launches": (3 if fused_used.get(1) else 4 if p2p_used else 2) * args.steps}
        print(json.dumps(line), flush=True)
    for ex in list(exchanges.values()) + list(fexchanges.values()):
        if ex is not None:
            ex.close()
    dist.barrier()
    dist.destroy_process_group()
