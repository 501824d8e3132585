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


def local_layer(layer: dict, rank: int, world: int) -> dict:
    """This rank's slice of a full layer dict (experts [rank*E/W, (rank+1)*E/W))."""
    E = layer["w13_lo"].shape[0]
    per = E // world
    return {k: (v[rank * per:(rank + 1) * per] if v.dim() == 3 else v) for k, v in layer.items()}


def cuda_expert_fn(local: dict):
    """expert_fn running the B200 kernels on a rank's local expert slice (decode for small
    batches, the tcgen05 grouped GEMM above the decode pair limit)."""
    from . import synth
    from .kernels.vq2_kernel import vq2_moe_fused_10b

    def fn(x, ids, w, expert_base, E_local):
        return vq2_moe_fused_10b(x, ids, w, *synth.layer_args(local), expert_base=expert_base)

    return fn


# ----------------------------------------------------------------------------- benchmark (N > 1)
def bench_ep(args, rank, world, metric):
    """Weak-scaling expert-parallel decode: every rank contributes `per_rank` decode tokens per
    step (1 = the config-1 batch per rank); the 256 experts are split over the ranks. Device time
    with CUDA events, the max over ranks."""
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

    def run(per_rank, steps, warmup):
        xs = [synth.make_tokens(per_rank, H, seed=50 + 97 * rank + j, device=dev) for j in range(8)]
        rs = [synth.route_uniform(per_rank, E, K, seed=500 + 97 * rank + j, device=dev) for j in range(8)]
        gather = per_rank * world <= 512
        moe = ep_moe_gather if gather else ep_moe
        step = lambda i: moe(xs[i % 8], rs[i % 8][0], rs[i % 8][1], fns[i % nlayers], E)
        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        if gather:
            # the gather-mode step has no host read: replay it from CUDA graphs, one per input set
            try:
                gs = []
                for j in range(8):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        step(j)
                    gs.append(g)
                torch.cuda.synchronize()
                dist.barrier()
                step = lambda i: gs[i % 8].replay()
                graphs_used[per_rank] = True
            except Exception as ex:            # fall back to eager launches
                graphs_used[per_rank] = f"eager ({type(ex).__name__})"
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for i in range(steps):
            step(i)
        e.record()
        e.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        return ms.item()

    ms1 = run(1, args.steps, max(args.warmup, 3))
    extra = {}
    for total in (64, 256):
        if total % world == 0:
            m = run(total // world, max(3, args.steps // 4), 3)
            extra[f"config3_{total}_tokens"] = {"ms_per_step": m, "us_per_token": m * 1e3 / total}
    if rank == 0:
        line = {"metric": metric, "value": ms1 * 1e3 / world, "unit": "us/token", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms1,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16x2+f32 (10-bit VQ indices, fp16 codebook/scales)",
                "data": "synthetic (seeded per-rank expert shards, uniform top-8 routing)",
                "config": {"workload": "expert-parallel decode, 1 token per rank per step",
                           "H": H, "I": I, "E": E, "topk": K, "experts_per_rank": per,
                           "parallelism": f"ep{world}", "l2": f"{nlayers} layers cycled"},
                "ep": extra, "cuda_graphs": {str(k): v for k, v in graphs_used.items()},
                "gpu_launches": 2 * args.steps}
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()
