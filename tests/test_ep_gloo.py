"""Expert-parallel dispatch / combine bookkeeping on CPU gloo ranks (world size 2 and 4).

The expert compute is the oracle's dense MoE restricted to the rank's expert window, so the test
checks the partition, the all-to-all split sizes, the dedup of tokens per destination rank and
the combine against a single-process run of the same layer."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, fail_rank):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "deepseek-v4-flash-2bit-gb10_b200"))
    sys.path.insert(0, os.path.dirname(here))
    from oracle import torch_ref
    from vq2_vllm import ep, synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        E, H, I = 8, 128, 64
        layer = synth.make_layer(E, H, I, seed=0)
        local = ep.local_layer(layer, rank, world)
        x = synth.make_tokens(6, H, seed=10 + rank)
        ids, w = synth.route_uniform(6, E, 3, seed=20 + rank)

        def fn(xr, idr, wr, base, E_local):
            return torch_ref.moe_ref(xr, idr, wr, local, expert_base=base, E=E_local)

        if rank == fail_rank:
            raise RuntimeError("injected failure before dispatch")
        out = ep.ep_moe(x, ids, w, fn, E)
        out_g = ep.ep_moe_gather(x, ids, w, fn, E)
        ref = torch_ref.moe_ref(x, ids, w, layer)
        # a load-balanced placement (the same on every rank: loads of a shared calibration draw):
        # ids relabelled to virtual slots, each rank holding its placed experts
        cal, _ = synth.route_uniform(64, E, 3, seed=99)
        order, virt = ep.balanced_placement(torch.bincount(cal.flatten().long(), minlength=E), world)
        local_p = ep.local_layer_placed(layer, order, rank, world)

        def fn_p(xr, idr, wr, base, E_local):
            return torch_ref.moe_ref(xr, idr, wr, local_p, expert_base=base, E=E_local)

        out_p = ep.ep_moe(x, virt[ids.long()], w, fn_p, E)
        q.put((rank, "ok", max(torch_ref.rel_l2(out, ref), torch_ref.rel_l2(out_g, ref), torch_ref.rel_l2(out_p, ref))))
    except Exception as ex:  # reported to the parent
        q.put((rank, "error", repr(ex)))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return sorted(res)


@pytest.mark.parametrize("world", [2, 4])
def test_ep_matches_single_device(world):
    res = _run(world)
    for rank, status, val in res:
        assert status == "ok", val
        assert val < 1e-5


def test_dispatch_plan_dedups_tokens_per_rank():
    from vq2_vllm import ep
    ids = torch.tensor([[0, 1, 5], [6, 7, 2], [3, 3, 3]])
    n_idx, counts = ep.dispatch_plan(ids, 8, 2)
    assert counts.tolist() == [3, 2]                # rank 0: tokens 0,1,2; rank 1: tokens 0,1
    assert n_idx.tolist() == [0, 1, 2, 0, 1]


def test_failed_rank_surfaces_as_error_on_the_others():
    """A rank that dies before the dispatch makes the survivors' collective fail (bounded by the
    process-group timeout) instead of hanging."""
    res = _run(2, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    assert res[0][1] == "error"


def test_exchange_region_layout():
    """Every field of the peer-exchange region is 256-byte aligned, in order, and sized for the
    step's largest token count (the kernels rely on 16-byte alignment of every slot)."""
    from vq2_vllm import ep
    for world in (1, 2, 8):
        for n_max in (1, 4, 32):
            lay = ep.P2PExchange.layout(world, n_max, 4096, 8, 4096 * 2)
            names = ["x", "ids", "w", "comb", "dflag", "cflag", "epoch"]
            offs = [lay[n] for n in names] + [lay["bytes"]]
            assert all(o % 256 == 0 for o in offs)
            assert offs == sorted(offs)
            assert lay["ids"] - lay["x"] >= world * n_max * 8192
            assert lay["dflag"] - lay["comb"] >= world * n_max * 4096 * 4
            assert lay["cflag"] - lay["dflag"] >= world * ep.EP_CTAS * 4


def test_balanced_placement_evens_a_zipf_load():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "deepseek-v4-flash-2bit-gb10_b200"))
    from vq2_vllm import ep, synth
    E, W = 256, 8
    ids, _ = synth.route_zipf(8192, E, 8, s=1.1, seed=5, draw_seed=6)
    load = torch.bincount(ids.flatten().long(), minlength=E).double()
    order, virt = ep.balanced_placement(load, W)
    assert sorted(order.tolist()) == list(range(E))                 # a permutation
    assert torch.equal(virt[order], torch.arange(E))
    per = E // W
    placed = torch.stack([load[order[r * per:(r + 1) * per]].sum() for r in range(W)])
    contiguous = load.view(W, per).sum(1)
    assert placed.max() / placed.mean() < 1.1                     # contiguous: about 1.6-2.5
    assert placed.max() < contiguous.max()
