"""Benchmark of the vq2 routed-expert MoE path (BASELINE.json metric:
"vq2 MoE layer: decode us/token (% HBM roofline); prefill tok/s (% fp8 TC peak)").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one call of the MoE layer on one decode batch (config 1: H=4096, I=2048, 256 routed
experts, top-8, batch 1; batch 3 is reported beside it). Weights are seeded synthetic tensors
in the reference layout. Four independent layers (8.8 GB) are cycled step by step, so every
step streams its experts from HBM (the working set of the cycle is far above the 126 MB L2).

N > 1 (torchrun, one rank per GPU): expert-parallel decode (config 3 shapes) — experts
partitioned over the ranks, NCCL all-to-all dispatch and combine — timed as the max over ranks.

--impl reference: the reference's CPU path (fp32 dequant + matmul, restated in
oracle/torch_ref.py) on the host cores, on the same metric; rank 0 only.

--ref-gpu: the reference's own GPU kernels (an unmodified install in baseline/_ref; its prefill
extension built for sm_100a by baseline/build_ref_ext.py) timed beside ours on the same inputs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "deepseek-v4-flash-2bit-gb10_b200"))
sys.path.insert(0, HERE)

import torch  # noqa: E402

METRIC = "vq2 MoE layer: decode us/token (% HBM roofline); prefill tok/s (% fp8 TC peak)"
H, I, E, K = 4096, 2048, 256, 8
IDX_BYTES_PER_EXPERT = 3 * H * I // 4 + 3 * H * I // 16          # lo + hi planes (gate, up, down)
SC_BYTES_PER_EXPERT = 3 * H * I // 64 * 2                          # fp16 group scales
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1590.0)), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampler running during the timed region (clocks + throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p is None:
            return
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) >= 9:
                self.rows.append(f)

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_model():
    """Host CPU model name (for the CPU baselines), from /proc/cpuinfo."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# DRAM bytes (read + write) per distinct expert of one decode layer call, from the ncu capture in
# profiles/decode_config1_b1.txt (69.97 MB over 8 distinct experts, both kernels), so the roofline
# line scales it to its own run's distinct-expert count.
NCU_DECODE_BYTES_PER_EXPERT = 70.03e6 / 8


def make_routing(x, seed):
    from vq2_vllm import synth
    return synth.route_softmax_topk(x, E, K, w_std=0.02, seed=seed)


_CPU_LAYER = []


def _cpu_layer():
    if not _CPU_LAYER:
        from vq2_vllm import synth
        _CPU_LAYER.append(synth.make_layer(8, H, I, seed=0))
    return _CPU_LAYER[0]


def cpu_reference_us_per_token(threads, tokens=1, reps=1):
    """The reference's CPU dequant+matmul path (oracle/torch_ref.py) on a bounded sample:
    `tokens` decode tokens routed over 8 resident experts of the config-1 shape."""
    from oracle import torch_ref
    from vq2_vllm import synth
    torch.set_num_threads(threads)
    layer = _cpu_layer()
    x = synth.make_tokens(tokens, H, seed=1)
    ids = torch.stack([torch.randperm(8, generator=torch.Generator().manual_seed(t))[:K] for t in range(tokens)]).int()
    w = torch.full((tokens, K), 1.0 / K)
    torch_ref.moe_ref(x, ids, w, layer)                      # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        torch_ref.moe_ref(x, ids, w, layer)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts) * 1e6 / tokens, f"{tokens} token(s), top-8 over 8 resident experts, H=4096 I=2048"


def cpu_reference_prefill_tok_per_s(threads, tokens=256):
    """The reference's CPU path on a bounded prefill sample: `tokens` tokens, each routed top-8
    over 8 resident experts of the config-1 shape, i.e. `tokens` pairs per expert (256 is the
    config-2 mean, 65,536 pairs over 256 experts); scaled to config 2 (8192 tokens, 256 experts)."""
    from oracle import torch_ref
    from vq2_vllm import synth
    torch.set_num_threads(threads)
    layer = _cpu_layer()
    x = synth.make_tokens(tokens, H, seed=2)
    ids = torch.arange(8, dtype=torch.int32).repeat(tokens, 1)
    w = torch.full((tokens, K), 1.0 / K)
    t0 = time.perf_counter()
    torch_ref.moe_ref(x, ids, w, layer)
    t_sample = time.perf_counter() - t0
    t_layer = t_sample * E / 8
    return 8192 / t_layer, (f"{tokens} tokens x top-8 over 8 resident experts ({tokens} pairs per expert), "
                            f"{t_sample:.2f} s, scaled by 256/8 experts to config 2")


def time_decode_graph(layers, xs, routes, steps, stream):
    """The same decode steps replayed from CUDA graphs (one graph per (layer, input) pair of the
    cycle), as a serving engine captures decode."""
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    from vq2_vllm import synth
    nL, nX = len(layers), len(xs)
    ncyc = nL * nX // __import__("math").gcd(nL, nX)
    graphs = []
    for i in range(ncyc):
        vq2_moe_fused_10b(xs[i % nX], *routes[i % len(routes)], *synth.layer_args(layers[i % nL]))
    torch.cuda.synchronize()
    for i in range(ncyc):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            vq2_moe_fused_10b(xs[i % nX], *routes[i % len(routes)], *synth.layer_args(layers[i % nL]))
        graphs.append(g)
    for i in range(ncyc):
        graphs[i].replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    torch.cuda._sleep(5_000_000)
    s.record(stream)
    for i in range(steps):
        graphs[i % ncyc].replay()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / steps


def time_router(dev, reps=200):
    """The fused router (top-k of softmax(x @ W_r), config-1 shapes, batch 1) against the same
    formula as torch ops, both replayed from CUDA graphs; us per call."""
    from vq2_vllm.kernels.router import router_topk
    g = torch.Generator(device=dev).manual_seed(900)
    x = torch.randn(1, H, generator=g, device=dev).bfloat16()
    wr = (torch.randn(H, E, generator=g, device=dev) * 0.02).bfloat16()

    def torch_route():
        p = torch.softmax(x.float() @ wr.float(), -1)
        return torch.topk(p, K, -1)

    res = {}
    for name, f in (("ours_us", lambda: router_topk(x, wr, K)), ("torch_ops_us", torch_route)):
        for _ in range(5):
            f()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            f()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda._sleep(3_000_000)
        s.record()
        for _ in range(reps):
            gr.replay()
        e.record()
        e.synchronize()
        res[name] = s.elapsed_time(e) * 1e3 / reps
    return res


def time_pack(dev):
    """The VQ packer (offline) on 8 experts of the config-1 gate/up tensor (8 x 4096 x 4096 bf16,
    33.5M sub-vectors): the whole mirrored pack_vq2_experts_10b call (sample draw, k-means on
    200k samples for 12 iterations, assignment with planes, scales and dq) and the assignment
    kernel alone, beside the reference's assignment step as torch ops (torch.cdist + argmin over
    1M-row chunks, vq2_kernel.py:59-62) on the same normalised sub-vectors. ms, device events."""
    from vq2_vllm import _lib
    from vq2_vllm.kernels.vq2_pack import pack_vq2_experts_10b
    g = torch.Generator(device=dev).manual_seed(77)
    W3 = (torch.randn(8, 2 * I, H, generator=g, device=dev) * 0.02).bfloat16()
    rows, D = 8 * 2 * I, H
    nvec = rows * D // 4

    def ev(f, reps=2):
        f()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for _ in range(reps):
            f()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / reps

    res = {}
    out = {}
    res["pack_call_ms"] = ev(lambda: out.update(r=pack_vq2_experts_10b(W3, iters=12)))
    C = out["r"][0]
    lo = torch.empty(nvec, dtype=torch.uint8, device=dev)
    hi = torch.empty(nvec // 4, dtype=torch.uint8, device=dev)
    sc = torch.empty(rows * D // 64, dtype=torch.float32, device=dev)
    L = _lib.lib()
    res["assign_kernel_ms"] = ev(lambda: _lib.check(L.vq2_pack_assign(
        W3.data_ptr(), 0, rows, D, C.data_ptr(), C.shape[0], lo.data_ptr(), hi.data_ptr(), None, sc.data_ptr(), None,
        _lib.stream_ptr(dev)), "vq2_pack_assign"))
    from vq2_vllm.kernels.vq2_kernel import _hadamard
    Hm = _hadamard(64).to(dev)
    wn = W3.view(-1, 64).float() @ Hm
    wn = (wn / wn.abs().amax(1, keepdim=True).clamp_min(1e-8)).view(-1, 4)
    idx = torch.empty(nvec, dtype=torch.long, device=dev)

    def ref_assign():
        for i in range(0, nvec, 1 << 20):
            idx[i:i + (1 << 20)] = torch.cdist(wn[i:i + (1 << 20)], C).argmin(1)
    res["reference_ops_assign_ms"] = ev(ref_assign, reps=1)
    res["same_ids_as_reference_ops"] = float((idx == (lo.long() | ((hi.long().repeat_interleave(4) >> (
        (torch.arange(nvec, device=dev) & 3) * 2)) & 3) << 8)).float().mean().item())
    res["Gsubvectors_per_s_assign"] = nvec / (res["assign_kernel_ms"] * 1e-3) / 1e9
    del W3, wn, idx, out
    torch.cuda.empty_cache()
    return res


def time_routed_plus_shared(layers, dev):
    """Config 1, batch 1: the routed decode plus the shared expert per layer call, (a) one after
    the other on one stream and (b) co-scheduled by vq2_decode_with_shared (the shared expert's
    kernels on a partition of the SMs, concurrently with the routed ones). Four routed layers and
    four shared-weight copies cycled; 8 calls per CUDA graph, 25 replays (us per call)."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.shared_expert import moe_with_shared_expert, shared_expert_fused
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    g = torch.Generator(device=dev).manual_seed(41)
    sh = [((torch.randn(2 * I, H, generator=g, device=dev) * 0.02).bfloat16(),
           (torch.randn(H, I, generator=g, device=dev) * 0.02).bfloat16()) for _ in range(4)]
    xs = [synth.make_tokens(1, H, seed=100 + j, device=dev) for j in range(8)]
    routes = [make_routing(xs[j], seed=200 + j) for j in range(8)]
    nl = len(layers)

    def timed(step):
        for i in range(8):
            step(i)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(8):
                step(i)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        st, en = torch.cuda.Event(True), torch.cuda.Event(True)
        st.record()
        for _ in range(25):
            gr.replay()
        en.record()
        en.synchronize()
        return st.elapsed_time(en) * 1e3 / 200

    def seq(i):
        o = vq2_moe_fused_10b(xs[i % 8], *routes[i % 8], *synth.layer_args(layers[i % nl]))
        shared_expert_fused(xs[i % 8], *sh[i % 4], out=o)

    res = {"workload": "config1 batch 1: routed layer + shared expert (bf16 [4096, 4096] + [4096, 2048])",
           "sequential_us": timed(seq),
           "coscheduled_us": timed(lambda i: moe_with_shared_expert(
               xs[i % 8], *routes[i % 8], *synth.layer_args(layers[i % nl]), *sh[i % 4])),
           "shared_sms": "library default (VQ2_SHARED_SMS_DEFAULT)"}
    del sh
    torch.cuda.empty_cache()
    return res


def time_shared(dev, hbm):
    """The config-1 shared expert (bf16 gate/up [4096, 4096], down [4096, 2048]) for batch 1 and
    3: four copies of its weights (201 MB > L2) cycled, one call per copy captured in a CUDA
    graph, replayed 10 times between CUDA events (us per call); beside it the same layer as torch
    bf16 ops (two cuBLAS GEMMs and silu * mul), captured and replayed the same way."""
    from vq2_vllm.kernels.shared_expert import shared_expert_fused
    Is = I
    g = torch.Generator(device=dev).manual_seed(31)
    ws = [((torch.randn(2 * Is, H, generator=g, device=dev) * 0.02).bfloat16(),
           (torch.randn(H, Is, generator=g, device=dev) * 0.02).bfloat16()) for _ in range(4)]
    nbytes = (2 * Is * H + H * Is) * 2

    def torch_ops(x, w13, w2):
        h = torch.nn.functional.linear(x, w13)
        return torch.nn.functional.linear(torch.nn.functional.silu(h[:, :Is]) * h[:, Is:], w2)

    res = {"bytes_per_call": nbytes, "how": "CUDA graph of 4 calls (one per weight copy), 10 replays"}
    for N in (1, 3):
        x = torch.randn(N, H, generator=g, device=dev).bfloat16()
        for name, f in (("ours", lambda a, b: shared_expert_fused(x, a, b)), ("torch_ops", lambda a, b: torch_ops(x, a, b))):
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for i in range(8):
                    f(*ws[i % 4])
            torch.cuda.current_stream().wait_stream(s)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for i in range(4):
                    f(*ws[i])
            gr.replay()
            torch.cuda.synchronize()
            st, en = torch.cuda.Event(True), torch.cuda.Event(True)
            st.record()
            for _ in range(10):
                gr.replay()
            en.record()
            en.synchronize()
            us = st.elapsed_time(en) * 1e3 / 40
            res[f"{name}_us_b{N}"] = us
            if name == "ours":
                res[f"ours_GBps_b{N}"] = nbytes / (us * 1e-6) / 1e9
                res[f"ours_frac_hbm_b{N}"] = nbytes / (us * 1e-6) / 1e9 / hbm
            del gr
    del ws
    torch.cuda.empty_cache()
    return res


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps = []
    for _ in range(max(args.warmup, 0)):
        cpu_reference_us_per_token(threads)
    for _ in range(args.steps):
        v, sample = cpu_reference_us_per_token(threads)
        steps.append(v)
    v = statistics.median(steps)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "us/token", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v / 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1 decode batch 1 (CPU sample)", "H": H, "I": I, "E": E, "topk": K},
            "cpu_baseline": {"value": v, "unit": "us/token", "cores": threads, "kind": "port", "sample": sample,
                             "cpu_model": cpu_model()},
            "e2e": {"value": v, "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def time_decode(layers, xs, routes, steps, warmup, stream, soak_s=0.6):
    """CUDA-event time per step (ms), cycling layers; inputs resident in HBM."""
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
    from vq2_vllm import synth
    nL = len(layers)

    def step(i):
        L = layers[i % nL]
        ids, tw = routes[i % len(routes)]
        return vq2_moe_fused_10b(xs[i % len(xs)], ids, tw, *synth.layer_args(L))

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()                # untimed soak: clocks settle and get sampled
    i = 0
    while time.perf_counter() - t0 < soak_s:
        step(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    torch.cuda._sleep(5_000_000)          # queue ahead so host launch cost is hidden
    s.record(stream)
    for i in range(steps):
        step(i)
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / steps


def time_prefill(layers, dev, args, N=8192):
    """Config 2: one prefill layer call (8192 tokens, Zipf(1.1) top-8), both operand precisions.
    CUDA events around `reps` calls (layers cycled), after warm-up."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    _, bf16_peak, src = peaks()
    x = synth.make_tokens(N, H, seed=300, device=dev)
    ids, tw = synth.route_zipf(N, E, K, s=1.1, seed=301, device=dev)
    flops = 2.0 * N * K * H * 2 * I + 2.0 * N * K * I * H
    res = {"workload": "config2 prefill: 8192 tokens, Zipf(1.1) top-8, H=4096 I=2048 E=256",
           "algorithmic_tflop_per_call": flops / 1e12}
    reps = max(3, min(args.steps, 10))
    for prec in ("fp8", "f16"):
        for i in range(3):
            vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(layers[i % len(layers)]), precision=prec)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for i in range(reps):
            vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(layers[i % len(layers)]), precision=prec)
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / reps
        tf = flops / (ms * 1e-3) / 1e12
        peak = 2 * bf16_peak if prec == "fp8" else bf16_peak
        res[prec] = {"ms_per_call": ms, "tok_per_s": N / (ms * 1e-3), "tflops": tf,
                     "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                                  "frac": tf / peak,
                                  "peak_source": (f"2x {src} bf16 (fp8 dense rate is twice bf16)" if prec == "fp8"
                                                  else f"{src} bf16 (fp16 rate equals bf16)")}}
    return res


STACK_LAYERS, STACK_TOKENS = 8, 65536


def stack_flops(tokens=STACK_TOKENS, layers=STACK_LAYERS):
    """Algorithmic FLOPs of the config-4 stack: per layer 2*M*H*2I + 2*M*I*H over M = tokens*top-k."""
    M = tokens * K
    return layers * (2.0 * M * H * 2 * I + 2.0 * M * I * H)


def time_stack(dev, args, tokens=STACK_TOKENS):
    """Config 4 on one GPU: 8 seeded layers (all 256 experts resident), 65,536 tokens, Zipf(1.1)
    top-8 routing drawn per layer, fp8 prefill (the plugin's default), x = x + moe(x) in bf16.
    One step = the whole stack; CUDA events around `reps` steps after one warm-up step."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    _, bf16_peak, src = peaks()
    layers = [synth.make_layer(E, H, I, seed=4000 + l, device=dev) for l in range(STACK_LAYERS)]
    routes = [synth.route_zipf(tokens, E, K, s=1.1, seed=4100 + l, device=dev) for l in range(STACK_LAYERS)]
    x0 = synth.make_tokens(tokens, H, seed=4200, device=dev)
    per_layer_ms = [0.0] * STACK_LAYERS
    ev = [torch.cuda.Event(True) for _ in range(STACK_LAYERS + 1)]

    def step(record):
        x = x0
        if record:
            ev[0].record()
        for l in range(STACK_LAYERS):
            x = x + vq2_moe_grouped_wmma(x, *routes[l], *synth.layer_args(layers[l]), precision="fp8").to(x.dtype)
            if record:
                ev[l + 1].record()
        return x

    step(False)
    torch.cuda.synchronize()
    reps = max(1, min(args.steps, 3))
    tot = 0.0
    for _ in range(reps):
        step(True)
        ev[-1].synchronize()
        for l in range(STACK_LAYERS):
            per_layer_ms[l] += ev[l].elapsed_time(ev[l + 1]) / reps
        tot += ev[0].elapsed_time(ev[-1]) / reps
    fl = stack_flops(tokens) / STACK_LAYERS
    peak = 2 * bf16_peak
    out = {"workload": f"config4 stack on 1 GPU: {STACK_LAYERS} layers, {tokens} tokens, Zipf(1.1) top-8 per layer, fp8, residual",
           "ms_per_stack": tot, "tok_per_s": tokens / (tot * 1e-3),
           "per_layer_ms": [round(v, 3) for v in per_layer_ms],
           "per_layer_tensor_frac": [round(fl / (v * 1e-3) / 1e12 / peak, 4) for v in per_layer_ms],
           "tensor_frac_peak": f"2x {src} bf16 (fp8 dense rate is twice bf16)", "reps": reps}
    del layers
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world):
    from vq2_vllm import synth
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    if world > 1:
        from vq2_vllm import ep
        return ep.bench_ep(args, rank, world, METRIC, Clocks, peaks)
    hbm, _, src = peaks()
    stream = torch.cuda.current_stream()
    nlayers = 4
    layers = [synth.make_layer(E, H, I, seed=10 + l, device=dev) for l in range(nlayers)]
    res = {}
    for B in (1, 3):
        xs = [synth.make_tokens(B, H, seed=100 + j, device=dev) for j in range(8)]
        routes = [make_routing(xs[j], seed=200 + j) for j in range(8)]
        distinct = sum(torch.unique(routes[j % 8][0]).numel() for j in range(args.steps)) / args.steps
        with Clocks(dev.index) as ck:
            ms = time_decode(layers, xs, routes, args.steps, max(args.warmup, 3), stream, soak_s=args.soak)
        res[B] = (ms, distinct, ck.summary())
        if B == 1:
            ms_graph = time_decode_graph(layers, xs, routes, args.steps, stream)
    ms1, u1, clocks = res[1]
    us_tok = ms1 * 1e3 / 1
    idx_bytes = u1 * IDX_BYTES_PER_EXPERT + 1 * H * 2 + 1 * H * 4
    all_bytes = idx_bytes + u1 * SC_BYTES_PER_EXPERT + 2 * 8192
    achieved = idx_bytes / (ms1 * 1e-3) / 1e9

    # e2e: the public host-buffer API (HostDecodeSession, one per layer): every step copies its
    # token row, ids and routing weights from page-locked host memory to the device (one copy)
    # and the fp32 result back, inside the timed region; the host waits on a slot's previous step
    # before reusing it
    from vq2_vllm.kernels.vq2_kernel import HostDecodeSession
    xh = [x.cpu() for x in [synth.make_tokens(1, H, seed=100 + j) for j in range(8)]]
    rh = [(r[0].cpu(), r[1].cpu()) for r in
          [make_routing(synth.make_tokens(1, H, seed=100 + j, device=dev), 200 + j) for j in range(8)]]
    sessions = [HostDecodeSession(*synth.layer_args(L), N=1, k=K) for L in layers]

    def e2e_step(i):
        sessions[i % nlayers].step(xh[i % 8], *rh[i % 8])

    for i in range(8):
        e2e_step(i)
    torch.cuda.synchronize()
    # the timed region ends with the last download: a device-wide event after all streams joined
    t0 = time.perf_counter()
    s = torch.cuda.Event(True)
    s.record()
    for i in range(args.steps):
        e2e_step(i)
    for ss in sessions:
        torch.cuda.current_stream().wait_stream(ss.s_out)
    e = torch.cuda.Event(True)
    e.record()
    e.synchronize()
    e2e_ms = s.elapsed_time(e) / args.steps
    e2e_wall_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    h2d = sessions[0].nin                # one copy of the packed slot: x | ids | w (256-byte aligned parts)
    del sessions
    d2h = H * 4

    prefill = time_prefill(layers, dev, args)
    try:
        with_shared = time_routed_plus_shared(layers, dev)
    except Exception as ex:  # a figure beside the headline must not cost the headline line
        with_shared = {"error": f"{type(ex).__name__}: {ex}"[:300]}
    del layers
    torch.cuda.empty_cache()
    try:
        stack = time_stack(dev, args)
    except Exception as ex:  # a figure beside the headline must not cost the headline line
        stack = {"error": f"{type(ex).__name__}: {ex}"[:300]}
    router = time_router(dev)
    try:
        shared = time_shared(dev, hbm)
    except Exception as ex:  # a figure beside the path must not cost the headline line
        shared = {"error": f"{type(ex).__name__}: {ex}"[:300]}
    try:
        pack = time_pack(dev)
    except Exception as ex:  # an offline-tool figure must not cost the headline line
        pack = {"error": f"{type(ex).__name__}: {ex}"[:300]}

    cpu_v, cpu_sample = (None, None)
    cpu_pf, cpu_pf_sample = (None, None)
    if not args.no_cpu:
        cpu_v, cpu_sample = cpu_reference_us_per_token(os.cpu_count() or 1)
        cpu_pf, cpu_pf_sample = cpu_reference_prefill_tok_per_s(os.cpu_count() or 1)
    ms3, u3, _ = res[3]
    line = {"metric": METRIC, "value": us_tok, "unit": "us/token", "n_gpus": 1, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms1, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16x2+f32 (10-bit VQ indices, fp16 codebook/scales)",
            "data": "synthetic (seeded weights in the reference layout, softmax top-8 routing)",
            "config": {"workload": "config1 decode batch 1 (batch 3 in decode_b3)", "H": H, "I": I, "E": E,
                       "topk": K, "batch": 1, "l2": f"{nlayers} layers cycled per step (8.8 GB > L2)",
                       "distinct_experts_per_step": u1},
            "router": {**router, "workload": "top-8 of softmax(x @ W_r), x [1, 4096], W_r [4096, 256], graph replay"},
            "shared_expert": {**shared, "workload": "config1 shared expert, bf16 gate/up [4096, 4096] + down [4096, 2048], 4 weight copies cycled (> L2)"},
            "routed_plus_shared": with_shared,
            "pack": {**pack, "workload": "VQ packer on 8 experts of the gate/up tensor, 8 x 4096 x 4096 bf16"},
            "decode_graph": {"us_per_token": ms_graph * 1e3,
                             "how": "the same batch-1 steps replayed from CUDA graphs"},
            "decode_b3": {"us_per_token": ms3 * 1e3 / 3, "us_per_layer_call": ms3 * 1e3, "distinct_experts": u3,
                          "idx_act_GBps": (u3 * IDX_BYTES_PER_EXPERT + 3 * H * 6) / (ms3 * 1e-3) / 1e9},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm,
                         # dram read+write of one layer call (both decode kernels), from the ncu
                         # capture summarised in profiles/decode_config1_b1.txt (8 distinct experts)
                         "traffic": NCU_DECODE_BYTES_PER_EXPERT * u1, "traffic_unit": "bytes per layer call",
                         "traffic_source": "ncu dram read+write per distinct expert (profiles/decode_config1_b1.txt) x this run's distinct experts",
                         "kernel": "decode layer call (gate/up + down kernels, CUDA events around both)",
                         "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else src,
                         "bytes": "index planes of distinct experts + x + out per layer call",
                         "achieved_incl_scales": all_bytes / (ms1 * 1e-3) / 1e9},
            "cpu_baseline": {"value": cpu_v, "unit": "us/token", "cores": os.cpu_count(), "kind": "port",
                             "cpu_model": cpu_model(),
                             "sample": cpu_sample},
            "cpu_baseline_prefill": {"value": cpu_pf, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                                     "cpu_model": cpu_model(),
                                     "sample": cpu_pf_sample},
            "e2e": {"value": e2e_ms * 1e3, "unit": "us/token", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "host_wall_us_per_step": e2e_wall_ms * 1e3,
                    "how": "HostDecodeSession: per step one upload (copy stream), the decode kernels, one download (second copy stream)"},
            "prefill": prefill,
            "stack": stack,
            "gpu_launches": 2 * args.steps,
            "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_ref_gpu(args):
    """--ref-gpu: the reference's own GPU path on this B200 beside ours, same layers and inputs:
    decode (its Triton kernels, vq2_moe_fused_10b) at config 1, N=1 and N=3, eager and CUDA-graph
    replayed; prefill (its vq2_grouped.cu fp8 path, vq2_moe_grouped_wmma) at config 2. Reports
    both timings and the relative L2 distance between the two outputs. One JSON line."""
    from vq2_vllm import synth
    from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma as ours_pf
    from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b as ours_dec
    from oracle import torch_ref
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    try:
        from baseline.ref_modules import RefModules
        refs = RefModules()
    except Exception as ex:      # reference absent or not importable: say why, exit cleanly
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"{type(ex).__name__}: {ex}"}), flush=True)
        return
    ref_dec = refs.mods["vq2_kernel"].vq2_moe_fused_10b
    ref_pf = refs.mods["ds4_vq2_cuda"].vq2_moe_grouped_wmma
    nlayers = 4
    layers = [synth.make_layer(E, H, I, seed=1000 * l, device=dev) for l in range(nlayers)]
    stream = torch.cuda.current_stream()

    def timed(fn, steps, graph):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        if graph:
            gs = []
            for j in range(nlayers):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn(j)
                gs.append(g)
            torch.cuda.synchronize()
            run = lambda i: gs[i % nlayers].replay()
        else:
            run = fn
        for i in range(3):
            run(i)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda._sleep(5_000_000)
        s.record(stream)
        for i in range(steps):
            run(i)
        e.record(stream)
        e.synchronize()
        return s.elapsed_time(e) / steps

    out = {"impl": "reference-gpu", "metric": METRIC, "n_gpus": 1, "steps": args.steps,
           "config": {"workload": "config1 decode (N=1, 3) and config2 prefill, reference GPU path vs ours",
                      "H": H, "I": I, "E": E, "topk": K, "l2": f"{nlayers} layers cycled"},
           "reference": "baseline/_ref (unmodified install); prefill extension built for sm_100a by "
                        "baseline/build_ref_ext.py", "decode": {}}
    for N in (1, 3):
        x = synth.make_tokens(N, H, seed=400 + N, device=dev)
        ids, tw = make_routing(x, 500 + N)
        res = {}
        for name, fn in (("ours", ours_dec), ("reference", ref_dec)):
            call = lambda i, fn=fn: fn(x, ids, tw, *synth.layer_args(layers[i % nlayers]))
            with refs:
                res[name] = {"eager_us_per_call": 1e3 * timed(call, args.steps, False)}
                try:
                    res[name]["graph_us_per_call"] = 1e3 * timed(call, args.steps, True)
                except Exception as ex:
                    res[name]["graph_us_per_call"] = None
                    res[name]["graph_error"] = f"{type(ex).__name__}: {ex}"[:200]
        with refs:
            a = ours_dec(x, ids, tw, *synth.layer_args(layers[0]))
            b = ref_dec(x, ids, tw, *synth.layer_args(layers[0]))
            d = torch_ref.moe_ref(x, ids, tw, layers[0])
        res["rel_l2_ours_vs_reference"] = torch_ref.rel_l2(a, b)
        res["rel_l2_ours_vs_fp32"] = torch_ref.rel_l2(a, d)
        res["rel_l2_reference_vs_fp32"] = torch_ref.rel_l2(b, d)
        out["decode"][f"N={N}"] = res
    if refs.has_prefill:
        Np = 8192
        x = synth.make_tokens(Np, H, seed=300, device=dev)
        ids, tw = synth.route_zipf(Np, E, K, s=1.1, seed=301, device=dev)
        flops = 2.0 * Np * K * H * 2 * I + 2.0 * Np * K * I * H
        pf = {}
        reps = max(3, min(args.steps, 10))
        for name, fn in (("ours", lambda i: ours_pf(x, ids, tw, *synth.layer_args(layers[i % nlayers]), precision="fp8")),
                         ("reference", lambda i: ref_pf(x, ids, tw, *synth.layer_args(layers[i % nlayers])))):
            with refs:
                ms = timed(fn, reps, False)
            pf[name] = {"fp8_ms_per_call": ms, "tok_per_s": Np / (ms * 1e-3), "tflops": flops / (ms * 1e-3) / 1e12}
        with refs:
            a = ours_pf(x, ids, tw, *synth.layer_args(layers[0]), precision="fp8")
            b = ref_pf(x, ids, tw, *synth.layer_args(layers[0]))
        pf["rel_l2_ours_vs_reference"] = torch_ref.rel_l2(a, b)
        out["prefill"] = pf
    else:
        out["prefill"] = {"unavailable": "reference extension not built for sm_100a (baseline/build_ref_ext.py)"}
    print(json.dumps(out), flush=True)


def run_profile_case(case):
    """--profile-case: a small, self-contained invocation of one hot kernel for ncu captures (a few
    GB on the device at most, a handful of launches): "decode" = four config-1 decode layer calls
    at batch 1 over two layers; "prefill" = two fp8 grouped-GEMM calls, 2048 tokens over 64
    experts, Zipf(1.1) top-8 (a small case of the config-2 kernels); "prefill-config2" = three fp8
    calls at config 2 (8192 tokens, 256 experts: 2.2 GB of weights, a launch-list capture only)."""
    from vq2_vllm import synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if case == "decode":
        from vq2_vllm.kernels.vq2_kernel import vq2_moe_fused_10b
        layers = [synth.make_layer(E, H, I, seed=s, device=dev) for s in range(2)]
        x = synth.make_tokens(1, H, seed=1, device=dev)
        ids, tw = make_routing(x, 2)
        for i in range(4):
            vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(layers[i % 2]))
    elif case == "prefill-config2":
        from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
        L = synth.make_layer(E, H, I, seed=10, device=dev)
        x = synth.make_tokens(8192, H, seed=300, device=dev)
        ids, tw = synth.route_zipf(8192, E, K, s=1.1, seed=301, device=dev)
        for _ in range(3):
            vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(L), precision="fp8")
    else:
        from vq2_vllm.kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
        L = synth.make_layer(64, H, I, seed=0, device=dev)
        x = synth.make_tokens(2048, H, seed=1, device=dev)
        ids, tw = synth.route_zipf(2048, 64, K, seed=2, device=dev)
        for _ in range(2):
            vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(L), precision="fp8")
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "ok": True}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--soak", type=float, default=0.6, help="untimed seconds before the timed decode steps")
    ap.add_argument("--ref-gpu", action="store_true",
                    help="time the reference's own GPU path (baseline/_ref) beside ours; one JSON line")
    ap.add_argument("--profile-case", choices=["decode", "prefill", "prefill-config2"],
                    help="run a small invocation of one hot kernel (for ncu captures) and exit")
    args = ap.parse_args()
    if args.profile_case:
        return run_profile_case(args.profile_case)
    if args.ref_gpu:
        return run_ref_gpu(args)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world)


if __name__ == "__main__":
    main()
