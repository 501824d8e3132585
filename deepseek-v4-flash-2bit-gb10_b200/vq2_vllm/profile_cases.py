"""Small, self-contained invocations of the hot kernels for profilers (ncu captures).

    python -m vq2_vllm.profile_cases decode   # config-1 decode layer, batch 1, 4 calls
    python -m vq2_vllm.profile_cases prefill  # grouped GEMM: 2048 tokens, 64 experts, Zipf top-8

Run from deepseek-v4-flash-2bit-gb10_b200/ (or with it on PYTHONPATH). Each case keeps a few GB
on the device at most and launches each kernel a handful of times.
"""
import sys

import torch


def decode(calls=4):
    from . import synth
    from .kernels.vq2_kernel import vq2_moe_fused_10b
    layers = [synth.make_layer(256, 4096, 2048, seed=s, device="cuda") for s in range(2)]
    x = synth.make_tokens(1, 4096, seed=1, device="cuda")
    ids, tw = synth.route_softmax_topk(x, 256, 8, w_std=0.02, seed=2)
    for i in range(calls):
        vq2_moe_fused_10b(x, ids, tw, *synth.layer_args(layers[i % 2]))
    torch.cuda.synchronize()


def prefill(calls=2, prec="fp8"):
    from . import synth
    from .kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    L = synth.make_layer(64, 4096, 2048, seed=0, device="cuda")
    x = synth.make_tokens(2048, 4096, seed=1, device="cuda")
    ids, tw = synth.route_zipf(2048, 64, 8, seed=2, device="cuda")
    for _ in range(calls):
        vq2_moe_grouped_wmma(x, ids, tw, *synth.layer_args(L), precision=prec)
    torch.cuda.synchronize()


if __name__ == "__main__":
    case = sys.argv[1] if len(sys.argv) > 1 else "decode"
    {"decode": decode, "prefill": prefill}[case]()
    print(f"profile case {case}: ok")
