"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

from golden_io import load_config0


def config0_cuda():
    z, layer, x = load_config0()
    dev = "cuda"
    L = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in layer.items()}
    xb = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    ids = torch.from_numpy(z["topk_ids"]).to(dev)
    tw = torch.from_numpy(z["topk_w"]).to(dev)
    return z, L, xb, ids, tw


def args(L):
    return (L["w13_cb"], L["w13_lo"], L["w13_hi"], L["w13_sc"], L["w2_cb"], L["w2_lo"], L["w2_hi"], L["w2_sc"])
