"""Load the committed golden fixtures (produced by tests/golden/make_golden.py from the reference)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KEYS = ("w13_cb", "w13_lo", "w13_hi", "w13_sc", "w2_cb", "w2_lo", "w2_hi", "w2_sc")


def f16(a):
    return np.asarray(a).view(np.float16)


def load_config0():
    z = dict(np.load(os.path.join(GOLDEN, "config0.npz")))
    layer = {}
    for k in KEYS:
        layer[k] = f16(z[k]) if (k.endswith("_cb") or k.endswith("_sc")) else z[k]
    bits = z["x_bf16_bits"].astype(np.uint16).astype(np.uint32) << 16
    x = bits.view(np.float32)
    return z, layer, x


def load_align():
    z = dict(np.load(os.path.join(GOLDEN, "align.npz")))
    n = len([k for k in z if k.endswith("_ids")])
    return [(z[f"c{i}_ids"], int(z[f"c{i}_meta"][0]), int(z[f"c{i}_meta"][1]), int(z[f"c{i}_meta"][2]),
             z[f"c{i}_st"], z[f"c{i}_ss"], z[f"c{i}_val"], z[f"c{i}_be"]) for i in range(n)]


def load_pack():
    """The reference packer's fixtures: case a (pack_vq2_experts_10b, fp32 W [2, 48, 256], k=1024,
    12 iterations) and case b (pack_vq2, bf16 W [40, 200] padded to 256, k=256, 6 iterations),
    each with the sample the reference drew (si) and its initial-codebook positions (init)."""
    z = dict(np.load(os.path.join(GOLDEN, "pack.npz")))
    bits = z["b_W_bf16_bits"].astype(np.uint16).astype(np.uint32) << 16
    z["b_W"] = bits.view(np.float32)
    return z
