"""vLLM binding of the vq2 routed-expert method (the drop-in boundary).

Mirrors the reference plugin's MoE part (vq2_vllm/__init__.py:136-259 ``Vq2MoEMethod`` and
:272-357 ``_Vq2Config``, registered by ``register()`` at :678-692): the quantisation method
"vq2" with the same parameter names, shapes, dtypes and weight-loading contract, and the same
``apply`` dispatch — batches of at least VQ2_WMMA_MIN tokens (default 256) go to the grouped GEMM
(``vq2_moe_grouped_wmma``), smaller ones to the decode kernel (``vq2_moe_fused_10b``); the fp32
result is cast to the activation dtype. The kernels are this package's sm_100a extension.

Only routed experts are served here. Other layers get vLLM's unquantised method (attention,
shared experts and lm_head quantisation of the reference recipe stay with the reference plugin).
vLLM is imported lazily so the package works without it.
"""
from __future__ import annotations

import os
import re

import torch

_WMMA_MIN = int(os.environ.get("VQ2_WMMA_MIN", "256"))
_WMMA_PREFILL = os.environ.get("VQ2_WMMA_PREFILL", "1") == "1"
PARAMS = ("w13_lo", "w13_hi", "w13_sc", "w2_lo", "w2_hi", "w2_sc", "w13_cb", "w2_cb")


def param_shapes(E, H, I, vdim=4, k=1024, group=64):
    """Parameter shapes/dtypes of one layer (reference vq2_vllm/__init__.py:164-173)."""
    spg = group // vdim
    nsub_gu, nsub_dn = H // vdim, I // vdim
    return {
        "w13_lo": ((E, 2 * I, nsub_gu), torch.uint8),
        "w13_hi": ((E, 2 * I, nsub_gu // 4), torch.uint8),
        "w13_sc": ((E, 2 * I, nsub_gu // spg), torch.float16),
        "w2_lo": ((E, H, nsub_dn), torch.uint8),
        "w2_hi": ((E, H, nsub_dn // 4), torch.uint8),
        "w2_sc": ((E, H, nsub_dn // spg), torch.float16),
        "w13_cb": ((k, vdim), torch.float16),
        "w2_cb": ((k, vdim), torch.float16),
    }


def weight_loader(param, loaded_weight, weight_name, shard_id, expert_id, return_success=False):
    """Per-expert loading (reference vq2_vllm/__init__.py:178-192): codebooks are copied whole;
    w1 goes to rows [0, I) (gate) and w3 to rows [I, 2I) (up) of the fused w13 tensors."""
    lw = loaded_weight.to(param.device)
    if weight_name.endswith("cb"):
        param.data.copy_(lw.to(param.dtype))
    elif shard_id == "w2":
        param.data[expert_id].copy_(lw.to(param.dtype))
    else:
        half = param.shape[1] // 2
        rows = slice(0, half) if shard_id == "w1" else slice(half, None)
        param.data[expert_id, rows].copy_(lw.to(param.dtype))
    return True if return_success else None


def apply_moe(layer, x, topk_weights, topk_ids, group=64):
    """The reference's apply dispatch (vq2_vllm/__init__.py:197-218) on the B200 kernels."""
    from .kernels.ds4_vq2_cuda import vq2_moe_grouped_wmma
    from .kernels.vq2_kernel import vq2_moe_fused_10b
    args = (layer.w13_cb, layer.w13_lo, layer.w13_hi, layer.w13_sc, layer.w2_cb, layer.w2_lo, layer.w2_hi,
            layer.w2_sc)
    base = int(getattr(layer, "vq2_expert_base", 0))   # set when the layer holds a slice of the experts
    if _WMMA_PREFILL and x.shape[0] >= _WMMA_MIN:
        out = vq2_moe_grouped_wmma(x, topk_ids, topk_weights, *args, group=group, expert_base=base)
    else:
        out = vq2_moe_fused_10b(x, topk_ids, topk_weights, *args, group=group, expert_base=base)
    return out.to(x.dtype)


def read_fused_layer(path: str, device="cpu", expert_range=None) -> dict:
    """The 8 tensors of one ``experts_fused_layer_{L}.safetensors`` file (reference layout,
    vq2_vllm/__init__.py:233-235). ``expert_range=(lo, hi)`` reads only experts [lo, hi) of the
    per-expert tensors (slices of the file, so a rank of an expert-parallel group reads only its
    share); the codebooks are read whole."""
    from safetensors import safe_open
    out = {}
    with safe_open(path, "pt", device=str(device)) as f:
        for name in PARAMS:
            if expert_range is not None and not name.endswith("cb"):
                lo, hi = expert_range
                out[name] = f.get_slice(name)[lo:hi]
            else:
                out[name] = f.get_tensor(name)
    return out


def load_fused_layer_file(layer, layer_index: int, directory: str | None = None, expert_range=None) -> bool:
    """Fast load of ``experts_fused_layer_{L}.safetensors`` (the 8 tensors, directly onto the
    parameters' device) when present (reference vq2_vllm/__init__.py:220-235). With
    ``expert_range`` only those experts are read (the layer then holds E = hi - lo experts)."""
    d = directory or os.environ.get("VQ2_EXPERTS_DIR", "models/DeepSeek-V4-Flash-2bit")
    path = f"{d}/experts_fused_layer_{layer_index}.safetensors"
    if not os.path.exists(path):
        return False
    t = read_fused_layer(path, device=layer.w13_lo.device, expert_range=expert_range)
    for name in PARAMS:
        getattr(layer, name).data.copy_(t[name])
    return True


def process_weights_after_loading(layer, directory: str | None = None) -> bool:
    """The method's post-load hook (reference vq2_vllm/__init__.py:220-235): when the fused file
    of the layer's index (from ``layer_name`` / ``prefix``, "...layers.{L}....") exists, its 8
    tensors are read straight onto the parameters' device. A layer holding fewer experts than the
    file (expert parallelism: ``local_num_experts`` and ``ep_rank``, as vLLM's FusedMoE has them)
    reads only its contiguous slice [ep_rank * local, (ep_rank + 1) * local) and records the first
    one as ``vq2_expert_base``, so apply() maps the global expert ids onto it."""
    m = re.search(r"layers\.(\d+)\.", str(getattr(layer, "layer_name", "") or getattr(layer, "prefix", "")))
    if m is None:
        return False
    E_local = int(layer.w13_lo.shape[0])
    rng = None
    if getattr(layer, "local_num_experts", None) is not None and getattr(layer, "ep_rank", None) is not None:
        lo = int(layer.ep_rank) * int(layer.local_num_experts)
        rng = (lo, lo + E_local)
    ok = load_fused_layer_file(layer, int(m.group(1)), directory, expert_range=rng)
    if ok and rng is not None:
        layer.vq2_expert_base = rng[0]
    return ok


_CONFIG_CLS = None


def _bind():
    global _CONFIG_CLS
    if _CONFIG_CLS is not None:
        return _CONFIG_CLS
    from vllm.model_executor.layers.fused_moe import FusedMoE, FusedMoEMethodBase, RoutedExperts
    from vllm.model_executor.layers.linear import LinearBase, UnquantizedLinearMethod
    from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
    from vllm.model_executor.utils import set_weight_attrs

    class Vq2MoEMethod(FusedMoEMethodBase):
        """Routed experts: shared codebook + 10-bit byte-plane VQ indices (sm_100a kernels)."""

        def __init__(self, quant_config, moe):
            super().__init__(moe)
            self.quant_config = quant_config

        def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                           **extra_weight_attrs):
            q = self.quant_config
            shapes = param_shapes(num_experts, hidden_size, intermediate_size_per_partition, q.vdim, q.k, q.group)
            for name, (shape, dtype) in shapes.items():
                p = torch.nn.Parameter(torch.empty(*shape, dtype=dtype), requires_grad=False)
                layer.register_parameter(name, p)
                set_weight_attrs(p, {"weight_loader": weight_loader})

        def get_fused_moe_quant_config(self, layer):
            return None

        def apply(self, layer, x, topk_weights, topk_ids, shared_experts, shared_experts_input):
            return apply_moe(layer, x, topk_weights, topk_ids, group=self.quant_config.group)

        def process_weights_after_loading(self, layer):
            process_weights_after_loading(layer)

    class Vq2Config(QuantizationConfig):
        """Quantisation config "vq2" (reference vq2_vllm/__init__.py:293-357, MoE part)."""

        def __init__(self, vdim=4, k=1024, group=64, full_config=None):
            super().__init__()
            if (vdim, k, group) != (4, 1024, 64):
                raise ValueError(f"vq2 (B200): only vdim=4, k=1024, group=64 are supported, got {(vdim, k, group)}")
            self.vdim, self.k, self.group = vdim, k, group
            self.full_config = full_config or {}

        @classmethod
        def get_name(cls):
            return "vq2"

        @classmethod
        def get_supported_act_dtypes(cls):
            return [torch.bfloat16, torch.half]

        @classmethod
        def get_min_capability(cls):
            return 100          # the kernels are built for sm_100a

        @staticmethod
        def get_config_filenames():
            return []

        @classmethod
        def from_config(cls, config):
            return cls(vdim=int(config.get("vdim", 4)), k=int(config.get("k", 1024)),
                       group=int(config.get("group", 64)), full_config=config)

        def get_quant_method(self, layer, prefix):
            if isinstance(layer, (FusedMoE, RoutedExperts)):
                return Vq2MoEMethod(self, layer.moe_config)
            if isinstance(layer, LinearBase):
                return UnquantizedLinearMethod()
            return None

    Vq2Config.MoEMethod = Vq2MoEMethod
    _CONFIG_CLS = Vq2Config
    return Vq2Config


def register():
    """vLLM general-plugin entry point: registers the "vq2" quantisation config
    (reference vq2_vllm/__init__.py:678-684)."""
    from vllm.model_executor.layers.quantization import register_quantization_config
    cls = _bind()
    try:
        register_quantization_config("vq2")(cls)
    except ValueError:
        pass               # already registered in this process
    return cls
