"""vq2_vllm (B200): the vq2 routed-expert MoE path of the reference vLLM plugin, drop-in.

Kernel entry points keep the reference's module names: ``vq2_vllm.kernels.vq2_kernel``
(vq2_moe_fused_10b, had_act_batch), ``vq2_vllm.kernels.ds4_vq2_cuda`` (vq2_moe_grouped_wmma,
quant_fp8_rows), ``vq2_vllm.kernels.moe_align`` (moe_align). The reference put its kernels dir
on sys.path and imported them by bare name; the same bare names resolve here too.
``register`` is the vLLM general-plugin entry point.
"""
import sys

from .kernels import ds4_vq2_cuda, moe_align, vq2_kernel  # noqa: F401
from .plugin import register  # noqa: F401

for _name, _mod in (("vq2_kernel", vq2_kernel), ("ds4_vq2_cuda", ds4_vq2_cuda), ("moe_align", moe_align)):
    sys.modules.setdefault(_name, _mod)
