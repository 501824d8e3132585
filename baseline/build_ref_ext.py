"""Build the reference's prefill CUDA extension (its unmodified vq2_grouped.cu) for sm_100a.

The reference JIT-builds this file for sm_121a only (vq2_vllm/kernels/ds4_vq2_cuda.py:38-47). This
recipe compiles the same source, with the reference's own flags except the target, into
baseline/_ref/_ext_sm100a/ so that `bench.py --ref-gpu` can time the reference's prefill path on a
B200 without compiling there. Run it after installing the reference into baseline/_ref:

    python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \\
        --target baseline/_ref <copy of the reference checkout>
    python baseline/build_ref_ext.py
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_KERNELS = os.path.join(HERE, "_ref", "vq2_vllm", "kernels")
OUT = os.path.join(HERE, "_ref", "_ext_sm100a")
NAME = "vq2_grouped_sm100a"


def main():
    src = os.path.join(REF_KERNELS, "vq2_grouped.cu")
    if not os.path.exists(src):
        sys.exit(f"reference not installed: {src} missing")
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    load(name=NAME, sources=[src], build_directory=OUT, verbose=False,
         extra_cuda_cflags=["-O3", "--use_fast_math", "-DVQ2_DIAG=0", "-gencode=arch=compute_100a,code=sm_100a"])
    print(os.path.join(OUT, NAME + ".so"))


if __name__ == "__main__":
    main()
