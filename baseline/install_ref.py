"""Install the unmodified reference into baseline/_ref and build its prefill extension for sm_100a.

    python baseline/install_ref.py

Both steps are skipped when their output is already present. The install copies the reference
checkout to a temporary directory first (its build writes into the source tree, and the checkout
is read-only) and runs the one offline pip install the benchmark contract allows:

    python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \\
        --target baseline/_ref <copy of the reference checkout>

(`--no-deps`: torch, triton and vLLM are already in the image). The extension build is
build_ref_ext.py (the reference's vq2_grouped.cu with its own flags, target sm_100a; about five
minutes of nvcc). The GPU box has no reference checkout: it only uses what this leaves in
baseline/_ref, which travels with the working tree.
"""
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
REF_SRC = os.environ.get("VQ2_REFERENCE_SRC", "/root/reference")


def installed() -> bool:
    return os.path.exists(os.path.join(REF_DIR, "vq2_vllm", "kernels", "vq2_kernel.py"))


def ext_built() -> bool:
    d = os.path.join(REF_DIR, "_ext_sm100a")
    return os.path.isdir(d) and any(f.endswith(".so") for f in os.listdir(d))


def install(log=print) -> bool:
    if installed():
        return True
    if not os.path.isdir(REF_SRC):
        log(f"reference checkout {REF_SRC} absent: baseline/_ref not installed")
        return False
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "reference")
        shutil.copytree(REF_SRC, src, ignore=shutil.ignore_patterns(".git"))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", REF_DIR, src]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            log("reference install failed: " + (r.stderr or r.stdout)[-400:])
            return False
    return installed()


def build_ext(log=print) -> bool:
    if ext_built():
        return True
    if not installed():
        return False
    r = subprocess.run([sys.executable, os.path.join(HERE, "build_ref_ext.py")], capture_output=True, text=True)
    if r.returncode != 0:
        log("reference extension build failed: " + (r.stderr or r.stdout)[-400:])
        return False
    return ext_built()


def main(log=print) -> bool:
    return install(log) and build_ext(log)


if __name__ == "__main__":
    ok = main()
    print("baseline/_ref ready" if ok else "baseline/_ref not ready")
    sys.exit(0 if ok else 1)
