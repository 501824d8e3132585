"""The reference's own kernel modules from baseline/_ref (an unmodified install of the reference,
made by `pip install --target baseline/_ref`), for timing and parity checks beside this package.

The reference's code imports its sibling modules by bare name (`import vq2_kernel`, vq2_vllm/kernels/
ds4_vq2_cuda.py:76-77). This package registers the same bare names for itself, so the reference's
entries are swapped into sys.modules only while reference code runs (`with refs:`). The reference
JIT-builds its prefill extension for sm_121a only (ds4_vq2_cuda.py:38-47); build_ref_ext.py builds
the same source for sm_100a, and its module is installed as the reference module's extension handle.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


class RefModules:
    """Reference kernel modules; `mods` maps bare name -> module; `has_prefill` tells whether the
    sm_100a build of the prefill extension is present."""
    NAMES = ("vq2_kernel", "moe_align", "ds4_vq2_cuda")

    def __init__(self):
        kdir = os.path.join(HERE, "_ref", "vq2_vllm", "kernels")
        if not os.path.isdir(kdir):
            raise FileNotFoundError("reference not installed in baseline/_ref")
        import importlib
        import importlib.machinery
        import importlib.util
        saved = {n: sys.modules.pop(n, None) for n in self.NAMES}
        sys.path.insert(0, kdir)
        try:
            self.mods = {n: importlib.import_module(n) for n in self.NAMES}
        finally:
            sys.path.remove(kdir)
            for n in self.NAMES:
                sys.modules.pop(n, None)
                if saved[n] is not None:
                    sys.modules[n] = saved[n]
        self.saved = {}
        so = os.path.join(HERE, "_ref", "_ext_sm100a", "vq2_grouped_sm100a.so")
        self.has_prefill = os.path.exists(so)
        if self.has_prefill:
            loader = importlib.machinery.ExtensionFileLoader("vq2_grouped_sm100a", so)
            spec = importlib.util.spec_from_loader("vq2_grouped_sm100a", loader)
            ext = importlib.util.module_from_spec(spec)
            loader.exec_module(ext)
            self.mods["ds4_vq2_cuda"]._EXT = ext

    def __enter__(self):
        self.saved = {n: sys.modules.get(n) for n in self.NAMES}
        sys.modules.update(self.mods)
        return self.mods

    def __exit__(self, *exc):
        for n in self.NAMES:
            sys.modules.pop(n, None)
            if self.saved.get(n) is not None:
                sys.modules[n] = self.saved[n]
        return False
