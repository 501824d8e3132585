"""Kernel entry points of the vq2 routed-expert path (B200 C-ABI extension)."""
