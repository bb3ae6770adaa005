"""B200-native (sm_100a) Gemma-3 int4 decode path behind the reference's
operator surface (badnikhil/Xpose, "Vulkore").

* ``xpose_b200.vulkore``  -- Context / Buffer / Program / launch / Batch / Fence
* ``xpose_b200.decode``   -- DecodeConfig / Sampling / DecodeSession
* ``include/xp_cuda.h``   -- the C ABI both sit on (libxp_cuda.so)
"""
from ._lib import XpError, lib  # noqa: F401

__all__ = ["XpError", "lib"]
