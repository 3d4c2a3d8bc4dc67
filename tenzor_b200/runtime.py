"""Device context: one B200, its default stream and the op-level scratch arena (tz_cuda_*)."""
from __future__ import annotations

import ctypes as C
import weakref

from . import _lib as L


class Context:
    """Owns a tz_ctx_t.  Replaces the CPU ThreadPool handle of the reference (main.zig:787-789):
    every model / op call takes one."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        L.check(L.lib().tz_cuda_create(device, C.byref(h)))
        self.handle = h
        self.device = device
        self._owned = weakref.WeakSet()  # models on this context: closed before the context

    def _adopt(self, obj):
        self._owned.add(obj)

    @property
    def sm_count(self) -> int:
        return L.lib().tz_cuda_sm_count(self.handle)

    def set_sm_reserve(self, n: int):
        """Leave n SMs free in the persistent GEMM grids (for a collective running concurrently)."""
        L.check(L.lib().tz_cuda_set_sm_reserve(self.handle, int(n)))

    def synchronize(self):
        L.check(L.lib().tz_cuda_synchronize(self.handle))

    def check_status(self):
        """Raises if a kernel's bounded wait expired or a device bounds check fired."""
        L.check(L.lib().tz_cuda_check_status(self.handle))

    def close(self):
        if self.handle:
            for obj in list(self._owned):
                obj.close()
            L.lib().tz_cuda_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def version() -> str:
    return L.lib().tz_version().decode()
