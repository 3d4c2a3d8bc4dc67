"""LeNet-5 batch inference on the sm_100a kernels of tz_lenet.cu.

Mirrors the reference's ``LeNet`` (lenet.zig:218-321): weights by the names of ``LeNetWeights``
(conv1_weight [6,5,5,1] ... fc3_bias [10], NHWC conv layout), ``forward(input, batch_size)``
returning ``[batch, 10]``.  ``variant`` selects lenet.zig as written (``LENET_REF``: conv1 valid,
256 features, logits) or the padded benchmark network (``LENET_PAD2``: conv1 padding 2, 400
features, softmax).  There is no CPU fallback: the CUDA library must be present.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .runtime import Context

LENET_REF, LENET_PAD2 = 0, 1
# LeNetWeights field names (lenet.zig:33-52) -> tz_lenet_weights members
FIELDS = (("conv1_weight", "conv1_w"), ("conv1_bias", "conv1_b"), ("conv2_weight", "conv2_w"),
          ("conv2_bias", "conv2_b"), ("fc1_weight", "fc1_w"), ("fc1_bias", "fc1_b"), ("fc2_weight", "fc2_w"),
          ("fc2_bias", "fc2_b"), ("fc3_weight", "fc3_w"), ("fc3_bias", "fc3_b"))


class _Weights(C.Structure):
    _fields_ = [(c, C.c_void_p) for _, c in FIELDS]


class LeNet:
    """Device-resident LeNet-5 (weights + scratch) on one B200."""

    def __init__(self, ctx: Context, weights: dict, variant: int = LENET_PAD2):
        feat = 400 if variant == LENET_PAD2 else 256
        shapes = {"conv1_w": (6, 5, 5, 1), "conv1_b": (6,), "conv2_w": (16, 5, 5, 6), "conv2_b": (16,),
                  "fc1_w": (120, feat), "fc1_b": (120,), "fc2_w": (84, 120), "fc2_b": (84,), "fc3_w": (10, 84),
                  "fc3_b": (10,)}
        host = {}
        for ref_name, c_name in FIELDS:
            a = weights.get(c_name, weights.get(ref_name))
            if a is None:
                raise KeyError(f"missing LeNet weight {ref_name}")
            a = np.ascontiguousarray(a, dtype=np.float32)
            if a.size != int(np.prod(shapes[c_name])):
                raise ValueError(f"{ref_name}: {a.size} values, expected shape {shapes[c_name]}")
            host[c_name] = a
        st = _Weights(*[host[c].ctypes.data for _, c in FIELDS])
        h = C.c_void_p()
        L.check(L.lib().tz_lenet_load(ctx.handle, C.byref(st), variant, C.byref(h)))
        self.ctx, self.handle, self.variant = ctx, h, variant
        ctx._adopt(self)

    @classmethod
    def from_tenzor(cls, ctx: Context, path: str, variant: int = LENET_PAD2) -> "LeNet":
        """A LeNet training checkpoint in .tenzor form (main.zig:502-511, runEval 638-667)."""
        h = C.c_void_p()
        L.check(L.lib().tz_lenet_load_tenzor(ctx.handle, path.encode(), variant, C.byref(h)))
        self = cls.__new__(cls)
        self.ctx, self.handle, self.variant = ctx, h, variant
        ctx._adopt(self)
        return self

    def close(self):
        if self.handle:
            L.lib().tz_lenet_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, n: int):
        L.check(L.lib().tz_lenet_reserve(self.handle, n))

    def forward(self, images: np.ndarray) -> np.ndarray:
        """Host images [n, 28, 28, 1] (or [n, 784]) -> [n, 10] (synchronous)."""
        x = np.ascontiguousarray(images, dtype=np.float32).reshape(-1, 784)
        out = np.empty((x.shape[0], 10), np.float32)
        L.check(L.lib().tz_lenet_forward(self.handle, x.ctypes.data, x.shape[0], out.ctypes.data))
        return out

    def forward_device(self, d_images: int, n: int, d_out: int, stream: int = 0):
        """Device pointers; asynchronous on ``stream`` (a CUDA stream handle, 0 = the context's)."""
        L.check(L.lib().tz_lenet_forward_device(self.handle, C.c_void_p(d_images), n, C.c_void_p(d_out),
                                                C.c_void_p(stream) if stream else None))
