"""Checkpoint quantiser: the reference's src/quantize_arctic_xs.zig run on the GPU.

Every 2-D f32 '.weight' that is not a LayerNorm and has >= 4096 elements (shouldQuantize,
quantize_arctic_xs.zig:22-34) becomes int8 with a per-row IEEE-half scale '<name>.scale'
(quantize_arctic_xs.zig:94-115, kernel tz_quantize_weight_rows); everything else is copied.

    python -m tenzor_b200.quantize in.safetensors out.safetensors
"""
from __future__ import annotations

import sys

import numpy as np
import torch

from . import ops
from . import safetensors as st
from .runtime import Context


def should_quantize(name: str, a: np.ndarray) -> bool:
    return (a.dtype == np.float32 and a.ndim == 2 and name.endswith(".weight") and "LayerNorm" not in name
            and a.shape[0] > 0 and a.shape[1] > 0 and a.size >= 4096)


def quantize_checkpoint(ctx: Context, ckpt: dict) -> dict:
    out = {}
    dev = torch.device("cuda", ctx.device)
    for name, a in ckpt.items():
        if not should_quantize(name, a):
            out[name] = a
            continue
        w = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        q, s = ops.quantize_weight_rows(ctx, w)
        torch.cuda.synchronize(dev)
        out[name] = q.cpu().numpy()
        out[name + ".scale"] = s.cpu().numpy().view(np.uint16)
    return out


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__)
        return 2
    ctx = Context(0)
    q = quantize_checkpoint(ctx, st.load(argv[0]))
    st.save(argv[1], q)
    n = sum(1 for k in q if k.endswith(".scale"))
    print(f"Wrote {argv[1]} ({n} weights quantized)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
