"""tz_linear_w8a8_noalloc: the W8A8 linear for callers that must not allocate device memory while
they run (for example inside a CUDA graph capture, or when another allocator has reserved all device
memory).  Called through the C ABI, its output must equal tz_linear_w8a8's on two calls in a row
(the second call reuses the library's fixed scratch array that the first one filled).  This file is
named so that pytest collects it last; it also passes on its own in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(fn, ctx, x, wq, s16, bias, y, m, k, n):
    from tenzor_b200 import _lib as L
    L.check(fn(ctx.handle, x.data_ptr(), wq.data_ptr(), s16.data_ptr(), bias.data_ptr(), y.data_ptr(), m, k, n,
               C.c_void_p(0x1)))  # cudaStreamLegacy: torch's default stream


def test_noalloc_matches_allocating_entry_point(ctx, oracle):
    from tenzor_b200 import _lib as L
    lib = L.lib()
    rng = np.random.default_rng(2024)
    for m, k, n in [(1000, 384, 1536), (300, 1536, 384)]:
        x = torch.from_numpy(rng.normal(0, 1, (m, k)).astype(np.float32)).cuda()
        wq = torch.from_numpy(rng.integers(-127, 128, (n, k)).astype(np.int8)).cuda()
        s16 = torch.from_numpy(rng.uniform(1e-3, 1e-2, n).astype(np.float16).view(np.int16)).cuda()
        bias = torch.from_numpy(rng.normal(0, 0.02, n).astype(np.float32)).cuda()
        ref = torch.empty((m, n), device="cuda")
        _call(lib.tz_linear_w8a8, ctx, x, wq, s16, bias, ref, m, k, n)
        # the CPU oracle's W8A8 linear (per-token quantiser, exact integer GEMM, one-rounding epilogue)
        want = oracle.linear_w8a8(x.cpu().numpy(), wq.cpu().numpy(), s16.cpu().numpy().view(np.uint16),
                                  bias.cpu().numpy())
        for _ in range(2):  # two calls in a row share the fixed scratch
            out = torch.full((m, n), float("nan"), device="cuda")
            _call(lib.tz_linear_w8a8_noalloc, ctx, x, wq, s16, bias, out, m, k, n)
            torch.cuda.synchronize()
            # same kernels on the same operands: equal within 0 (the tests' int8 tolerance is exact)
            assert torch.equal(out, ref), float((out - ref).abs().max())
            assert np.array_equal(out.cpu().numpy(), want), float(np.abs(out.cpu().numpy() - want).max())
    ctx.check_status()


def test_noalloc_rejects_oversized_problem(ctx):
    from tenzor_b200 import _lib as L
    lib = L.lib()
    m, k, n = 32768, 384, 384  # needs 12.6 MB of scratch > the fixed 8 MiB
    x = torch.zeros((m, k), device="cuda")
    wq = torch.zeros((n, k), dtype=torch.int8, device="cuda")
    s16 = torch.zeros(n, dtype=torch.int16, device="cuda")
    bias = torch.zeros(n, device="cuda")
    y = torch.zeros((m, n), device="cuda")
    rc = lib.tz_linear_w8a8_noalloc(ctx.handle, x.data_ptr(), wq.data_ptr(), s16.data_ptr(), bias.data_ptr(),
                                    y.data_ptr(), m, k, n, C.c_void_p(0x1))
    assert rc == L.TZ_EINVAL and b"fixed scratch" in lib.tz_get_last_error()


def test_noalloc_rejects_other_current_device(ctx):
    """The kernels run on the current device: a context of another device is refused."""
    from tenzor_b200 import _lib as L
    from tenzor_b200.runtime import Context
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib = L.lib()
    other = Context(1)
    try:
        torch.cuda.set_device(0)
        t = torch.zeros(16, device="cuda:0")
        rc = lib.tz_linear_w8a8_noalloc(other.handle, t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                                        t.data_ptr(), 1, 16, 1, C.c_void_p(0x1))
        assert rc == L.TZ_EINVAL and b"current device" in lib.tz_get_last_error()
    finally:
        other.close()
        torch.cuda.set_device(0)
