"""Op-level kernels vs the CPU oracle / reference known answers, through the C ABI.  Needs a B200."""
import numpy as np
import pytest
import torch

import kats

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


GEMM_SHAPES = [(1, 128, 384), (128, 128, 128), (200, 384, 384), (333, 1152, 384), (1000, 384, 1536),
               (130, 1536, 384), (77, 96, 64), (4096, 384, 1536)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_gemm_i8_i32_bit_exact(ctx, oracle, m, n, k):
    from tenzor_b200 import ops
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    c = host(ops.gemm_i8_i32(ctx, dev(a), dev(w)))
    ref = oracle.gemm_i8_i32(a, w)
    assert c.dtype == np.int32 and (c == ref).all(), f"{(c != ref).sum()} mismatches"
    ctx.check_status()


def test_gemm_i8_extremes_bit_exact(ctx, oracle):
    # +-127 everywhere at K=1536: |acc| = 24.8M > 2^24, the int32 path must not round.
    from tenzor_b200 import ops
    a = np.full((128, 1536), 127, np.int8)
    a[1::2] = -127
    w = np.full((128, 1536), -127, np.int8)
    c = host(ops.gemm_i8_i32(ctx, dev(a), dev(w)))
    assert (c == oracle.gemm_i8_i32(a, w)).all()


@pytest.mark.parametrize("m,n,k", [(256, 384, 384), (513, 1536, 384), (300, 384, 1536)])
def test_linear_w8a8_bit_exact(ctx, oracle, m, n, k):
    from tenzor_b200 import ops
    rng = np.random.default_rng(m + n)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    x[5] = 0.0
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    wq, s16 = oracle.quantize_weight_rows(w)
    bias = rng.normal(0, 0.02, n).astype(np.float32)
    y = host(ops.linear_w8a8(ctx, dev(x), dev(wq), dev(s16.view(np.int16)), dev(bias)))
    ref = oracle.linear_w8a8(x, wq, s16, bias)
    assert (y == ref).all(), f"max diff {np.abs(y - ref).max()}"


@pytest.mark.parametrize("m,n,k", [(64, 384, 384), (300, 1536, 384), (129, 384, 1536)])
def test_linear_w8a32_vs_oracle(ctx, oracle, m, n, k):
    from tenzor_b200 import ops
    rng = np.random.default_rng(n + k)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    wq, s16 = oracle.quantize_weight_rows(w)
    bias = rng.normal(0, 0.02, n).astype(np.float32)
    y = host(ops.linear_w8a32(ctx, dev(x), dev(wq), dev(s16.view(np.int16)), dev(bias)))
    ref = oracle.linear_w8a32(x, wq, s16, bias)
    # activations are rounded to f16 (11-bit significand) on the way into the tensor core
    assert np.abs(y - ref).max() <= 2e-3 * np.abs(ref).max()


@pytest.mark.parametrize("m,n,k", [(1, 128, 384), (200, 384, 384), (1000, 1536, 384), (129, 384, 1536)])
def test_linear_f32_tf32_vs_fp32(ctx, m, n, k):
    from tenzor_b200 import ops
    rng = np.random.default_rng(k + m)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 0.05, (n, k)).astype(np.float32)
    b = rng.normal(0, 1, n).astype(np.float32)
    r = rng.normal(0, 1, (m, n)).astype(np.float32)
    y = host(ops.linear(ctx, dev(x), dev(w), dev(b), dev(r)))
    ref = x.astype(np.float64) @ w.T.astype(np.float64) + b + r
    # tf32 keeps 10 explicit mantissa bits: tolerance 2^-9 relative to the product scale
    assert np.abs(y - ref).max() <= 2e-3 * np.sqrt(k) * 0.05 * 4


def test_matmul_epilogue_kat(ctx):
    from tenzor_b200 import ops
    a, b, bias, chain, want = kats.MATMUL_EPILOGUE
    # 2x2 problem: K=2 is below the 16-byte TMA row minimum, so pad K with zeros (same product)
    a = np.pad(np.array(a, np.float32), ((0, 0), (0, 2)))
    b = np.pad(np.array(b, np.float32), ((0, 2), (0, 0)))
    c = host(ops.matmul_epilogue(ctx, dev(a), dev(b), dev(np.array(bias, np.float32)), chain))
    assert (c == np.array(want, np.float32)).all()


@pytest.mark.parametrize("trans_b", [False, True])
def test_matmul_epilogue_bias_gelu(ctx, oracle, trans_b):
    from tenzor_b200 import ops
    rng = np.random.default_rng(3)
    m, k, n = 300, 384, 1536
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k) if trans_b else (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    c = host(ops.matmul_epilogue(ctx, dev(a), dev(b), dev(bias), ["add", "gelu"], trans_b=trans_b))
    ref = oracle.matmul_epilogue(a, b, bias, [1, 3], trans_b=trans_b)
    scale = np.sqrt(k) * 0.6
    assert np.abs(c - ref).max() <= 4e-3 * scale


@pytest.mark.parametrize("m,k,n", [(77, 40, 260), (129, 64, 128), (1, 96, 4), (300, 384, 200)])
def test_matmul_epilogue_n_major_b_ragged(ctx, oracle, m, k, n):
    """B [k, n] read N-major by the tf32 MMA: ragged M, K not a multiple of the 32-element K block,
    N a multiple of 4 but not of the tile width."""
    from tenzor_b200 import ops
    rng = np.random.default_rng(m * 1000 + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    for chain, codes in ((["add"], [1]), (["add", "gelu"], [1, 3])):
        c = host(ops.matmul_epilogue(ctx, dev(a), dev(b), dev(bias), chain))
        ref = oracle.matmul_epilogue(a, b, bias, codes)
        assert np.abs(c - ref).max() <= 4e-3 * np.sqrt(k) * 0.6, chain


def test_quantize_weight_rows_bit_exact(ctx, oracle):
    from tenzor_b200 import ops
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.02, (1536, 384)).astype(np.float32)
    w[7] = 0.0
    w[8, 3] = 1e-30
    q, s = ops.quantize_weight_rows(ctx, dev(w))
    qo, so = oracle.quantize_weight_rows(w)
    assert (host(q) == qo).all() and (host(s).view(np.uint16) == so).all()


def test_quantize_act_rows_bit_exact(ctx, oracle):
    from tenzor_b200 import ops
    rng = np.random.default_rng(12)
    x = rng.normal(0, 3, (999, 384)).astype(np.float32)
    x[0] = 0.0
    q, s = ops.quantize_act_rows(ctx, dev(x))
    qo, so = oracle.quantize_act_rows(x)
    assert (host(q) == qo).all() and (host(s) == so).all()


def test_quantize_act_rows_ties_bit_exact(ctx, oracle):
    """Rounding edge cases of q = clamp(round_half_away(x / s)): rows whose |max| is 127 have s = 1,
    so x / s = x exactly and every half-integer is a tie."""
    from tenzor_b200 import ops
    edge = np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 125.5, -125.5, 126.5, -126.5, 127.0, -127.0,
                     0.49999997, -0.49999997, 0.50000006, -0.50000006, 2.4999998, -2.4999998, 0.0, -0.0,
                     1e-30, -1e-30, 63.5, -63.5, 126.49999, -126.49999, 3.0, -3.0], np.float32)
    rng = np.random.default_rng(13)
    rows = []
    for _ in range(64):
        r = rng.choice(edge, 384).astype(np.float32)
        r[rng.integers(0, 384)] = 127.0 if rng.random() < 0.5 else -127.0
        rows.append(r)
    halves = (rng.integers(-254, 255, (64, 384)) / 2.0).astype(np.float32)  # every value a tie or an integer
    halves[:, 0] = 127.0
    x = np.concatenate([np.stack(rows), halves, rng.normal(0, 3, (32, 384)).astype(np.float32) * 37.0])
    q, s = ops.quantize_act_rows(ctx, dev(x))
    qo, so = oracle.quantize_act_rows(x)
    assert (host(s) == so).all()
    assert (host(q) == qo).all()


@pytest.mark.parametrize("case", kats.LAYERNORM, ids=[c[0] for c in kats.LAYERNORM])
def test_layernorm_kats(ctx, case):
    from tenzor_b200 import ops
    _, x, g, b, check = case
    y = ops.layer_norm_last_dim(ctx, dev(np.array(x, np.float32)), dev(np.array(g, np.float32)),
                                dev(np.array(b, np.float32)), kats.LN_EPS_DEFAULT)
    kats.check_layernorm(check, host(y))


@pytest.mark.parametrize("rows,cols", [(32768, 384), (1, 384), (1000, 100), (77, 1024)])
def test_layernorm_vs_oracle(ctx, oracle, rows, cols):
    from tenzor_b200 import ops
    rng = np.random.default_rng(rows + cols)
    x = rng.normal(0.5, 2, (rows, cols)).astype(np.float32)
    g = rng.normal(1, 0.1, cols).astype(np.float32)
    b = rng.normal(0, 0.1, cols).astype(np.float32)
    y = host(ops.layer_norm_last_dim(ctx, dev(x), dev(g), dev(b), 1e-12))
    assert np.abs(y - oracle.layernorm(x, g, b, 1e-12)).max() < 2e-5


@pytest.mark.parametrize("case", kats.SOFTMAX, ids=[c[0] for c in kats.SOFTMAX])
def test_softmax_kats(ctx, case):
    from tenzor_b200 import ops
    _, x, mask, want, tol = case
    y = ops.softmax_last_axis(ctx, dev(np.array(x, np.float32)),
                              None if mask is None else dev(np.array(mask, np.float32)))
    assert np.abs(host(y) - np.array(want)).max() <= tol


def test_softmax_masked_vs_oracle(ctx, oracle):
    from tenzor_b200 import ops
    rng = np.random.default_rng(5)
    x = rng.normal(0, 3, (96, 128, 128)).astype(np.float32)
    lens = rng.integers(16, 129, 96).astype(np.int32)
    mask = np.where(np.arange(128)[None, None, :] < lens[:, None, None], 0.0, -np.inf).astype(np.float32)
    mask = np.broadcast_to(mask, x.shape).copy()
    ref = oracle.softmax(x, mask)
    y = host(ops.softmax_last_axis(ctx, dev(x), dev(mask)))
    assert np.abs(y - ref).max() < 1e-6
    yk = host(ops.softmax_keylen(ctx, dev(x), dev(lens)))
    assert np.abs(yk - ref).max() < 1e-6
    y2 = host(ops.softmax_last_axis(ctx, dev(x[:, :, :100].copy())))
    assert np.abs(y2 - oracle.softmax(x[:, :, :100])).max() < 1e-6


def test_ew_chain(ctx, oracle):
    from tenzor_b200 import ops
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (512, 4096)).astype(np.float32)
    c = rng.uniform(-1, 1, (512, 4096)).astype(np.float32)
    b = rng.uniform(-1, 1, 4096).astype(np.float32)
    y = host(ops.ew_add_mul_exp(ctx, dev(a), dev(b), dev(c)))
    ref = oracle.ew_add_mul_exp(a, b, c)
    assert np.abs(y / ref - 1).max() < 1e-6
    x, chain, want, tol = kats.EW_CHAIN
    z = host(ops.ew_unary_chain(ctx, dev(np.array(x, np.float32)), chain))
    assert np.abs(z - np.array(want)).max() <= tol


def test_reduce(ctx, oracle):
    from tenzor_b200 import ops
    for op, pre, x, want, tol in kats.REDUCE:
        assert abs(host(ops.reduce(ctx, op, pre, dev(np.array(x, np.float32))))[0] - want) <= tol
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, 10_000_019).astype(np.float32)
    for op, code in (("sum", 0), ("mean", 1), ("max", 3), ("min", 4)):
        got = host(ops.reduce(ctx, op, ["relu"], dev(x)))[0]
        want = oracle.reduce(code, [2], x)
        assert abs(got - want) <= 1e-5 * max(1.0, abs(want)), op
    empty = host(ops.reduce(ctx, "sum", [], dev(np.zeros(0, np.float32))))[0]
    assert empty == 0.0


def test_gather(ctx):
    from tenzor_b200 import ops, TenzorError
    for _, table, ids, want in kats.GATHER:
        y = ops.gather_rows(ctx, dev(np.array(table, np.float32)), dev(np.array(ids, np.uint32).view(np.int32)))
        assert (host(y) == np.array(want, np.float32)).all()
    y = ops.gather_rows(ctx, dev(np.ones((4, 8), np.float32)), dev(np.array([0, 9], np.int32)))
    torch.cuda.synchronize()
    with pytest.raises(TenzorError):
        ctx.check_status()
    assert (host(y)[1] == 0).all()
    ctx.check_status()  # cleared by the read


def test_bounded_device_wait_expires_and_context_stays_usable(ctx, oracle):
    """Failure detection without a GPU fault: a kernel waits on an mbarrier nothing arrives on; its
    bounded wait (the one every kernel uses) expires after ~1 s, the kernel returns, the host reads
    TZ_ETIMEOUT from the status word, and the same context keeps computing correctly."""
    import time
    from tenzor_b200 import _lib as L, ops
    t0 = time.perf_counter()
    rc = L.lib().tz_cuda_selftest_wait(ctx.handle)
    dt = time.perf_counter() - t0
    assert rc == L.TZ_ETIMEOUT, rc
    assert 0.5 < dt < 30
    assert L.lib().tz_cuda_check_status(ctx.handle) == L.TZ_OK  # the status word was cleared
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (64, 384)).astype(np.float32)
    g, b = np.ones(384, np.float32), np.zeros(384, np.float32)
    y = host(ops.layer_norm_last_dim(ctx, dev(x), dev(g), dev(b), 1e-12))
    assert np.abs(y - oracle.layernorm(x, g, b, 1e-12)).max() < 2e-5
