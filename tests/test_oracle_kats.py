"""Pins the CPU oracle (oracle/tz_oracle.c) against the reference's own unit-test known answers and
against an independent PyTorch-f32 restatement of the Arctic forward.  CPU only."""
import numpy as np
import pytest

import kats
from tenzor_b200 import synthetic as S


def test_gelu_model_kats(oracle):
    for _, x, want, tol in kats.GELU_MODEL:
        assert abs(oracle.gelu_model(x) - want) <= tol
    assert -0.01 < oracle.gelu_model(-3.0) < 0  # arctic.zig:1037-1039
    assert oracle.gelu_model(1.0) < oracle.gelu_model(2.0)  # monotone, arctic.zig:1044


def test_l2_normalize_kat(oracle):
    x, want, tol = kats.L2
    y = oracle.l2_normalize(np.array(x, np.float32))
    assert np.abs(y - np.array(want)).max() <= tol
    assert abs(np.linalg.norm(y) - 1.0) <= tol
    z = oracle.l2_normalize(np.zeros(4, np.float32))  # norm <= 1e-12: untouched, arctic.zig:860
    assert (z == 0).all()


@pytest.mark.parametrize("case", kats.LAYERNORM, ids=[c[0] for c in kats.LAYERNORM])
def test_layernorm_kats(oracle, case):
    _, x, g, b, check = case
    y = oracle.layernorm(np.array(x, np.float32), np.array(g, np.float32), np.array(b, np.float32),
                         kats.LN_EPS_DEFAULT)
    kats.check_layernorm(check, y)


@pytest.mark.parametrize("case", kats.SOFTMAX, ids=[c[0] for c in kats.SOFTMAX])
def test_softmax_kats(oracle, case):
    _, x, mask, want, tol = case
    y = oracle.softmax(np.array(x, np.float32), None if mask is None else np.array(mask, np.float32))
    assert np.abs(y - np.array(want)).max() <= tol


def test_softmax_stability(oracle):
    y = oracle.softmax(np.array(kats.SOFTMAX_STABILITY, np.float32))[0]
    assert np.isfinite(y).all() and abs(y.sum() - 1) < 1e-5 and y[2] > y[1] > y[0]


@pytest.mark.parametrize("case", kats.MATMUL_NN, ids=[c[0] for c in kats.MATMUL_NN])
def test_matmul_kats(oracle, case):
    _, a, b, want = case
    c = oracle.sgemm_nn(np.array(a, np.float32), np.array(b, np.float32))
    assert np.abs(c - np.array(want)).max() <= 1e-6
    ct = oracle.sgemm_nt(np.array(a, np.float32), np.array(b, np.float32).T.copy())
    assert np.abs(ct - np.array(want)).max() <= 1e-6


def test_matmul_pattern(oracle):
    a, b, want = kats.matmul_pattern()
    assert np.abs(oracle.sgemm_nn(a, b) - want).max() <= 1e-4


def test_fusion_kats(oracle):
    a, b, bias, ops, want = kats.MATMUL_EPILOGUE
    codes = [{"add": 1, "relu": 2}[o] for o in ops]
    c = oracle.matmul_epilogue(np.array(a, np.float32), np.array(b, np.float32), np.array(bias, np.float32), codes)
    assert (c == np.array(want, np.float32)).all()
    x, chain, want, tol = kats.EW_CHAIN
    y = [oracle.unary(2, oracle.unary(6, v)) for v in x]
    assert np.abs(np.array(y) - np.array(want)).max() <= tol
    for op, pre, x, want, tol in kats.REDUCE:
        codes = [{"exp": 6, "relu": 2}[p] for p in pre]
        assert abs(oracle.reduce(0, codes, np.array(x, np.float32)) - want) <= tol


def test_gelu_variants_close(oracle):
    # The model GELU (std.math.tanh) and the fusion GELU (2*sigmoid(2x)-1) are two f32
    # formulations of the same function; they agree to a few ulps-of-1.
    for x in np.linspace(-6, 6, 101):
        assert abs(oracle.gelu_model(x) - oracle.gelu_simd(x)) < 1e-5


def test_f16_rounding_matches_ieee(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500), [65504, 65520, 1e-8, 6e-8, -0.0, 3e-5]])
    x = x.astype(np.float32)
    ours = oracle.f32_to_f16_bits(x)
    ref = x.astype(np.float16).view(np.uint16)
    assert (ours == ref).all()


def test_weight_quantizer_rule(oracle):
    # quantize_arctic_xs.zig:94-115: s = f16(max/127); q = clamp(round(w / f32(s)))
    w = np.array([[0.5, -1.0, 0.25, 0.0], [0, 0, 0, 0], [1e-3, -2e-3, 3e-3, 127.0]], np.float32)
    q, s = oracle.quantize_weight_rows(w)
    s32 = s.view(np.float16).astype(np.float32)
    assert s32[1] == 1.0 and (q[1] == 0).all()  # all-zero row -> scale 1
    for r in range(3):
        inv = np.float32(1.0) / s32[r]
        t = (w[r] * inv).astype(np.float32)
        want = np.clip(np.sign(t) * np.floor(np.abs(t) + 0.5), -127, 127)  # half away from zero
        assert (q[r] == want).all()
    assert q[0, 1] == -127 and q[2, 3] == 127


def test_act_quantizer_and_w8a8_linear(oracle):
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, (17, 64)).astype(np.float32)
    x[3] = 0
    wq = rng.integers(-127, 128, (40, 64)).astype(np.int8)
    s16 = (rng.uniform(1e-3, 1e-2, 40).astype(np.float16)).view(np.uint16)
    bias = rng.normal(0, 1, 40).astype(np.float32)
    q, s = oracle.quantize_act_rows(x)
    assert s[3] == 1.0 and (q[3] == 0).all()
    acc = oracle.gemm_i8_i32(q, wq)
    assert (acc == q.astype(np.int64) @ wq.astype(np.int64).T).all()
    y = oracle.linear_w8a8(x, wq, s16, bias)
    assert (y == oracle.dequant_epilogue(acc, s, s16, bias)).all()


def _torch_forward(w, ids, lens):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))

    def lin(x, n):
        return x @ t(w[n + ".weight"]).T + t(w[n + ".bias"])

    def ln(x, n):
        return torch.nn.functional.layer_norm(x, (384,), t(w[n + ".weight"]), t(w[n + ".bias"]), 1e-12)

    outs = []
    for b in range(len(lens)):
        L = int(lens[b])
        tok = torch.from_numpy(ids[b, :L].astype(np.int64))
        x = t(w["embeddings.word_embeddings.weight"])[tok] + t(w["embeddings.position_embeddings.weight"])[:L] \
            + t(w["embeddings.token_type_embeddings.weight"])[0]
        x = ln(x, "embeddings.LayerNorm")
        for i in range(6):
            n = S.layer_names(i)
            q, k, v = (lin(x, n[c]).view(L, 12, 32).transpose(0, 1) for c in ("q", "k", "v"))
            p = torch.softmax((q @ k.transpose(1, 2)) * (1 / np.sqrt(32.0)), -1)
            o = (p @ v).transpose(0, 1).reshape(L, 384)
            x = ln(x + lin(o, n["o"]), n["ln1"])
            h = lin(x, n["ffn1"])
            h = 0.5 * h * (1 + torch.tanh(0.7978845608 * (h + 0.044715 * h ** 3)))
            x = ln(x + lin(h, n["ffn2"]), n["ln2"])
        outs.append((x[0] / x[0].norm()).numpy())
    return np.stack(outs)


def test_oracle_forward_vs_independent_torch(oracle):
    w = S.arctic_weights(99, random_ln=True)
    ids, lens = S.token_batch(4, 40, 1, 40, seed=3)
    packed, cu = S.pack(ids, lens)
    ref = oracle.OracleModel(w).forward(packed, cu, oracle.MODE_F32)
    alt = _torch_forward(w, ids, lens)
    assert np.abs(ref - alt).max() < 2e-6


def test_oracle_int8_modes_close_to_f32(oracle):
    w = S.arctic_weights(5)
    ids, lens = S.token_batch(3, 32, 8, 32, seed=4)
    packed, cu = S.pack(ids, lens)
    f32 = oracle.OracleModel(w).forward(packed, cu, oracle.MODE_F32)
    qm = oracle.OracleModel(oracle.quantize_checkpoint(w))
    for mode in (oracle.MODE_W8A32, oracle.MODE_W8A8):
        y = qm.forward(packed, cu, mode)
        cos = (y * f32).sum(1)
        assert cos.min() > 0.999 and np.abs(y - f32).max() < 5e-3


def test_oracle_rejects_bad_input(oracle):
    m = oracle.OracleModel(S.arctic_weights(5))
    with pytest.raises(ValueError):
        m.forward(np.array([101, 30522], np.uint32), np.array([0, 2], np.int32), oracle.MODE_F32)
    with pytest.raises(ValueError):
        m.forward(np.zeros(0, np.uint32), np.array([0, 0], np.int32), oracle.MODE_F32)
