"""selfAttention (arctic.zig:639-747) on the CUDA kernels through the C ABI (`tz_attention`) against the
oracle's attention core (`tzo_attention_packed`, the same per-head scores / softmax / P V loop the
oracle's forward runs) on the same 16-bit Q / K / V.

Batches whose longest sequence exceeds 128 keys run the 8-warp kernel (128 queries per CTA, one
staging barrier per 64-key chunk); shorter batches the 4-warp kernel.  Tolerances: P and the
output are rounded to the 16-bit type (f16: 11 mantissa bits, outputs of magnitude <= ~4 here, half
an ulp = 1e-3; bf16: 8 bits)."""
import numpy as np
import pytest

import synthetic_qkv as Q

F16_ATOL, BF16_ATOL = 4e-3, 3e-2


def _run(ctx, qkv_np, lens, max_len, bf16=False):
    import torch
    from tenzor_b200 import ops
    dt = torch.bfloat16 if bf16 else torch.float16
    qkv = torch.from_numpy(qkv_np).to(dt).cuda()
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    out = ops.attention(ctx, qkv, cu, max_len)
    torch.cuda.synchronize()
    ctx.check_status()
    return out.float().cpu().numpy(), qkv.float().cpu().numpy(), cu.cpu().numpy()


def _check(ctx, oracle, qkv_np, lens, max_len, atol, bf16=False):
    got, q32, cu = _run(ctx, qkv_np, lens, max_len, bf16)
    ref = oracle.attention_packed(q32, cu)
    assert np.isfinite(got).all()
    d = np.abs(got - ref)
    worst = [(int(lens[b]), float(d[cu[b]:cu[b + 1]].max())) for b in range(len(lens)) if lens[b] > 0]
    print("per-length max-abs:", worst)
    assert d.max() < atol, worst
    return got, ref


LONG_LENS = [1, 512, 63, 64, 65, 127, 128, 129, 191, 192, 255, 256, 257, 300, 448, 511, 33, 2]


@pytest.mark.gpu
def test_long_sequences_vs_oracle(ctx, oracle):
    lens = np.array(LONG_LENS, np.int32)
    _check(ctx, oracle, Q.normal_qkv(int(lens.sum()), seed=1), lens, 512, F16_ATOL)


@pytest.mark.gpu
@pytest.mark.parametrize("max_len", [130, 192, 257, 320])
def test_max_len_between_block_edges(ctx, oracle, max_len):
    """lpad (max_len rounded up to 64) sizes the K / V staging; every length up to it."""
    lens = np.array([max_len, max_len - 1, 129, 1, 64, max_len // 2], np.int32)
    lens = np.minimum(lens, max_len)
    _check(ctx, oracle, Q.normal_qkv(int(lens.sum()), seed=max_len), lens, max_len, F16_ATOL)


@pytest.mark.gpu
def test_short_sequences_vs_oracle(ctx, oracle):
    lens = np.array([1, 2, 15, 16, 17, 63, 64, 65, 100, 127, 128, 31, 33], np.int32)
    _check(ctx, oracle, Q.normal_qkv(int(lens.sum()), seed=2), lens, 128, F16_ATOL)


@pytest.mark.gpu
def test_growing_scores_rescale_path(ctx, oracle):
    """Scores that grow by ~100 raw units per 64-key block on half of the query rows (Q = +1) and
    shrink on the other half (Q = -1), alternating row by row: the online softmax must rescale O and
    the row sum at every block for the growing rows and leave the others alone."""
    lens = np.array([512, 300, 200, 131], np.int32)
    qkv = Q.ramp_qkv(lens, seed=3)
    got, ref = _check(ctx, oracle, qkv, lens, 512, F16_ATOL)
    # the growing rows concentrate on their last keys, the shrinking ones on their first: both forms
    # of the softmax are exercised (not a degenerate constant output)
    assert np.abs(got[0] - got[1]).max() > 0.1


@pytest.mark.gpu
def test_bf16_long_sequences_vs_oracle(ctx, oracle):
    lens = np.array([512, 129, 300, 64, 1], np.int32)
    _check(ctx, oracle, Q.normal_qkv(int(lens.sum()), seed=4), lens, 512, BF16_ATOL, bf16=True)


@pytest.mark.gpu
def test_staging_size_does_not_change_rows(ctx, oracle):
    """The same sequences under max_len 512 and under their own maximum give the same rows (the
    staging size does not change the arithmetic)."""
    lens = np.array([200, 150, 133], np.int32)
    qkv = Q.normal_qkv(int(lens.sum()), seed=5)
    a, _, _ = _run(ctx, qkv, lens, 512)
    b, _, _ = _run(ctx, qkv, lens, 200)
    assert np.array_equal(a, b)


@pytest.mark.gpu
def test_length_beyond_max_len_is_refused(ctx):
    import torch
    from tenzor_b200 import ops
    from tenzor_b200._lib import TenzorError
    lens = np.array([300, 20], np.int32)
    qkv = torch.from_numpy(Q.normal_qkv(int(lens.sum()), seed=6)).half().cuda()
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    ops.attention(ctx, qkv, cu, 200)  # staging for 256 keys: the 300-key sequence is refused on the device
    torch.cuda.synchronize()
    with pytest.raises(TenzorError):
        ctx.check_status()
    out = ops.attention(ctx, qkv, cu, 300)  # the context stays usable
    torch.cuda.synchronize()
    ctx.check_status()
    assert torch.isfinite(out.float()).all()


@pytest.mark.gpu
def test_more_sequences_than_one_grid_dimension(ctx, oracle):
    """70,000 short sequences: the launches are split at 65,535 sequences (the grid's y extent)."""
    from tenzor_b200 import synthetic as S
    lens = S.randint(17, 70000, 1, 4).astype(np.int32)
    _check(ctx, oracle, Q.normal_qkv(int(lens.sum()), seed=9), lens, 4, F16_ATOL)
