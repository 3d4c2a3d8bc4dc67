"""LeNet-5 batch inference (lenet.zig:262-321).

CPU: the C restatement (oracle/tz_oracle_lenet.c) against an independent PyTorch forward built from
torch.nn.functional (the reference ships no LeNet forward fixtures).  GPU: tz_lenet_* against the
restatement for both variants, ragged batch sizes (partial image groups and FC tiles), the host
and device entry points, and a user stream.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tenzor_b200 import synthetic as S

REF, PAD2 = S.LENET_REF, S.LENET_PAD2


def torch_lenet(w, variant, x):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    X = t(x).reshape(-1, 28, 28, 1).permute(0, 3, 1, 2)
    y = F.relu(F.conv2d(X, t(w["conv1_w"]).permute(0, 3, 1, 2), t(w["conv1_b"]), padding=2 if variant else 0))
    y = F.max_pool2d(y, 2, 2)
    y = F.relu(F.conv2d(y, t(w["conv2_w"]).permute(0, 3, 1, 2), t(w["conv2_b"])))
    y = F.max_pool2d(y, 2, 2)
    y = y.permute(0, 2, 3, 1).reshape(X.shape[0], -1)  # NHWC flatten, as lenet.zig
    y = F.relu(F.linear(y, t(w["fc1_w"]), t(w["fc1_b"])))
    y = F.relu(F.linear(y, t(w["fc2_w"]), t(w["fc2_b"])))
    y = F.linear(y, t(w["fc3_w"]), t(w["fc3_b"]))
    return (torch.softmax(y, -1) if variant else y).numpy()


@pytest.mark.parametrize("variant", [REF, PAD2])
def test_oracle_matches_torch(oracle, variant):
    w = S.lenet_weights(4321, variant, random_bias=True)
    x = S.lenet_images(96, seed=3)
    a = oracle.lenet_forward(w, variant, x)
    b = torch_lenet(w, variant, x)
    assert np.abs(a - b).max() <= 2e-5 * max(1.0, np.abs(b).max())
    if variant == PAD2:
        assert np.allclose(a.sum(1), 1.0, atol=1e-5)


def test_oracle_relu_pool_edge(oracle):
    """All-zero images: every conv output is its bias; ReLU then pooling pass biases through."""
    w = S.lenet_weights(5, REF, random_bias=True)
    x = np.zeros((3, 28, 28, 1), np.float32)
    a = oracle.lenet_forward(w, REF, x)
    b = torch_lenet(w, REF, x)
    assert np.abs(a - b).max() < 1e-5 and np.allclose(a[0], a[2])


def _tol(ref):
    return 1e-4 * max(1.0, float(np.abs(ref).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [REF, PAD2])
@pytest.mark.parametrize("n", [1, 5, 7, 64, 77, 1000])
def test_lenet_forward_vs_oracle(ctx, oracle, variant, n):
    from tenzor_b200.lenet import LeNet
    w = S.lenet_weights(4321, variant, random_bias=True)
    x = S.lenet_images(n, seed=n)
    m = LeNet(ctx, w, variant)
    try:
        out = m.forward(x)
    finally:
        m.close()
    ref = oracle.lenet_forward(w, variant, x)
    assert out.shape == (n, 10) and np.isfinite(out).all()
    assert np.abs(out - ref).max() <= _tol(ref)
    if variant == PAD2:
        assert np.allclose(out.sum(1), 1.0, atol=1e-5)


@pytest.mark.gpu
def test_lenet_device_forward_user_stream(ctx, oracle):
    from tenzor_b200.lenet import LeNet
    w = S.lenet_weights(99, PAD2)
    x = S.lenet_images(4099, seed=5)
    m = LeNet(ctx, w, PAD2)
    try:
        d_x = torch.from_numpy(x).cuda()
        d_o = torch.empty((4099, 10), device="cuda")
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            m.forward_device(d_x.data_ptr(), 4099, d_o.data_ptr(), s.cuda_stream)
        s.synchronize()
        out = d_o.cpu().numpy()
        host = m.forward(x)
    finally:
        m.close()
    assert np.array_equal(out, host)
    ref = oracle.lenet_forward(w, PAD2, x)
    assert np.abs(out - ref).max() <= _tol(ref)


@pytest.mark.gpu
def test_lenet_full_batch_properties(ctx, oracle):
    """configs[4] size (65536 images): rows are probability vectors; a strided sample of rows
    matches the restatement."""
    from tenzor_b200.lenet import LeNet
    n = 65536
    w = S.lenet_weights(4321, PAD2)
    x = S.lenet_images(n, seed=11)
    m = LeNet(ctx, w, PAD2)
    try:
        out = m.forward(x)
    finally:
        m.close()
    assert np.isfinite(out).all() and np.allclose(out.sum(1), 1.0, atol=1e-5)
    idx = np.arange(0, n, 257)
    ref = oracle.lenet_forward(w, PAD2, x[idx])
    assert np.abs(out[idx] - ref).max() <= _tol(ref)


@pytest.mark.gpu
def test_lenet_missing_weight_rejected(ctx):
    from tenzor_b200.lenet import LeNet
    w = S.lenet_weights(1, REF)
    del w["fc2_b"]
    with pytest.raises(KeyError):
        LeNet(ctx, w, REF)
