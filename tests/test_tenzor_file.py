"""The .tenzor checkpoint format (src/io/tenzor_format.zig): the C reader (memory-mapped, through
the C ABI, no GPU needed) against the Python writer, the reference's own format tests
(tenzor_format.zig:491-575), published FNV-1a vectors, corrupt files, and on the GPU the two model
loaders against the in-memory and safetensors loaders (bit-identical outputs)."""
import os
import struct
import tempfile

import numpy as np
import pytest

from tenzor_b200 import synthetic as S
from tenzor_b200 import tenzor_file as TF
from tenzor_b200._lib import TZ_EMISSING, TenzorError, lib


def _tmp(d, name="t.tenzor"):
    return os.path.join(d, name)


def test_hash_name_published_fnv1a_vectors():
    # FNV-1a 64-bit test vectors from the FNV reference material
    for s, h in [("", 0xCBF29CE484222325), ("a", 0xAF63DC4C8601EC8C), ("foobar", 0x85944171F73967E8)]:
        assert TF.hash_name(s) == h
        assert lib().tz_tenzor_hash_name(s.encode(), len(s.encode())) == h


def test_hash_name_distinguishes_names():  # tenzor_format.zig "hash name"
    assert TF.hash_name("conv1.weight") == TF.hash_name("conv1.weight")
    assert TF.hash_name("conv1.weight") != TF.hash_name("conv1.bias")


def test_write_and_read():  # tenzor_format.zig "write and read tenzor file"
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        w1 = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
        w2 = np.array([0.1, 0.2, 0.3], np.float32)
        TF.write(p, {"layer1.weight": w1, "layer1.bias": w2}, '{"model":"test"}')
        raw = open(p, "rb").read()
        assert raw[:8] == b"TENZOR\x00\x00" and struct.unpack_from("<I", raw, 8)[0] == 1
        index_offset, data_offset = struct.unpack_from("<QQ", raw, 24)
        assert index_offset == 64 + 16 and data_offset % 4096 == 0 and len(raw) == data_offset + 36
        with TF.TenzorFile(p) as f:
            assert len(f) == 2
            e = f.entry(0)
            assert e["shape"] == (2, 3) and e["dtype"] == 0 and e["bytes"] == 24
            assert e["name_hash"] == TF.hash_name("layer1.weight")
            assert np.array_equal(f.get("layer1.weight"), w1)
            assert np.array_equal(f.get("layer1.bias"), w2)
            assert f.metadata() == {"model": "test"}
            with pytest.raises(TenzorError) as ei:
                f.get("layer2.weight")
            assert ei.value.code == TZ_EMISSING


def test_dtypes_and_ranks_round_trip():
    rng = np.random.default_rng(3)
    t = [("a", rng.standard_normal((2, 3, 4, 5, 2)).astype(np.float32)),
         ("b", rng.integers(-128, 127, (7,), dtype=np.int8)),
         ("c", rng.standard_normal((3, 5)).astype(np.float16)),
         ("d", rng.integers(0, 1 << 40, (4,), dtype=np.int64)),
         ("e", np.array(3.5, np.float64)),
         ("f", rng.integers(0, 65535, (2, 2), dtype=np.uint16), 2)]  # bf16 words, stored under code 2
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        TF.write(p, t)
        with TF.TenzorFile(p) as f:
            for it in t:
                got = f.get(it[0])
                assert got.shape == it[1].shape and np.array_equal(got.view(it[1].dtype), it[1])
            assert f.entry(5)["dtype"] == 2


def _corrupt(raw, off, fmt, val):
    b = bytearray(raw)
    struct.pack_into(fmt, b, off, val)
    return bytes(b)


def test_corrupt_files_are_rejected():
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        TF.write(p, {"x": np.ones((4, 4), np.float32)})
        raw = open(p, "rb").read()
        bad = {
            "magic": b"TENSOR\x00\x00" + raw[8:],
            "version": _corrupt(raw, 8, "<I", 2),
            "index past end": _corrupt(raw, 24, "<Q", len(raw)),
            "count past end": _corrupt(raw, 16, "<I", 1 << 20),
            "data past end": _corrupt(raw, 64 + 8 + 32, "<Q", 1 << 40),   # entry 0's data offset
            "size vs shape": _corrupt(raw, 64 + 8 + 40, "<Q", 60),        # entry 0's size
            "rank": _corrupt(raw, 64 + 8 + 9, "<B", 6),
            "truncated": raw[:40],
        }
        for why, blob in bad.items():
            q = _tmp(d, why.replace(" ", "_") + ".tenzor")
            open(q, "wb").write(blob)
            with pytest.raises(TenzorError):
                TF.TenzorFile(q)
        with pytest.raises(TenzorError):
            TF.TenzorFile(_tmp(d, "absent.tenzor"))


def test_empty_file_and_empty_tensor():
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        TF.write(p, {}, "")
        with TF.TenzorFile(p) as f:
            assert len(f) == 0 and f.metadata() == {}
        TF.write(p, {"z": np.zeros((0, 4), np.float32), "a": np.ones(2, np.float32)})
        with TF.TenzorFile(p) as f:
            assert f.get("z").shape == (0, 4) and np.array_equal(f.get("a"), np.ones(2, np.float32))


def test_repeated_hash_first_entry_wins():
    # getTensorByHash's linear scan returns the first matching entry
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        TF.write(p, [("w", np.zeros(3, np.float32)), ("w", np.ones(3, np.float32))])
        with TF.TenzorFile(p) as f:
            assert len(f) == 2 and np.array_equal(f.get("w"), np.zeros(3, np.float32))


def _lenet_ckpt(w):
    from tenzor_b200.lenet import FIELDS
    return {ref: w[c] if c in w else w[ref] for ref, c in FIELDS}


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [S.LENET_REF, S.LENET_PAD2])
def test_lenet_from_tenzor_matches_in_memory(ctx, variant):
    from tenzor_b200.lenet import LeNet
    w = S.lenet_weights(77, variant, random_bias=True)
    x = S.lenet_images(300, seed=5)
    with tempfile.TemporaryDirectory() as d:
        p = _tmp(d)
        TF.write(p, _lenet_ckpt(w), '{"epoch":1,"model_name":"lenet"}')
        a, b = LeNet(ctx, w, variant), LeNet.from_tenzor(ctx, p, variant)
        try:
            assert np.array_equal(a.forward(x), b.forward(x))
        finally:
            a.close()
            b.close()
        ck = _lenet_ckpt(w)
        del ck["fc2_bias"]
        TF.write(p, ck)
        with pytest.raises(TenzorError) as ei:
            LeNet.from_tenzor(ctx, p, variant)
        assert ei.value.code == TZ_EMISSING
        TF.write(p, _lenet_ckpt(S.lenet_weights(77, 1 - variant)))  # the other network's fc1 width
        with pytest.raises(TenzorError):
            LeNet.from_tenzor(ctx, p, variant)


@pytest.mark.gpu
def test_arctic_from_tenzor_matches_safetensors(ctx, oracle):
    from tenzor_b200 import safetensors as st
    from tenzor_b200.arctic import ArcticModel
    w = S.arctic_weights(99, random_ln=True)
    q = oracle.quantize_checkpoint(w)
    ids, lens = S.token_batch(6, 128, 16, 128, seed=3)
    packed, cu = S.pack(ids, lens)
    with tempfile.TemporaryDirectory() as d:
        for name, ck, mode in [("f32", {"bert." + k: v for k, v in w.items()}, "f32"), ("i8", q, "w8a8")]:
            ps, pt = _tmp(d, name + ".safetensors"), _tmp(d, name + ".tenzor")
            st.save(ps, ck)
            TF.convert_from_safetensors(ps, pt)
            a, b = ArcticModel.from_safetensors(ctx, ps, mode), ArcticModel.from_tenzor(ctx, pt, mode)
            try:
                assert np.array_equal(a.forward_packed(packed, cu), b.forward_packed(packed, cu))
            finally:
                a.close()
                b.close()
