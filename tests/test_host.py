"""Host-side logic: seeded generators, packing, safetensors IO, sharding, quantiser rule, weight
name resolution, bench bookkeeping.  CPU only."""
import os
import sys

import numpy as np
import pytest

from tenzor_b200 import synthetic as S

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_splitmix64_known_values():
    # splitmix64 seeded with 0: the published first outputs
    assert [int(x) for x in S.splitmix64(0, 3)] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def test_token_batch_distribution():
    ids, lens = S.token_batch(256, 128, 16, 128, seed=7)
    assert ids.shape == (256, 128) and ids.dtype == np.uint32
    assert lens.min() >= 16 and lens.max() <= 128
    assert (ids[:, 0] == 101).all()
    for b in range(256):
        L = lens[b]
        assert ids[b, 1:L].min() >= 1000 and ids[b, 1:L].max() <= 30521
        assert (ids[b, L:] == 0).all()
    ids2, lens2 = S.token_batch(256, 128, 16, 128, seed=7)
    assert (ids == ids2).all() and (lens == lens2).all()
    packed, cu = S.pack(ids, lens)
    assert cu[0] == 0 and cu[-1] == lens.sum() and len(packed) == lens.sum()


def test_weights_shapes_and_stats():
    w = S.arctic_weights(1)
    assert w["embeddings.word_embeddings.weight"].shape == (30522, 384)
    assert w["encoder.layer.5.output.dense.weight"].shape == (384, 1536)
    assert abs(float(w["embeddings.word_embeddings.weight"].std()) - 0.02) < 2e-4
    assert (w["encoder.layer.0.attention.output.LayerNorm.weight"] == 1).all()
    assert len(w) == 5 + 6 * 16


def test_safetensors_roundtrip(tmp_path):
    from tenzor_b200 import safetensors as st
    t = {"a.weight": np.arange(12, dtype=np.float32).reshape(3, 4), "a.weight.scale": np.array([15360, 1], np.uint16),
         "q": np.array([[-1, 2]], np.int8)}
    p = tmp_path / "x.safetensors"
    st.save(str(p), t)
    raw = p.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    assert raw[8:9] == b"{" and b'"F16"' in raw[8:8 + n]
    back = st.load(str(p))
    for k in t:
        assert (back[k] == t[k]).all() and back[k].dtype == t[k].dtype


def test_should_quantize_rule():
    from tenzor_b200 import quantize as Q  # imports torch lazily via ops; no device use here
    assert Q.should_quantize("encoder.layer.0.attention.self.query.weight", np.zeros((384, 384), np.float32))
    assert Q.should_quantize("embeddings.word_embeddings.weight", np.zeros((30522, 384), np.float32))
    assert not Q.should_quantize("embeddings.token_type_embeddings.weight", np.zeros((2, 384), np.float32))
    assert not Q.should_quantize("embeddings.LayerNorm.weight", np.zeros((384,), np.float32))
    assert not Q.should_quantize("x.LayerNorm.weight", np.zeros((64, 64), np.float32))
    assert not Q.should_quantize("x.bias", np.zeros((64, 64), np.float32))
    assert Q.should_quantize("x.weight", np.zeros((64, 64), np.float32))
    assert not Q.should_quantize("x.weight", np.zeros((63, 64), np.float32))


def test_shard_by_tokens_partition_and_balance():
    from tenzor_b200.shard import shard_by_tokens, work
    ids, lens = S.token_batch(2048, 512, 32, 512, seed=11)
    for world in (1, 2, 4, 8):
        parts = shard_by_tokens(lens, world)
        allidx = np.sort(np.concatenate(parts))
        assert (allidx == np.arange(2048)).all()
        loads = [work(lens[p]).sum() for p in parts]
        assert max(loads) / min(loads) < 1.01


def test_host_weight_resolution_aliases():
    from tenzor_b200.arctic import _HostWeights
    w = S.arctic_weights(2)
    alt = {"bert." + k.replace("LayerNorm.weight", "LayerNorm.gamma").replace("LayerNorm.bias", "LayerNorm.beta"): v
           for k, v in w.items()}
    a = _HostWeights(w).struct
    b = _HostWeights(alt).struct
    assert a.layers[3].output_ln_gamma and b.layers[3].output_ln_gamma
    assert a.word_embeddings.f32 and not a.word_embeddings.q8
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    q = O.quantize_checkpoint({k: v for k, v in w.items() if "layer.0." in k or "embeddings" in k})
    hq = _HostWeights(q).struct
    assert hq.layers[0].query.q8 and hq.layers[0].query.scale_f16 and not hq.layers[0].query.f32
    assert hq.token_type_embeddings.f32  # 768 elements: never quantised


def test_bench_flop_accounting():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.flop_useful([72]) == 6 * (3538944 * 72 + 1536 * 72 * 72)
    assert abs(bench.flop_useful([128]) / 1e9 - 2.869) < 1e-3


def test_bench_inputs_weak_and_strong_sharding():
    """configs[1] weak scaling: every rank gets the one-GPU batch's lengths (equal work) and its own
    tokens; configs[3] strong scaling: the fixed batch is dealt so that every sequence lands on exactly
    one rank."""
    sys.path.insert(0, ROOT)
    import bench
    ids, lens, shards = bench.make_inputs("c2", 4)
    assert len(shards) == 4 and all(len(s) == 256 for s in shards)
    for s in shards[1:]:
        assert np.array_equal(lens[s], lens[shards[0]])
        assert not np.array_equal(ids[s], ids[shards[0]])
    ids, lens, shards = bench.make_inputs("c4", 8, batch_override=512)
    allrows = np.sort(np.concatenate(shards))
    assert np.array_equal(allrows, np.arange(512))


def test_bench_metric_and_bytes_bookkeeping():
    sys.path.insert(0, ROOT)
    import bench
    # both arms print the same metric string (the driver divides them)
    assert bench.arctic_metric("c2", "w8a8") == bench.arctic_metric("c2", "w8a32") == "Arctic-embed-xs seq/s @seq128 (int8)"
    assert bench.arctic_metric("c4", "f32") == "Arctic-embed-xs seq/s @seq512 (f32)"
    # the fused FFN block's algorithmic bytes are the split pair's minus the GELU output's round trip
    T = 18106
    split = bench.class_bytes(5, T, 256, True) + bench.class_bytes(7, T, 256, True)
    fused = bench.class_bytes(6, T, 256, True)
    h_round_trip = T * (1536 * 2 + 4) * 2  # f16 H + its row |max|, written by FFN1 and read by FFN2
    assert split - fused == h_round_trip


def test_bench_clock_sampler_without_polling():
    """A rank that does not poll (under torchrun only rank 0 polls) still opens and closes cleanly."""
    sys.path.insert(0, ROOT)
    import bench
    c = bench.Clocks(0, poll=False)
    with c:
        c.begin()
        c.mark()
        c.end()
    assert c.t is None and c.proc is None
    assert "samples" in c.summary()
