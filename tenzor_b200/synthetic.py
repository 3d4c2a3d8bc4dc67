"""Seeded synthetic inputs and weights for the Arctic-embed-xs hot path.

There is no network and no checkpoint, so every benchmark and parity case runs on seeded synthetic
data with the shapes and distributions of the reference workloads:

* weights: N(0, 0.02) for every Linear weight/bias and every embedding table, LayerNorm gamma=1,
  beta=0 (``random_ln=True`` perturbs them for the parity tests so that a dropped gamma/beta shows);
* token batches: a leading CLS id 101, body ids uniform in [1000, 30521], per-row valid length
  uniform in [lmin, lmax], padding id 0.

One documented PRNG drives everything: counter-based splitmix64 (value i of stream ``seed`` is
``mix(seed + (i+1) * 0x9E3779B97F4A7C15)``, identical to sequential splitmix64 seeded with
``seed``), and Box-Muller (in float64) for normals.  Tensor names follow the reference's
non-prefixed safetensors naming (``embeddings.*``, ``encoder.layer.{i}.*``,
arctic.zig:138-149 and 302-339).
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
HIDDEN, LAYERS, HEADS, FFN, VOCAB, MAX_POS, TYPES = 384, 6, 12, 1536, 30522, 512, 2
CLS_ID = 101


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n consecutive outputs of splitmix64 seeded with ``seed`` (uint64 array)."""
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform01(seed: int, n: int) -> np.ndarray:
    """float64 uniforms in (0, 1) from the top 53 bits."""
    z = splitmix64(seed, n)
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def uniform(seed: int, shape, lo: float, hi: float) -> np.ndarray:
    n = int(np.prod(shape))
    return (lo + (hi - lo) * uniform01(seed, n)).astype(np.float32).reshape(shape)


def normal(seed: int, shape, std: float) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u = uniform01(seed, 2 * m)
    r = np.sqrt(-2.0 * np.log(u[0::2]))
    t = 2.0 * np.pi * u[1::2]
    z = np.empty(2 * m, dtype=np.float64)
    z[0::2] = r * np.cos(t)
    z[1::2] = r * np.sin(t)
    return (z[:n] * std).astype(np.float32).reshape(shape)


def randint(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Uniform integers in [lo, hi] (inclusive)."""
    z = splitmix64(seed, n)
    return (np.uint64(lo) + z % np.uint64(hi - lo + 1)).astype(np.int64)


def _layer_names(i: int):
    p = f"encoder.layer.{i}."
    return {
        "q": p + "attention.self.query",
        "k": p + "attention.self.key",
        "v": p + "attention.self.value",
        "o": p + "attention.output.dense",
        "ln1": p + "attention.output.LayerNorm",
        "ffn1": p + "intermediate.dense",
        "ffn2": p + "output.dense",
        "ln2": p + "output.LayerNorm",
    }


def arctic_weights(seed: int = 1234, std: float = 0.02, random_ln: bool = False) -> dict:
    """All f32 tensors of an Arctic-embed-xs checkpoint, by reference name."""
    w = {}
    s = [seed * 1000003]

    def nxt():
        s[0] += 1
        return s[0]

    def ln(name, n):
        if random_ln:
            w[name + ".weight"] = (1.0 + normal(nxt(), (n,), 0.1)).astype(np.float32)
            w[name + ".bias"] = normal(nxt(), (n,), 0.1)
        else:
            w[name + ".weight"] = np.ones(n, np.float32)
            w[name + ".bias"] = np.zeros(n, np.float32)

    w["embeddings.word_embeddings.weight"] = normal(nxt(), (VOCAB, HIDDEN), std)
    w["embeddings.position_embeddings.weight"] = normal(nxt(), (MAX_POS, HIDDEN), std)
    w["embeddings.token_type_embeddings.weight"] = normal(nxt(), (TYPES, HIDDEN), std)
    ln("embeddings.LayerNorm", HIDDEN)
    for i in range(LAYERS):
        n = _layer_names(i)
        for key, (o, k) in (("q", (HIDDEN, HIDDEN)), ("k", (HIDDEN, HIDDEN)),
                            ("v", (HIDDEN, HIDDEN)), ("o", (HIDDEN, HIDDEN)),
                            ("ffn1", (FFN, HIDDEN)), ("ffn2", (HIDDEN, FFN))):
            w[n[key] + ".weight"] = normal(nxt(), (o, k), std)
            w[n[key] + ".bias"] = normal(nxt(), (o,), std)
        ln(n["ln1"], HIDDEN)
        ln(n["ln2"], HIDDEN)
    return w


def layer_names(i: int) -> dict:
    return _layer_names(i)


def token_batch(batch: int, seq: int, lmin: int, lmax: int, seed: int = 7):
    """Padded ids [B, S] (uint32), valid lengths [B] (int32): ids[:,0]=101, body U{1000..30521},
    padding 0, L_i ~ U{lmin..lmax}."""
    lens = randint(seed * 2 + 1, batch, lmin, lmax).astype(np.int32)
    body = randint(seed * 2 + 2, batch * seq, 1000, VOCAB - 1).reshape(batch, seq)
    ids = np.zeros((batch, seq), np.uint32)
    for b in range(batch):
        L = int(lens[b])
        ids[b, 0] = CLS_ID
        ids[b, 1:L] = body[b, 1:L]
    return ids, lens


def token_batch_with_lengths(lens: np.ndarray, seq: int, seed: int):
    """Padded ids [B, S] with the given valid lengths and their own seeded body ids (the token
    distribution of token_batch): equal-work batches with different tokens."""
    lens = np.asarray(lens, np.int32)
    body = randint(seed * 2 + 2, len(lens) * seq, 1000, VOCAB - 1).reshape(len(lens), seq)
    ids = np.zeros((len(lens), seq), np.uint32)
    for b in range(len(lens)):
        L = int(lens[b])
        ids[b, 0] = CLS_ID
        ids[b, 1:L] = body[b, 1:L]
    return ids


def pack(ids: np.ndarray, lens: np.ndarray):
    """Padded [B,S] ids + lengths -> (packed ids [T] uint32, cu_seqlens [B+1] int32)."""
    cu = np.zeros(len(lens) + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    packed = np.concatenate([ids[b, : int(lens[b])] for b in range(len(lens))]).astype(np.uint32)
    return packed, cu


# ---- LeNet-5 (lenet.zig) ----
LENET_REF, LENET_PAD2 = 0, 1


def lenet_weights(seed: int = 4321, variant: int = LENET_PAD2, random_bias: bool = False) -> dict:
    """Kaiming-uniform LeNet-5 weights (init.zig:33-38: U(-a, a), a = sqrt(6 / fan_in)); biases 0
    (initKaiming, lenet.zig:74-95) unless ``random_bias`` (parity tests).  Conv weights are
    [out, kh, kw, in] (NHWC), FC weights [out, in]; FC1 takes 256 (lenet.zig) or 400 (pad-2
    variant) features."""
    feat = 400 if variant == LENET_PAD2 else 256
    shapes = {"conv1_w": ((6, 5, 5, 1), 25), "conv2_w": ((16, 5, 5, 6), 150), "fc1_w": ((120, feat), feat),
              "fc2_w": ((84, 120), 120), "fc3_w": ((10, 84), 84)}
    w = {}
    for i, (k, (shape, fan_in)) in enumerate(shapes.items()):
        a = float(np.sqrt(6.0 / fan_in))
        w[k] = uniform(seed * 101 + i, shape, -a, a)
        b = k[:-2] + "_b"
        n = shape[0]
        w[b] = uniform(seed * 101 + 50 + i, (n,), -0.1, 0.1) if random_bias else np.zeros(n, np.float32)
    return w


def lenet_images(n: int, seed: int = 11) -> np.ndarray:
    """n images [n, 28, 28, 1] f32, U[0, 1] pixels."""
    return uniform(seed, (n, 28, 28, 1), 0.0, 1.0)
