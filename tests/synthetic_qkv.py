"""Seeded Q / K / V inputs for the attention tests ([T, 1152] f32 rows = Q | K | V, 12 heads of 32)."""
import numpy as np

from tenzor_b200 import synthetic as S


def normal_qkv(tokens: int, seed: int, std: float = 1.0) -> np.ndarray:
    """N(0, std) entries: scores of a few units, the spread of a trained model's attention logits."""
    return S.normal(seed * 7919 + 1, (tokens, 1152), std)


def ramp_qkv(lens, seed: int) -> np.ndarray:
    """Per sequence: K row t = 0.05 t in every dimension, so the score of key t is 1.6 t for Q = +1
    (growing by ~100 raw units per 64-key block) and -1.6 t for Q = -1; query rows alternate the sign
    (even rows +1), V is N(0, 1)."""
    T = int(np.sum(lens))
    x = np.zeros((T, 1152), np.float32)
    x[:, 768:] = S.normal(seed * 7919 + 2, (T, 384), 1.0)
    row = 0
    for L in lens:
        t = np.arange(L, dtype=np.float32)
        x[row:row + L, 384:768] = (0.05 * t)[:, None]
        x[row:row + L, :384] = np.where(t % 2 == 0, 1.0, -1.0).astype(np.float32)[:, None]
        row += L
    return x
