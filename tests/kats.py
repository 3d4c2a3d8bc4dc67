"""Known-answer cases transcribed from the reference's own unit tests (inputs and the assertions
they make), shared by the oracle tests (CPU) and the kernel tests (GPU).  Each entry cites the
reference test it restates."""
import math

import numpy as np

LN_EPS_DEFAULT = 1e-5  # layernorm.zig:16 default_eps

# layernorm.zig:413-528
LAYERNORM = [
    # (name, x rows, gamma, beta, check)
    ("basic 1D", [[1, 2, 3, 4]], [1, 1, 1, 1], [0, 0, 0, 0], "mean0_var1"),
    ("gamma/beta", [[1, 2, 3, 4]], [2, 2, 2, 2], [1, 1, 1, 1], "mean1"),
    ("2D batch", [[1, 2, 3, 4], [10, 20, 30, 40]], [1, 1, 1, 1], [0, 0, 0, 0], "rows_equal"),
    ("transformer", [[1, 2, 3, 4], [-1, 0, 1, 2]], [1, 1, 1, 1], [0, 0, 0, 0], "mean0"),
    ("stability", [[1e6, 1e6 + 1, 1e6 + 2, 1e6 + 3]], [1, 1, 1, 1], [0, 0, 0, 0], "finite_mean0"),
]


def check_layernorm(kind, y):
    y = np.asarray(y, np.float64)
    if kind in ("mean0", "mean0_var1"):
        for r in y:
            assert abs(r.mean()) < 1e-5
        if kind == "mean0_var1":
            v = ((y[0] - y[0].mean()) ** 2).mean()
            assert 0.9 < v < 1.1
    elif kind == "mean1":
        assert abs(y[0].mean() - 1.0) < 1e-5
    elif kind == "rows_equal":
        assert abs(y[0].mean()) < 1e-5 and abs(y[1].mean()) < 1e-5
        assert np.abs(y[0] - y[1]).max() < 1e-5
    elif kind == "finite_mean0":
        assert np.isfinite(y).all() and abs(y[0].mean()) < 1e-4


def _sm(v):
    e = [math.exp(x - max(v)) for x in v]
    s = sum(e)
    return [x / s for x in e]


# softmax.zig:357-440 (x rows, additive mask rows or None, expected rows, tol)
SOFTMAX = [
    ("basic 1D", [[1.0, 2.0, 3.0]], None, [_sm([1, 2, 3])], 1e-5),
    ("2D batch", [[1, 2, 3], [0, 0, 0]], None, [_sm([1, 2, 3]), [1 / 3] * 3], 1e-5),
    ("attention mask", [[1.0, 2.0, 3.0]], [[-1e9, 0.0, 0.0]], [[0.0] + _sm([2, 3])], 1e-5),
    ("4D pattern", [[1, 2], [3, 4], [0, 0], [1, -1]], None,
     [_sm([1, 2]), _sm([3, 4]), [0.5, 0.5], _sm([1, -1])], 1e-5),
]
SOFTMAX_STABILITY = [[1000.0, 1001.0, 1002.0]]  # softmax.zig:380-399: finite, sums to 1, ordered

# matmul.zig:985-1016 (C = A @ B) and blazt_backend.zig 2x2 test
MATMUL_NN = [
    ("naive 2x2", [[1, 2], [3, 4]], [[5, 6], [7, 8]], [[19, 22], [43, 50]]),
    ("identity 3x3", [[1, 2, 3], [4, 5, 6], [7, 8, 9]], [[1, 0, 0], [0, 1, 0], [0, 0, 1]],
     [[1, 2, 3], [4, 5, 6], [7, 8, 9]]),
]


def matmul_pattern():
    """matmul.zig:1018-1038 'matmulTiled vs naive': m=64, k=48, n=32, i%10/10 and (i+3)%10/10."""
    m, k, n = 64, 48, 32
    a = (np.arange(m * k) % 10 / 10.0).astype(np.float32).reshape(m, k)
    b = ((np.arange(k * n) + 3) % 10 / 10.0).astype(np.float32).reshape(k, n)
    return a, b, (a.astype(np.float64) @ b.astype(np.float64))


# codegen.zig:331-348 fused matmul epilogue: [[1,2],[3,4]] @ I + [-10, 10], relu -> [[0,12],[0,14]]
MATMUL_EPILOGUE = ([[1, 2], [3, 4]], [[1, 0], [0, 1]], [-10, 10], ["add", "relu"], [[0, 12], [0, 14]])

# codegen.zig:299-316 relu(exp(x)); 350-369 sum(exp(0)) = 4, sum(relu) = 3
EW_CHAIN = ([-1, 0, 1, 2], ["exp", "relu"], [0.368, 1.0, 2.718, 7.389], 0.01)
REDUCE = [("sum", ["exp"], [0, 0, 0, 0], 4.0, 1e-3), ("sum", ["relu"], [-2, -1, 0, 1, 2], 3.0, 1e-3)]

# gather.zig:81-145
GATHER = [
    ("basic", [[1, 2, 3], [4, 5, 6], [7, 8, 9], [10, 11, 12]], [0, 2, 1], [[1, 2, 3], [7, 8, 9], [4, 5, 6]]),
    ("single", [[1, 2, 3, 4], [5, 6, 7, 8]], [1], [[5, 6, 7, 8]]),
    ("repeated", [[1, 2], [3, 4]], [0, 0, 1, 1, 0], [[1, 2], [1, 2], [3, 4], [3, 4], [1, 2]]),
]

# arctic.zig:1032-1057
GELU_MODEL = [("gelu(0)=0", 0.0, 0.0, 1e-6), ("gelu(3)~3", 3.0, 3.0, 0.01)]
L2 = ([3.0, 4.0], [0.6, 0.8], 1e-6)


# tokenizer.zig:291-439 -- the reference's inline tokenizer tests: (name, vocabulary put into the
# hash map, text, expected encode output).
TOKENIZER = [
    ("basic", {"[PAD]": 0, "[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "hello": 7592, "world": 2088, "##ing": 2075,
               "test": 3231, "##s": 1055}, "hello world", [101, 7592, 2088, 102]),
    ("wordpiece split", {"[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "test": 3231, "##ing": 2075}, "testing",
     [101, 3231, 2075, 102]),
    ("unknown word", {"[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "hello": 7592}, "xyz", [101, 100, 102]),
    ("punctuation", {"[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "hello": 7592, ",": 1010, "world": 2088},
     "hello, world", [101, 7592, 1010, 2088, 102]),
    ("lowercase", {"[UNK]": 100, "[CLS]": 101, "[SEP]": 102, "hello": 7592}, "HELLO", [101, 7592, 102]),
]

# src/tests/tokenizer_parity_test.zig:15-31 -- HuggingFace token ids of the real arctic-embed-xs
# vocab.txt (absent here).  Tests derive the vocabulary entries these cases imply (texts whose basic
# tokens map one-to-one onto the expected ids) and pin the tokenizer on those cases.
TOKENIZER_HF = [
    ("Hello world", [101, 7592, 2088, 102]),
    ("hello world", [101, 7592, 2088, 102]),
    ("HELLO WORLD", [101, 7592, 2088, 102]),
    ("Hello, world!", [101, 7592, 1010, 2088, 999, 102]),
    ("The quick brown fox jumps over the lazy dog.", [101, 1996, 4248, 2829, 4419, 14523, 2058, 1996, 13971, 3899, 1012, 102]),
    ("What is machine learning?", [101, 2054, 2003, 3698, 4083, 1029, 102]),
    ("testing", [101, 5604, 102]),
    ("embeddings", [101, 7861, 8270, 4667, 2015, 102]),
    ("I love programming in Zig!", [101, 1045, 2293, 4730, 1999, 1062, 8004, 999, 102]),
    ("", [101, 102]),
    ("a", [101, 1037, 102]),
    ("123", [101, 13138, 102]),
    ("hello-world", [101, 7592, 1011, 2088, 102]),
    ("don't", [101, 2123, 1005, 1056, 102]),
    ("   spaces   ", [101, 7258, 102]),
]

# onnx/executor.zig:6197-6244 ("Executor basic elementwise") and 6246-6293 ("Executor MatMul"):
# (op, A, B, shape A, shape B, expected C)
ONNX_EXECUTOR = [
    ("Add", [1, 2, 3, 4], [10, 20, 30, 40], (4,), (4,), [11, 22, 33, 44]),
    ("MatMul", [1, 2, 3, 4, 5, 6], [1, 2, 3, 4, 5, 6], (2, 3), (3, 2), [22, 28, 49, 64]),
]
