"""Host-side mirror of the reference's Arctic-embed-xs model API (src/model/arctic.zig), backed by
the sm_100a kernels of libtenzor_cuda.so.

Reference -> here:
  Config (arctic.zig:29-45)                        -> Config
  ModelWeights.fromSafeTensors (arctic.zig:113)    -> ArcticModel.from_safetensors / from_checkpoint
  TenzorFile (tenzor_format.zig:140)               -> ArcticModel.from_tenzor
  forward(output, token_ids, weights, ctx) (874)   -> ArcticModel.forward(token_ids)
  forwardBatch / forwardBatchParallel (902, 959)   -> ArcticModel.forward_batch(list_of_ids)
  (packed device batch, no counterpart)            -> ArcticModel.forward_packed / forward_padded
Errors raise TenzorError carrying the C status (MissingWeight -> TZ_EMISSING, wrong dtype ->
TZ_EINVAL, as the reference's error unions at arctic.zig:194-201).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .runtime import Context

PRECS = {"f16": 0, "bf16": 1}
MODES = {"f32": L.QUANT_F32, "w8a32": L.QUANT_W8A32, "w8a8": L.QUANT_W8A8}


@dataclass(frozen=True)
class Config:
    """arctic.zig:29-45 (the kernels are built for exactly this configuration)."""
    hidden_size: int = 384
    num_hidden_layers: int = 6
    num_attention_heads: int = 12
    intermediate_size: int = 1536
    vocab_size: int = 30522
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12

    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


ARCTIC_EMBED_XS = Config()


def _names(i: int):
    p = f"encoder.layer.{i}."
    return {
        "query": p + "attention.self.query", "key": p + "attention.self.key",
        "value": p + "attention.self.value", "attn_output": p + "attention.output.dense",
        "intermediate": p + "intermediate.dense", "output": p + "output.dense",
        "attn_ln": p + "attention.output.LayerNorm", "output_ln": p + "output.LayerNorm",
    }


class _HostWeights:
    """Builds the C struct over a name -> numpy checkpoint (f32, or int8 + '<name>.scale' half
    bits), resolving the 'bert.' prefix and LayerNorm gamma/beta aliases like arctic.zig:130-156."""

    def __init__(self, ckpt: dict):
        prefix = "bert." if "bert.embeddings.word_embeddings.weight" in ckpt else ""
        self.keep = {}
        w = L.ArcticWeights()

        def arr(name, dtype):
            a = ckpt.get(prefix + name)
            if a is None:
                return None
            a = np.ascontiguousarray(a)
            if a.dtype != dtype:
                raise L.TenzorError(L.TZ_EINVAL, f"Weight {prefix + name} has wrong dtype {a.dtype}, expected {dtype}")
            self.keep[name] = a
            return a.ctypes.data

        def f32(name, alt=None):
            p = arr(name, np.float32)
            if p is None and alt:
                p = arr(alt, np.float32)
            return p

        def mat(name):
            a = ckpt.get(prefix + name)
            m = L.MatWeight()
            if a is None:
                return m
            if a.dtype == np.int8:
                m.q8 = arr(name, np.int8)
                s = ckpt.get(prefix + name + ".scale")
                if s is not None:
                    m.scale_f16 = arr(name + ".scale", np.uint16 if s.dtype != np.float16 else np.float16)
            else:
                m.f32 = arr(name, np.float32)
            return m

        e = "embeddings."
        w.word_embeddings = mat(e + "word_embeddings.weight")
        w.position_embeddings = mat(e + "position_embeddings.weight")
        w.token_type_embeddings = mat(e + "token_type_embeddings.weight")
        w.ln_gamma = f32(e + "LayerNorm.weight", e + "LayerNorm.gamma")
        w.ln_beta = f32(e + "LayerNorm.bias", e + "LayerNorm.beta")
        for i in range(6):
            n = _names(i)
            lw = w.layers[i]
            for k in ("query", "key", "value", "attn_output", "intermediate", "output"):
                setattr(lw, k, mat(n[k] + ".weight"))
                setattr(lw, k + "_bias", f32(n[k] + ".bias"))
            lw.attn_ln_gamma = f32(n["attn_ln"] + ".weight", n["attn_ln"] + ".gamma")
            lw.attn_ln_beta = f32(n["attn_ln"] + ".bias", n["attn_ln"] + ".beta")
            lw.output_ln_gamma = f32(n["output_ln"] + ".weight", n["output_ln"] + ".gamma")
            lw.output_ln_beta = f32(n["output_ln"] + ".bias", n["output_ln"] + ".beta")
        self.struct = w


class ArcticModel:
    """Device-resident Arctic-embed-xs (weights + workspace) on one B200."""

    def __init__(self, ctx: Context, handle: C.c_void_p, mode: str):
        self.ctx = ctx
        self.handle = handle
        self.mode = mode
        self.config = ARCTIC_EMBED_XS
        ctx._adopt(self)

    @classmethod
    def from_checkpoint(cls, ctx: Context, ckpt: dict, mode: str = "f32", prec: str = "f16") -> "ArcticModel":
        """`prec` is the 16-bit GEMM operand / activation type of the f32 and w8a32 modes: "f16" or
        "bf16" (tz_arctic_load_ex)."""
        hw = _HostWeights(ckpt)
        h = C.c_void_p()
        L.check(L.lib().tz_arctic_load_ex(ctx.handle, C.byref(hw.struct), MODES[mode], PRECS[prec], C.byref(h)))
        return cls(ctx, h, mode)

    @classmethod
    def from_safetensors(cls, ctx: Context, path: str, mode: str = "f32") -> "ArcticModel":
        h = C.c_void_p()
        L.check(L.lib().tz_arctic_load_safetensors(ctx.handle, path.encode(), MODES[mode], C.byref(h)))
        return cls(ctx, h, mode)

    @classmethod
    def from_tenzor(cls, ctx: Context, path: str, mode: str = "f32") -> "ArcticModel":
        """A .tenzor file converted from safetensors (tenzor_format.zig:441-485), memory-mapped."""
        h = C.c_void_p()
        L.check(L.lib().tz_arctic_load_tenzor(ctx.handle, path.encode(), MODES[mode], C.byref(h)))
        return cls(ctx, h, mode)

    def close(self):
        if self.handle:
            L.lib().tz_arctic_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, max_batch: int, max_tokens: int):
        L.check(L.lib().tz_arctic_reserve(self.handle, max_batch, max_tokens))

    # ---- forward variants -----------------------------------------------------------------
    def forward_packed(self, packed_ids: np.ndarray, cu_seqlens: np.ndarray,
                       out: np.ndarray | None = None) -> np.ndarray:
        """Host arrays in, host [B,384] out (H2D/D2H inside; synchronous)."""
        ids = np.ascontiguousarray(packed_ids, dtype=np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        B = len(cu) - 1
        if out is None:
            out = np.empty((B, 384), np.float32)
        L.check(L.lib().tz_arctic_forward(self.handle, ids.ctypes.data, cu.ctypes.data, B, out.ctypes.data))
        return out

    def forward_padded(self, ids: np.ndarray, lengths: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        lens = np.ascontiguousarray(lengths, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((B, 384), np.float32)
        L.check(L.lib().tz_arctic_forward_padded(self.handle, ids.ctypes.data, lens.ctypes.data, B, S,
                                                 out.ctypes.data))
        return out

    def forward_batch(self, token_ids_batch) -> np.ndarray:
        """forwardBatchParallel (arctic.zig:959): a list of 1-D id arrays -> [B, 384]."""
        seqs = [np.asarray(t, dtype=np.uint32) for t in token_ids_batch]
        cu = np.zeros(len(seqs) + 1, np.int32)
        cu[1:] = np.cumsum([len(s) for s in seqs])
        packed = np.concatenate(seqs) if seqs else np.zeros(0, np.uint32)
        return self.forward_packed(packed, cu)

    def forward(self, token_ids) -> np.ndarray:
        """forward (arctic.zig:874): one sequence -> its L2-normalised CLS embedding [384]."""
        return self.forward_batch([token_ids])[0]

    def embed_texts(self, tokenizer, texts) -> np.ndarray:
        """The embed CLI's text batch (main.zig:934-980): each text encoded into 512 ids
        ([CLS] ... [SEP]), one batched forward -> [n, 384]."""
        from .tokenizer import text_args
        bufs, ptrs, lens = text_args(texts)
        out = np.empty((len(bufs), 384), np.float32)
        L.check(L.lib().tz_arctic_embed_texts(self.handle, tokenizer.handle, C.cast(ptrs, C.c_void_p),
                                              lens.ctypes.data, len(bufs), out.ctypes.data))
        return out

    def embed_documents(self, tokenizer, documents) -> np.ndarray:
        """The embed CLI's long-document path (main.zig:796-925) for many documents at once:
        510-id chunks with 50 overlap, every chunk forwarded in one packed batch, the per-document
        mean of chunk embeddings L2-normalised on the device -> [n, 384]."""
        from .tokenizer import text_args
        bufs, ptrs, lens = text_args(documents)
        out = np.empty((len(bufs), 384), np.float32)
        L.check(L.lib().tz_arctic_embed_documents(self.handle, tokenizer.handle, C.cast(ptrs, C.c_void_p),
                                                  lens.ctypes.data, len(bufs), out.ctypes.data))
        return out

    def forward_device(self, d_ids, d_cu, batch: int, total_tokens: int, max_len: int, d_out,
                       stream=None):
        """Device-pointer variant (integers or torch tensors' data_ptr()), async on `stream` (a raw
        cudaStream_t handle; None = the context's own stream; 0x1 = the legacy default stream)."""
        L.check(L.lib().tz_arctic_forward_device(self.handle, int(d_ids), int(d_cu), batch, total_tokens,
                                                 max_len, int(d_out), C.c_void_p(stream) if stream else None))

    def set_ffn_fusion(self, fused: bool = True):
        """W8A8: the feed-forward block as one kernel with the GELU output kept on chip, or (the
        default, faster on B200) as the FFN1 GEMM + FFN2 kernel pair with the GELU output through
        device memory.  Both forms give bit-identical results."""
        L.check(L.lib().tz_arctic_set_ffn_fusion(self.handle, int(bool(fused))))

    # ---- parity hooks -----------------------------------------------------------------------
    def debug_hidden(self, stage: int, total_tokens: int) -> np.ndarray:
        out = np.empty((total_tokens, 384), np.float32)
        L.check(L.lib().tz_arctic_debug_hidden(self.handle, stage, out.ctypes.data, total_tokens))
        return out

    def enable_capture(self, on: bool = True):
        """Switches stage / operand capture on from the next forward (or off, freeing its buffers)."""
        L.check(L.lib().tz_arctic_debug_capture(self.handle, int(bool(on))))

    # K and N of layer 0's GEMMs: 0 QKV, 1 attention output, 2 FFN1, 3 FFN2
    GEMM_K = (384, 384, 384, 1536)
    GEMM_N = (1152, 384, 1536, 384)

    def debug_operand(self, which: int, total_tokens: int):
        """W8A8: layer 0's int8 A operand [T, K] and per-token scales [T] of GEMM `which`, as the
        forward's own kernel consumed them (for 1 and 3: quantised inside the gemm_ln mainloop)."""
        q = np.empty((total_tokens, self.GEMM_K[which]), np.int8)
        s = np.empty(total_tokens, np.float32)
        L.check(L.lib().tz_arctic_debug_operand(self.handle, which, q.ctypes.data, s.ctypes.data, total_tokens))
        return q, s

    def debug_accum(self, which: int, total_tokens: int) -> np.ndarray:
        """W8A8: the raw int32 accumulators [T, N] of layer 0's GEMM `which`, read by its epilogue."""
        acc = np.empty((total_tokens, self.GEMM_N[which]), np.int32)
        L.check(L.lib().tz_arctic_debug_accum(self.handle, which, acc.ctypes.data, total_tokens))
        return acc

    def debug_gemm_input(self, which: int, total_tokens: int) -> np.ndarray:
        """W8A8, which = 1 or 3: the f16 activation [T, K] that gemm_ln quantised per token (as f32)."""
        x = np.empty((total_tokens, self.GEMM_K[which]), np.uint16)
        L.check(L.lib().tz_arctic_debug_gemm_input(self.handle, which, x.ctypes.data, total_tokens))
        return x.view(np.float16).astype(np.float32)
