"""Seeded synthetic Llama models as GGUF v3 (stand-in for the Hephaistos exporter).

Shapes are the benchmark configurations of the Talos decode path; weights are
N(0, sigma) from the counter-based generator in synth.c (so a tensor's bytes
depend only on the seed and its name), quantized with the reference's own test
quantizers. Norm weights are 1.0. Metadata follows the reference's synthetic
GGUF writers (tests/gqa.rs:110-129): llama.* keys, a token list of vocab
strings, empty merges, unk/bos/eos ids.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, replace

import numpy as np

from ..build import SYNTH_LIB, build_synth
from ..gguf import BLOCK_BYTES, BLOCK_ELEMS, F32, Q4_0, Q6_K, Q8_0, GgufWriter

_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(SYNTH_LIB):
            build_synth()
        L = C.CDLL(SYNTH_LIB)
        L.synth_stream_of.restype = C.c_uint64
        L.synth_stream_of.argtypes = [C.c_char_p]
        L.synth_fill_normal.restype = None
        L.synth_fill_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_void_p]
        L.synth_quantize.restype = C.c_int
        L.synth_quantize.argtypes = [C.c_int, C.c_void_p, C.c_uint64, C.c_void_p]
        L.synth_tensor.restype = C.c_int
        L.synth_tensor.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int, C.c_float,
                                   C.c_void_p, C.c_int]
        L.synth_token_ids.restype = None
        L.synth_token_ids.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32, C.c_void_p]
        _lib = L
    return _lib


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def normal(seed: int, name: str, n: int, sigma: float = 1.0, start: int = 0) -> np.ndarray:
    L = _load()
    out = np.empty(n, np.float32)
    L.synth_fill_normal(seed, L.synth_stream_of(name.encode()), start, n, sigma, out.ctypes.data)
    return out


def token_ids(seed: int, n: int, vocab: int, name: str = "prompt") -> list[int]:
    """A seeded uniform-random prompt of n ids in [0, vocab)."""
    L = _load()
    out = np.empty(max(n, 1), np.uint32)
    L.synth_token_ids(seed, L.synth_stream_of(name.encode()), n, vocab, out.ctypes.data)
    return [int(v) for v in out[:n]]


def quantize(gtype: int, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.size // BLOCK_ELEMS[gtype] * BLOCK_BYTES[gtype], np.uint8)
    if _load().synth_quantize(gtype, x.ctypes.data, x.size, out.ctypes.data):
        raise ValueError("size is not a multiple of the block")
    return out


def tensor(seed: int, name: str, rows: int, cols: int, gtype: int, sigma: float = 0.02,
           threads: int | None = None) -> np.ndarray:
    """Raw GGUF bytes of a [rows, cols] N(0, sigma) tensor of `gtype`."""
    L = _load()
    out = np.empty(rows * (cols // BLOCK_ELEMS[gtype]) * BLOCK_BYTES[gtype], np.uint8)
    rc = L.synth_tensor(seed, L.synth_stream_of(name.encode()), rows, cols, gtype, sigma, out.ctypes.data,
                        threads or default_threads())
    if rc:
        raise ValueError(f"{name}: cols {cols} not a multiple of the block of type {gtype}")
    return out


@dataclass
class Shape:
    n_embd: int
    n_layer: int
    n_head: int
    n_head_kv: int
    n_ff: int
    vocab: int
    ctx: int
    rope_base: float = 10000.0
    eps: float = 1e-5

    @property
    def head_dim(self):
        return self.n_embd // self.n_head

    @property
    def kv_dim(self):
        return self.n_head_kv * self.head_dim


# Benchmark model shapes (dtypes are chosen per model): the tiny Llama, the
# Mistral-7B shape and the Llama-3-70B shape.
TINY = Shape(n_embd=288, n_layer=6, n_head=6, n_head_kv=2, n_ff=768, vocab=4096, ctx=256)
MISTRAL_7B = Shape(n_embd=4096, n_layer=32, n_head=32, n_head_kv=8, n_ff=14336, vocab=32000, ctx=4096,
                   rope_base=1e6)
LLAMA3_70B = Shape(n_embd=8192, n_layer=80, n_head=64, n_head_kv=8, n_ff=28672, vocab=128256, ctx=8192,
                   rope_base=5e5)


def llama_gguf(shape: Shape, seed: int, wtype: int = F32, out_type: int | None = None,
               embd_type: int | None = None, sigma: float = 0.02, norm_value: float = 1.0,
               threads: int | None = None) -> GgufWriter:
    """A GgufWriter for a synthetic Llama; tensors are generated as they are written."""
    out_type = wtype if out_type is None else out_type
    embd_type = wtype if embd_type is None else embd_type
    g = GgufWriter()
    g.add_str("general.architecture", "llama")
    g.add_u32("llama.context_length", shape.ctx)
    g.add_u32("llama.embedding_length", shape.n_embd)
    g.add_u32("llama.block_count", shape.n_layer)
    g.add_u32("llama.feed_forward_length", shape.n_ff)
    g.add_u32("llama.attention.head_count", shape.n_head)
    g.add_u32("llama.attention.head_count_kv", shape.n_head_kv)
    g.add_f32("llama.attention.layer_norm_rms_epsilon", shape.eps)
    g.add_u32("llama.rope.dimension_count", shape.head_dim)
    g.add_f32("llama.rope.freq_base", shape.rope_base)
    g.add_arr_str("tokenizer.ggml.tokens", ["<unk>" if i == 0 else f"t{i}" for i in range(shape.vocab)])
    g.add_arr_str("tokenizer.ggml.merges", [])
    g.add_u32("tokenizer.ggml.unknown_token_id", 0)
    g.add_u32("tokenizer.ggml.bos_token_id", 0)
    g.add_u32("tokenizer.ggml.eos_token_id", 0)
    E, F, V, KV = shape.n_embd, shape.n_ff, shape.vocab, shape.kv_dim

    def mat(name, rows, cols, t):
        g.add_tensor(name, [cols, rows], t, lambda: tensor(seed, name, rows, cols, t, sigma, threads))

    def norm(name):
        g.add_tensor(name, [E], F32, np.full(E, norm_value, np.float32).tobytes())

    mat("token_embd.weight", V, E, embd_type)
    norm("output_norm.weight")
    mat("output.weight", V, E, out_type)
    for l in range(shape.n_layer):
        p = f"blk.{l}."
        norm(p + "attn_norm.weight")
        mat(p + "attn_q.weight", E, E, wtype)
        mat(p + "attn_k.weight", KV, E, wtype)
        mat(p + "attn_v.weight", KV, E, wtype)
        mat(p + "attn_output.weight", E, E, wtype)
        norm(p + "ffn_norm.weight")
        mat(p + "ffn_gate.weight", F, E, wtype)
        mat(p + "ffn_up.weight", F, E, wtype)
        mat(p + "ffn_down.weight", E, F, wtype)
    return g


def write_llama(path: str, shape: Shape, seed: int, **kw) -> str:
    llama_gguf(shape, seed, **kw).write(path)
    return path


def llama_bytes(shape: Shape, seed: int, **kw) -> bytes:
    return llama_gguf(shape, seed, **kw).to_bytes()


def with_ctx(shape: Shape, ctx: int) -> Shape:
    return replace(shape, ctx=ctx)


__all__ = ["Shape", "TINY", "MISTRAL_7B", "LLAMA3_70B", "F32", "Q4_0", "Q8_0", "Q6_K", "llama_gguf",
           "write_llama", "llama_bytes", "tensor", "normal", "quantize", "with_ctx", "token_ids"]
