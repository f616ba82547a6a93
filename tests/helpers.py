"""Shared builders for the parity tests: the reference's self-contained synthetic
models (tests/gqa.rs, tests/forward_gpu.rs) and the benchmark shapes."""
from __future__ import annotations

import numpy as np

from talos_b200 import gguf, synth


def _base_meta(w: gguf.GgufWriter, *, ctx, embd, n_layer, ff, n_head, n_head_kv, vocab, hd):
    """tests/gqa.rs:110-129"""
    w.add_str("general.architecture", "llama")
    w.add_u32("llama.context_length", ctx)
    w.add_u32("llama.embedding_length", embd)
    w.add_u32("llama.block_count", n_layer)
    w.add_u32("llama.feed_forward_length", ff)
    w.add_u32("llama.attention.head_count", n_head)
    w.add_u32("llama.attention.head_count_kv", n_head_kv)
    w.add_f32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_u32("llama.rope.dimension_count", hd)
    w.add_f32("llama.rope.freq_base", 10000.0)
    w.add_arr_str("tokenizer.ggml.tokens", ["<unk>" if i == 0 else f"t{i}" for i in range(vocab)])
    w.add_arr_str("tokenizer.ggml.merges", [])
    w.add_u32("tokenizer.ggml.unknown_token_id", 0)
    w.add_u32("tokenizer.ggml.bos_token_id", 0)
    w.add_u32("tokenizer.ggml.eos_token_id", 0)


# tests/gqa.rs:12-22
EMBD, N_HEAD, N_HEAD_KV, FF, VOCAB, N_LAYER, CTX = 16, 4, 2, 32, 16, 2, 32
HD = EMBD // N_HEAD
GROUP = N_HEAD // N_HEAD_KV


def gqa_pair(seed: int = 7) -> tuple[bytes, bytes]:
    """The GQA model and its replicated-MHA twin of tests/gqa.rs:131-227, with
    U(-0.5, 0.5) weights from numpy's PCG64 (the Rust StdRng stream cannot be
    reproduced without Rust; the property does not depend on it)."""
    rng = np.random.default_rng(seed)

    def rv(n):
        return rng.uniform(-0.5, 0.5, n).astype(np.float32)

    embd, out_norm, out = rv(VOCAB * EMBD), rv(EMBD), rv(VOCAB * EMBD)
    layers = [dict(attn_norm=rv(EMBD), q=rv(EMBD * EMBD), k_full=rv(EMBD * EMBD), v_full=rv(EMBD * EMBD),
                   attn_output=rv(EMBD * EMBD), ffn_norm=rv(EMBD), ffn_gate=rv(FF * EMBD),
                   ffn_up=rv(FF * EMBD), ffn_down=rv(EMBD * FF)) for _ in range(N_LAYER)]

    def head_rows(full, h):
        return full[h * HD * EMBD:(h + 1) * HD * EMBD]

    def build(gqa: bool) -> bytes:
        w = gguf.GgufWriter()
        _base_meta(w, ctx=CTX, embd=EMBD, n_layer=N_LAYER, ff=FF, n_head=N_HEAD,
                   n_head_kv=N_HEAD_KV if gqa else N_HEAD, vocab=VOCAB, hd=HD)
        w.add_tensor("token_embd.weight", [EMBD, VOCAB], gguf.F32, embd.tobytes())
        w.add_tensor("output_norm.weight", [EMBD], gguf.F32, out_norm.tobytes())
        w.add_tensor("output.weight", [EMBD, VOCAB], gguf.F32, out.tobytes())
        for l, ly in enumerate(layers):
            kv_rows = N_HEAD_KV if gqa else N_HEAD
            ks, vs = [], []
            for r in range(kv_rows):
                leader = r * GROUP if gqa else (r // GROUP) * GROUP
                ks.append(head_rows(ly["k_full"], leader))
                vs.append(head_rows(ly["v_full"], leader))
            kv_dim = kv_rows * HD
            p = f"blk.{l}."
            w.add_tensor(p + "attn_norm.weight", [EMBD], gguf.F32, ly["attn_norm"].tobytes())
            w.add_tensor(p + "attn_q.weight", [EMBD, EMBD], gguf.F32, ly["q"].tobytes())
            w.add_tensor(p + "attn_k.weight", [EMBD, kv_dim], gguf.F32, np.concatenate(ks).tobytes())
            w.add_tensor(p + "attn_v.weight", [EMBD, kv_dim], gguf.F32, np.concatenate(vs).tobytes())
            w.add_tensor(p + "attn_output.weight", [EMBD, EMBD], gguf.F32, ly["attn_output"].tobytes())
            w.add_tensor(p + "ffn_norm.weight", [EMBD], gguf.F32, ly["ffn_norm"].tobytes())
            w.add_tensor(p + "ffn_gate.weight", [EMBD, FF], gguf.F32, ly["ffn_gate"].tobytes())
            w.add_tensor(p + "ffn_up.weight", [EMBD, FF], gguf.F32, ly["ffn_up"].tobytes())
            w.add_tensor(p + "ffn_down.weight", [FF, EMBD], gguf.F32, ly["ffn_down"].tobytes())
        return w.to_bytes()

    return build(True), build(False)


def forward_gpu_model(seed: int = 0) -> bytes:
    """tests/forward_gpu.rs:61-144: c 16, 4/2 heads, ff 32, vocab 16, 2 layers, ctx 8,
    U(-0.5, 0.5) F32 weights."""
    c, nh, nkv, ff, vocab, n_layer, ctx = 16, 4, 2, 32, 16, 2, 8
    kv = nkv * (c // nh)
    rng = np.random.default_rng(seed)

    def rv(n):
        return rng.uniform(-0.5, 0.5, n).astype(np.float32).tobytes()

    w = gguf.GgufWriter()
    _base_meta(w, ctx=ctx, embd=c, n_layer=n_layer, ff=ff, n_head=nh, n_head_kv=nkv, vocab=vocab, hd=c // nh)
    w.add_tensor("token_embd.weight", [c, vocab], gguf.F32, rv(vocab * c))
    w.add_tensor("output_norm.weight", [c], gguf.F32, rv(c))
    w.add_tensor("output.weight", [c, vocab], gguf.F32, rv(vocab * c))
    for l in range(n_layer):
        p = f"blk.{l}."
        w.add_tensor(p + "attn_norm.weight", [c], gguf.F32, rv(c))
        w.add_tensor(p + "attn_q.weight", [c, c], gguf.F32, rv(c * c))
        w.add_tensor(p + "attn_k.weight", [c, kv], gguf.F32, rv(kv * c))
        w.add_tensor(p + "attn_v.weight", [c, kv], gguf.F32, rv(kv * c))
        w.add_tensor(p + "attn_output.weight", [c, c], gguf.F32, rv(c * c))
        w.add_tensor(p + "ffn_norm.weight", [c], gguf.F32, rv(c))
        w.add_tensor(p + "ffn_gate.weight", [c, ff], gguf.F32, rv(ff * c))
        w.add_tensor(p + "ffn_up.weight", [c, ff], gguf.F32, rv(ff * c))
        w.add_tensor(p + "ffn_down.weight", [ff, c], gguf.F32, rv(c * ff))
    return w.to_bytes()


def tiny_model(wtype: int) -> bytes:
    """The tiny Llama benchmark model: N(0, 0.02) seed 42; every 2-D weight in wtype."""
    return synth.llama_bytes(synth.TINY, 42, wtype=wtype)


def prompt(n: int, vocab: int, seed: int) -> list[int]:
    """Seeded uniform-random prompt ids in [0, vocab)."""
    return synth.token_ids(seed, n, vocab)
