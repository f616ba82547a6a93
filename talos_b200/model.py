"""Host-side mirror of Talos's ``Model`` for the CUDA decode path.

Same names and argument meaning as the Rust API (Tsuskov/talos
``src/model/llama.rs:20-238``): ``Model.load`` / ``load_bytes``, ``forward_gpu`` /
``forward_hidden_gpu`` (the ``cuda`` twins of the Metal functions), ``step`` /
``step_hidden`` (the dispatch point of ``llama.rs:211-233``; with the CUDA build it
always takes the GPU path), ``reset`` and ``cap_context``. Weights are read from
the GGUF with the same names and shapes as ``Weights::from_gguf``
(``src/model/weights.rs:91-114``) and handed to the C ABI, which copies them to the
GPU once. There is no CPU forward here: the reference CPU ``forward`` is the
oracle used by the tests, not part of this package.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .gguf import F32, GgufError, GgufFile


@dataclass
class Config:
    """``Config`` (src/model/config.rs:14-67)."""

    n_layer: int
    n_head: int
    n_head_kv: int
    n_embd: int
    n_ff: int
    context_length: int
    vocab_size: int
    rms_eps: float
    rope_dim: int
    rope_freq_base: float

    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def kv_dim(self) -> int:
        return self.n_head_kv * self.head_dim()

    @classmethod
    def from_gguf(cls, g: GgufFile) -> "Config":
        """config.rs:40-67: llama.* keys, vocab = len(tokenizer.ggml.tokens),
        eps defaults to 1e-5, freq_base to 10000."""
        arch = g.get_str("general.architecture") or ""
        if arch != "llama":
            raise GgufError(f"unsupported architecture {arch!r} (expected \"llama\")")

        def u(k):
            v = g.get_u32(k)
            if v is None:
                raise GgufError(f"missing metadata key {k}")
            return v

        toks = g.get_arr_str("tokenizer.ggml.tokens")
        if toks is None:
            raise GgufError("missing tokenizer.ggml.tokens (needed for vocab size)")
        eps = g.get_f32("llama.attention.layer_norm_rms_epsilon")
        base = g.get_f32("llama.rope.freq_base")
        return cls(
            n_layer=u("llama.block_count"),
            n_head=u("llama.attention.head_count"),
            n_head_kv=u("llama.attention.head_count_kv"),
            n_embd=u("llama.embedding_length"),
            n_ff=u("llama.feed_forward_length"),
            context_length=u("llama.context_length"),
            vocab_size=len(toks),
            rms_eps=1e-5 if eps is None else eps,
            rope_dim=u("llama.rope.dimension_count"),
            rope_freq_base=10000.0 if base is None else base,
        )

    def to_c(self) -> _lib.Cfg:
        return _lib.Cfg(self.n_layer, self.n_head, self.n_head_kv, self.n_embd, self.n_ff,
                        self.context_length, self.vocab_size, self.rope_dim, self.rms_eps,
                        self.rope_freq_base)


def weight_shapes(cfg: Config) -> dict[str, tuple[int, int]]:
    """Tensor name -> (rows, cols) exactly as Weights::from_gguf binds them
    (src/model/weights.rs:91-114); norms are (1, n)."""
    c, ff, v, kv = cfg.n_embd, cfg.n_ff, cfg.vocab_size, cfg.kv_dim()
    out = {"token_embd.weight": (v, c), "output_norm.weight": (1, c), "output.weight": (v, c)}
    for l in range(cfg.n_layer):
        p = f"blk.{l}."
        out.update({
            p + "attn_norm.weight": (1, c),
            p + "attn_q.weight": (c, c),
            p + "attn_k.weight": (kv, c),
            p + "attn_v.weight": (kv, c),
            p + "attn_output.weight": (c, c),
            p + "ffn_norm.weight": (1, c),
            p + "ffn_gate.weight": (ff, c),
            p + "ffn_up.weight": (ff, c),
            p + "ffn_down.weight": (c, ff),
        })
    return out


def _ptr(a) -> int:
    return a.ctypes.data if isinstance(a, np.ndarray) else C.addressof(a)


def nccl_unique_id() -> bytes:
    """talos_nccl_unique_id: the 128-byte id rank 0 makes and shares with the other
    tensor-parallel ranks (out of band) before they create their contexts."""
    buf = C.create_string_buffer(128)
    _lib.check(_lib.load().talos_nccl_unique_id(buf))
    return buf.raw


class Context:
    """One ``talos_ctx``: a model's weights, KV cache and captured graphs on one GPU."""

    def __init__(self, cfg: Config, device: int = 0, tp_size: int = 1, tp_rank: int = 0,
                 nccl_id: bytes | None = None):
        L = _lib.load()
        self.cfg = cfg
        h = C.c_void_p()
        c = cfg.to_c()
        if tp_size == 1:
            _lib.check(L.talos_ctx_create(C.byref(c), device, C.byref(h)))
        else:
            idbuf = C.create_string_buffer(bytes(nccl_id), 128)
            _lib.check(L.talos_ctx_create_tp(C.byref(c), device, tp_size, tp_rank, idbuf, C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            _lib.load().talos_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload(self, name: str, raw, gtype: int, rows: int, cols: int):
        buf = np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8)
        buf = np.ascontiguousarray(buf)
        _lib.check(_lib.load().talos_weight_upload(self.h, name.encode(), _ptr(buf), buf.nbytes, gtype,
                                                   rows, cols))

    def set_step_kernel(self, kind: str):
        """"auto", "fused" (one per-token kernel) or "layered" (~5 kernels per layer)."""
        k = {"auto": _lib.STEP_AUTO, "fused": _lib.STEP_FUSED, "layered": _lib.STEP_LAYERED}[kind]
        _lib.check(_lib.load().talos_ctx_set_step_kernel(self.h, k))

    def step_kernel(self) -> str:
        """What the next step runs: "fused" or "layered"."""
        k = C.c_int()
        _lib.check(_lib.load().talos_ctx_step_kernel(self.h, C.byref(k)))
        return "fused" if k.value == _lib.STEP_FUSED else "layered"

    def set_kv_dtype(self, dtype: str):
        """"f32" (the reference's cache) or "f16" (opt-in: half the cache bytes;
        K/V rounded to f16 when appended). Empties the cache."""
        k = {"f32": _lib.KV_F32, "f16": _lib.KV_F16}[dtype]
        _lib.check(_lib.load().talos_ctx_set_kv_dtype(self.h, k))

    def kv_dtype(self) -> str:
        k = C.c_int()
        _lib.check(_lib.load().talos_ctx_kv_dtype(self.h, C.byref(k)))
        return "f16" if k.value == _lib.KV_F16 else "f32"

    def set_batch(self, max_seqs: int):
        """Reserve KV cache slots for up to ``max_seqs`` (<= TALOS_MAX_BATCH, 64)
        sequences decoded together by ``forward_batch`` (0 frees them). Under
        tensor parallelism every rank calls it with the same value."""
        _lib.check(_lib.load().talos_ctx_set_batch(self.h, int(max_seqs)))

    def forward_batch(self, tokens, positions) -> np.ndarray:
        """One step for sequences 0 .. n-1 (token i at positions[i] into cache slot
        i); returns [n, vocab_size] logits."""
        t = np.ascontiguousarray(tokens, np.uint32)
        p = np.ascontiguousarray(positions, np.uint64)
        n = len(t)
        if len(p) != n:
            raise ValueError("tokens and positions differ in length")
        out = np.empty((n, self.cfg.vocab_size), np.float32)
        _lib.check(_lib.load().talos_forward_batch(self.h, t.ctypes.data_as(C.POINTER(C.c_uint32)),
                                                   p.ctypes.data_as(C.POINTER(C.c_size_t)), n,
                                                   out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def prefill_slot(self, slot: int, tokens, pos0: int = 0, want_logits: bool = True):
        """talos_prefill_slot: sequence ``slot``'s prompt at pos0.. into its cache
        slot; the logits after the last token (or None)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        _lib.check(_lib.load().talos_prefill_slot(self.h, int(slot), t.ctypes.data_as(C.POINTER(C.c_uint32)),
                                                  t.size, int(pos0),
                                                  out.ctypes.data_as(C.POINTER(C.c_float)) if out is not None
                                                  else None))
        return out

    def generate_batch_greedy(self, tokens, positions, steps: int) -> np.ndarray:
        """talos_generate_batch_greedy: sequences 0 .. n-1 from (tokens[i],
        positions[i]); returns the chosen tokens as [steps, n]."""
        t = np.ascontiguousarray(tokens, np.uint32)
        p = np.ascontiguousarray(positions, np.uint64)
        n = len(t)
        if len(p) != n:
            raise ValueError("tokens and positions differ in length")
        out = np.empty((max(int(steps), 1), n), np.uint32)
        _lib.check(_lib.load().talos_generate_batch_greedy(self.h, t.ctypes.data_as(C.POINTER(C.c_uint32)),
                                                           p.ctypes.data_as(C.POINTER(C.c_size_t)), n, int(steps),
                                                           out.ctypes.data_as(C.POINTER(C.c_uint32))))
        return out[: int(steps)]

    def device_bytes(self) -> int:
        n = C.c_size_t()
        _lib.check(_lib.load().talos_ctx_device_bytes(self.h, C.byref(n)))
        return n.value

    def stream(self) -> int:
        """The cudaStream_t this context runs on (for CUDA-event timing)."""
        p = C.c_void_p()
        _lib.check(_lib.load().talos_ctx_stream(self.h, C.byref(p)))
        return p.value or 0

    def forward(self, token: int, pos: int, out: np.ndarray | None = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.cfg.vocab_size, np.float32)
        _lib.check(_lib.load().talos_forward(self.h, int(token), int(pos), _ptr(out)))
        return out

    def forward_hidden(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.cfg.n_embd, np.float32)
        _lib.check(_lib.load().talos_forward_hidden(self.h, int(token), int(pos), _ptr(out)))
        return out

    def generate_greedy(self, token: int, pos: int, n: int) -> np.ndarray:
        out = np.empty(max(n, 1), np.uint32)
        _lib.check(_lib.load().talos_generate_greedy(self.h, int(token), int(pos), int(n), _ptr(out)))
        return out[:n]

    def prefill(self, tokens, pos0: int = 0, want_logits: bool = True):
        toks = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        _lib.check(_lib.load().talos_prefill(self.h, _ptr(toks), toks.size, int(pos0),
                                             _ptr(out) if out is not None else None))
        return out

    def reset(self):
        _lib.check(_lib.load().talos_kv_reset(self.h))

    def tp_resync(self):
        """talos_ctx_tp_resync: after any rank's step failed, every rank calls this
        while no rank has a step in flight; the next step starts afresh."""
        _lib.check(_lib.load().talos_ctx_tp_resync(self.h))

    def perplexity(self, tokens) -> tuple[float, float, int]:
        """talos_perplexity: (perplexity, NLL sum, scored positions)."""
        toks = np.ascontiguousarray(tokens, np.uint32)
        ppl, nll, n = C.c_float(), C.c_double(), C.c_size_t()
        _lib.check(_lib.load().talos_perplexity(self.h, _ptr(toks), toks.size, C.byref(ppl), C.byref(nll),
                                                C.byref(n)))
        return ppl.value, nll.value, n.value

    KERNEL_KINDS = ("embed", "qkv", "attn", "oproj", "gateup", "down", "output")

    def profile_step(self, token: int, pos: int) -> tuple[dict, dict]:
        """Per-kernel-kind device ms and counts of one step: kernels launched one by
        one (layered), or the per-token kernel's phases timed on the device clock
        (fused)."""
        ms = (C.c_double * 7)()
        n = (C.c_uint32 * 7)()
        _lib.check(_lib.load().talos_profile_step(self.h, int(token), int(pos), ms, n))
        return ({k: ms[i] for i, k in enumerate(self.KERNEL_KINDS)},
                {k: int(n[i]) for i, k in enumerate(self.KERNEL_KINDS)})

    def profile_phases(self, token: int, pos: int) -> np.ndarray:
        """Per-token kernel stamps of one step: uint64 ns [phase][cta][4] = entered,
        staged, computed, arrived (0 where a stamp does not apply)."""
        cap = (self.cfg.n_layer * 5 + 1) * 256 * 4
        out = np.zeros(cap, np.uint64)
        nph, ncta = C.c_int(), C.c_int()
        _lib.check(_lib.load().talos_profile_phases(self.h, int(token), int(pos), _ptr(out), cap, C.byref(nph),
                                                    C.byref(ncta)))
        return out[: nph.value * ncta.value * 4].reshape(nph.value, ncta.value, 4)

    def cap_context(self, max_ctx: int):
        _lib.check(_lib.load().talos_cap_context(self.h, int(max_ctx)))
        self.cfg.context_length = min(self.cfg.context_length, max(int(max_ctx), 1))

    def matvec_resident(self, name: str, raw, gtype: int, x, rows: int, cols: int) -> np.ndarray:
        buf = np.ascontiguousarray(np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8))
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        _lib.check(_lib.load().talos_matvec_resident(self.h, name.encode(), gtype, _ptr(buf), buf.nbytes,
                                                     rows, cols, _ptr(x), _ptr(y)))
        return y


class Model:
    """``Model`` (src/model/llama.rs:20-238) with the CUDA backend."""

    def __init__(self, gguf: GgufFile, device: int = 0, tp_size: int = 1, tp_rank: int = 0,
                 nccl_id: bytes | None = None, max_ctx: int | None = None, step_kernel: str = "auto",
                 kv_dtype: str = "f32"):
        cfg = Config.from_gguf(gguf)
        if cfg.n_head_kv == 0 or cfg.n_head % cfg.n_head_kv != 0:
            raise GgufError(f"head_count {cfg.n_head} must be a positive multiple of head_count_kv "
                            f"{cfg.n_head_kv}")
        if max_ctx is not None:
            cfg.context_length = min(cfg.context_length, max(int(max_ctx), 1))
        self.cfg = cfg
        self.gguf = gguf
        self.ctx = Context(cfg, device, tp_size, tp_rank, nccl_id)
        if step_kernel != "auto":
            self.ctx.set_step_kernel(step_kernel)
        if kv_dtype != "f32":
            self.ctx.set_kv_dtype(kv_dtype)
        for name, (rows, cols) in weight_shapes(cfg).items():
            if rows == 1:
                data = gguf.tensor_f32(name)
                self.ctx.upload(name, data, F32, 1, cols)
            else:
                raw, gtype = gguf.tensor_raw(name)
                self.ctx.upload(name, raw, gtype, rows, cols)

    @classmethod
    def load(cls, path: str, **kw) -> "Model":
        return cls(GgufFile.open(path), **kw)

    @classmethod
    def load_bytes(cls, data: bytes, **kw) -> "Model":
        return cls(GgufFile.from_bytes(data), **kw)

    def close(self):
        self.ctx.close()

    def cap_context(self, max_ctx: int):
        """llama.rs:69-81"""
        self.ctx.cap_context(max_ctx)
        self.cfg.context_length = self.ctx.cfg.context_length

    def forward_gpu(self, token: int, pos: int) -> np.ndarray:
        """llama.rs:188-195"""
        return self.ctx.forward(token, pos)

    def forward_hidden_gpu(self, token: int, pos: int) -> np.ndarray:
        """llama.rs:199-206"""
        return self.ctx.forward_hidden(token, pos)

    def step(self, token: int, pos: int) -> np.ndarray:
        """llama.rs:211-220 (CUDA build: always the GPU forward)."""
        return self.forward_gpu(token, pos)

    def step_hidden(self, token: int, pos: int) -> np.ndarray:
        """llama.rs:224-233"""
        return self.forward_hidden_gpu(token, pos)

    def reset(self):
        """llama.rs:236-238"""
        self.ctx.reset()

    def generate_greedy(self, token: int, pos: int, n: int) -> np.ndarray:
        return self.ctx.generate_greedy(token, pos, n)

    def perplexity(self, tokens) -> float:
        """eval::perplexity (src/eval.rs:35-52) on the GPU."""
        return self.ctx.perplexity(tokens)[0]

    def prefill(self, tokens, pos0: int = 0):
        """src/main.rs:88-95 in one call: the logits after the last prompt token."""
        return self.ctx.prefill(tokens, pos0)

    def set_batch(self, max_seqs: int):
        """Cache slots for up to 64 sequences decoded together (0 frees them)."""
        self.ctx.set_batch(max_seqs)

    def prefill_slot(self, slot: int, tokens, pos0: int = 0):
        """Sequence ``slot``'s prompt into its cache slot; the logits after its last token."""
        return self.ctx.prefill_slot(slot, tokens, pos0)

    def generate_batch_greedy(self, tokens, positions, steps: int) -> np.ndarray:
        """Greedy tokens of sequences 0 .. n-1 decoded together on the GPU: [steps, n]."""
        return self.ctx.generate_batch_greedy(tokens, positions, steps)

    def forward_batch(self, tokens, positions) -> np.ndarray:
        """One step for sequences 0 .. n-1: token i at positions[i] in slot i;
        [n, vocab_size] logits (each row what forward_gpu gives that sequence alone)."""
        return self.ctx.forward_batch(tokens, positions)


# ----------------------------------------------------------------- kernel entry points

def dequant(gtype: int, raw, n_elems: int) -> np.ndarray:
    """talos_dequant: GgmlType::dequantize on the GPU (bit-exact)."""
    buf = np.ascontiguousarray(np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8))
    out = np.empty(n_elems, np.float32)
    _lib.check(_lib.load().talos_dequant(gtype, _ptr(buf), n_elems, _ptr(out)))
    return out


def argmax(logits) -> int:
    """talos_argmax: sample::argmax (src/sample.rs:7-14) on the GPU, total order,
    last maximal index on ties."""
    v = np.ascontiguousarray(logits, np.float32)
    out = C.c_uint32()
    _lib.check(_lib.load().talos_argmax(_ptr(v), v.size, C.byref(out)))
    return int(out.value)


def matvec(gtype: int, raw, x, rows: int, cols: int, device: int = 0) -> np.ndarray:
    """talos_matvec: one fused dequant-matvec (math::metal::matvec_quant twin)."""
    buf = np.ascontiguousarray(np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8))
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(rows, np.float32)
    _lib.check(_lib.load().talos_matvec(device, gtype, _ptr(buf), buf.nbytes, rows, cols, _ptr(x), _ptr(y)))
    return y


class Weight:
    """A packed weight on one device, for device-pointer matvecs (benchmarks)."""

    def __init__(self, gtype: int, raw, rows: int, cols: int, device: int = 0):
        buf = np.ascontiguousarray(np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8))
        h = C.c_void_p()
        _lib.check(_lib.load().talos_weight_create(device, gtype, _ptr(buf), buf.nbytes, rows, cols, C.byref(h)))
        self.h = h
        self.rows, self.cols, self.gtype = rows, cols, gtype

    def packed_bytes(self) -> int:
        n = C.c_size_t()
        _lib.check(_lib.load().talos_weight_packed_bytes(self.h, C.byref(n)))
        return n.value

    def matvec_dev(self, x_ptr: int, y_ptr: int, stream: int = 0):
        _lib.check(_lib.load().talos_matvec_dev(self.h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), C.c_void_p(stream)))

    def matvec_dev_noalloc(self, x_ptr: int, y_ptr: int, stream: int = 0):
        """talos_matvec_dev_noalloc: the split-K variant that allocates nothing
        (static scratch; calls in flight at once race)."""
        _lib.check(_lib.load().talos_matvec_dev_noalloc(self.h, C.c_void_p(x_ptr), C.c_void_p(y_ptr),
                                                        C.c_void_p(stream)))

    def close(self):
        if getattr(self, "h", None):
            _lib.load().talos_weight_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
