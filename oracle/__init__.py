"""ctypes bindings for the CPU oracle (oracle/talos_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and by
the cpu_baseline / ``--impl reference`` legs of bench.py, never by the product
package ``talos_b200``. It restates the Rust CPU path of Tsuskov/talos
(``src/model/llama.rs:96-183`` and the kernels it calls); each C function cites the
file:line it follows.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libtalos_oracle.so")

F32, Q4_0, Q8_0, Q6_K = 0, 2, 8, 14
BLOCK_ELEMS = {F32: 1, Q4_0: 32, Q8_0: 32, Q6_K: 256}
BLOCK_BYTES = {F32: 4, Q4_0: 18, Q8_0: 34, Q6_K: 210}

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    if force or not os.path.exists(LIB_PATH) or _stale():
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _stale() -> bool:
    t = os.path.getmtime(LIB_PATH)
    return any(
        os.path.getmtime(os.path.join(HERE, f)) > t
        for f in ("talos_oracle.c", "talos_oracle.h", "Makefile")
        if os.path.exists(os.path.join(HERE, f))
    )


class Config(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "n_layer", "n_head", "n_head_kv", "n_embd", "n_ff", "context_length", "vocab_size",
        "rope_dim")] + [("rms_eps", C.c_float), ("rope_freq_base", C.c_float)]


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = C.CDLL(LIB_PATH)
    vp, sz, fp = C.c_void_p, C.c_size_t, C.POINTER(C.c_float)
    sig = {
        "oracle_last_error": (C.c_char_p, []),
        "oracle_set_threads": (None, [C.c_int]),
        "oracle_get_threads": (C.c_int, []),
        "oracle_f16_to_f32": (C.c_float, [C.c_uint16]),
        "oracle_f32_to_f16": (C.c_uint16, [C.c_float]),
        "oracle_dequant": (C.c_int, [C.c_int, vp, sz, vp]),
        "oracle_dot": (C.c_float, [vp, vp, sz]),
        "oracle_matvec_f32": (None, [vp, vp, vp, sz, sz]),
        "oracle_matvec_quant": (C.c_int, [vp, C.c_int, vp, vp, sz, sz]),
        "oracle_rmsnorm": (None, [vp, vp, C.c_float, vp, sz]),
        "oracle_softmax": (None, [vp, sz]),
        "oracle_silu": (C.c_float, [C.c_float]),
        "oracle_swiglu": (None, [vp, vp, vp, sz]),
        "oracle_rope": (None, [vp, sz, sz, sz, C.c_float]),
        "oracle_argmax": (C.c_uint32, [vp, sz]),
        "oracle_quantize_q8_0": (None, [vp, sz, vp]),
        "oracle_quantize_q4_0": (None, [vp, sz, vp]),
        "oracle_quantize_q6_k": (None, [vp, sz, vp]),
        "oracle_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(vp)]),
        "oracle_gguf_from_bytes": (C.c_int, [vp, sz, C.POINTER(vp)]),
        "oracle_gguf_free": (None, [vp]),
        "oracle_gguf_get_u32": (C.c_int, [vp, C.c_char_p, C.POINTER(C.c_uint32)]),
        "oracle_gguf_get_f32": (C.c_int, [vp, C.c_char_p, fp]),
        "oracle_gguf_get_bool": (C.c_int, [vp, C.c_char_p, C.POINTER(C.c_int)]),
        "oracle_gguf_get_str": (C.c_int, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "oracle_gguf_arr_str_len": (C.c_int, [vp, C.c_char_p, C.POINTER(sz)]),
        "oracle_gguf_arr_str_item": (C.c_int, [vp, C.c_char_p, sz, C.POINTER(vp), C.POINTER(sz)]),
        "oracle_gguf_arr_i32": (C.c_int, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "oracle_gguf_n_tensors": (sz, [vp]),
        "oracle_gguf_tensor_name": (C.c_char_p, [vp, sz]),
        "oracle_gguf_tensor_meta": (C.c_int, [vp, sz, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                              C.POINTER(C.c_int), C.POINTER(C.c_uint64)]),
        "oracle_gguf_tensor_f32": (C.c_int, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "oracle_gguf_tensor_raw": (C.c_int, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz),
                                             C.POINTER(C.c_int)]),
        "oracle_model_open": (C.c_int, [C.c_char_p, C.POINTER(vp)]),
        "oracle_model_from_bytes": (C.c_int, [vp, sz, C.POINTER(vp)]),
        "oracle_model_free": (None, [vp]),
        "oracle_model_config": (C.c_int, [vp, C.POINTER(Config)]),
        "oracle_model_cap_context": (None, [vp, sz]),
        "oracle_model_reset": (None, [vp]),
        "oracle_model_set_kv_f16": (None, [C.c_void_p, C.c_int]),
        "oracle_forward": (C.c_int, [vp, C.c_uint32, sz, vp]),
        "oracle_forward_hidden": (C.c_int, [vp, C.c_uint32, sz, vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(lib().oracle_last_error().decode())


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def get_threads() -> int:
    return int(lib().oracle_get_threads())


def f16_to_f32(h: int) -> float:
    return float(lib().oracle_f16_to_f32(int(h)))


def f32_to_f16(f: float) -> int:
    return int(lib().oracle_f32_to_f16(float(f)))


def dequant(gtype: int, raw, n_elems: int) -> np.ndarray:
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw)
    out = np.empty(n_elems, np.float32)
    _check(lib().oracle_dequant(gtype, _ptr(raw), n_elems, _ptr(out)))
    return out


def dot(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().oracle_dot(_ptr(a), _ptr(b), a.size))


def matvec_f32(w, x, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(rows, np.float32)
    lib().oracle_matvec_f32(_ptr(w), _ptr(x), _ptr(out), rows, cols)
    return out


def matvec_quant(raw, gtype: int, x, rows: int, cols: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8) if isinstance(raw, np.ndarray) else np.frombuffer(bytes(raw), np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(rows, np.float32)
    _check(lib().oracle_matvec_quant(_ptr(raw), gtype, _ptr(x), _ptr(out), rows, cols))
    return out


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_ptr(x), _ptr(w), float(eps), _ptr(out), x.size)
    return out


def softmax(x) -> np.ndarray:
    x = np.array(x, np.float32)
    lib().oracle_softmax(_ptr(x), x.size)
    return x


def silu(x: float) -> float:
    return float(lib().oracle_silu(float(x)))


def swiglu(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    lib().oracle_swiglu(_ptr(g), _ptr(u), _ptr(out), g.size)
    return out


def rope(v, pos: int, n_head: int, head_dim: int, freq_base: float) -> np.ndarray:
    v = np.array(v, np.float32)
    lib().oracle_rope(_ptr(v), pos, n_head, head_dim, float(freq_base))
    return v


def argmax(logits) -> int:
    a = np.ascontiguousarray(logits, np.float32)
    return int(lib().oracle_argmax(_ptr(a), a.size))


def token_nll(logits, target: int) -> float:
    """src/eval.rs:18-23: -log softmax(logits)[target] via log-sum-exp in f64
    (max over f32, exp of the f32 difference widened to f64, sum in order)."""
    lg = np.ascontiguousarray(logits, np.float32)
    mx = np.float32(-np.inf)
    for v in lg:  # f32 fold with f32::max
        mx = max(mx, v)
    d = (lg - mx).astype(np.float32).astype(np.float64)
    sumexp = 0.0
    for e in np.exp(d):  # sequential f64 sum, as the iterator's .sum()
        sumexp += float(e)
    log_prob = float(np.float32(lg[target] - mx)) - np.log(sumexp)
    return float(np.float32(-log_prob))


def perplexity(model, tokens) -> float:
    """src/eval.rs:35-52: teacher-forced perplexity in chunks of the context length,
    each from a fresh KV cache."""
    assert len(tokens) >= 2
    ctx = model.cfg.context_length
    nll, scored = 0.0, 0
    for c0 in range(0, len(tokens), ctx):
        chunk = tokens[c0:c0 + ctx]
        if len(chunk) < 2:
            break
        model.reset()
        for pos in range(len(chunk) - 1):
            nll += token_nll(model.forward(chunk[pos], pos), chunk[pos + 1])
            scored += 1
    return float(np.float32(np.exp(nll / scored)))


def quantize(gtype: int, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    be, bb = BLOCK_ELEMS[gtype], BLOCK_BYTES[gtype]
    assert x.size % be == 0
    out = np.empty(x.size // be * bb, np.uint8)
    fn = {Q8_0: lib().oracle_quantize_q8_0, Q4_0: lib().oracle_quantize_q4_0,
          Q6_K: lib().oracle_quantize_q6_k}[gtype]
    fn(_ptr(x), x.size, _ptr(out))
    return out


class Gguf:
    """The oracle's own GGUF v3 reader (src/gguf/reader.rs:173-351)."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        h = C.c_void_p()
        if path is not None:
            _check(lib().oracle_gguf_open(path.encode(), C.byref(h)))
        else:
            self._buf = np.frombuffer(data, np.uint8)
            _check(lib().oracle_gguf_from_bytes(_ptr(self._buf), len(data), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().oracle_gguf_free(self.h)
            self.h = None

    __del__ = close

    def get_u32(self, key):
        v = C.c_uint32()
        return v.value if lib().oracle_gguf_get_u32(self.h, key.encode(), C.byref(v)) else None

    def get_f32(self, key):
        v = C.c_float()
        return v.value if lib().oracle_gguf_get_f32(self.h, key.encode(), C.byref(v)) else None

    def get_bool(self, key):
        v = C.c_int()
        return bool(v.value) if lib().oracle_gguf_get_bool(self.h, key.encode(), C.byref(v)) else None

    def get_str(self, key):
        p, n = C.c_void_p(), C.c_size_t()
        if not lib().oracle_gguf_get_str(self.h, key.encode(), C.byref(p), C.byref(n)):
            return None
        return C.string_at(p, n.value).decode()

    def get_arr_str(self, key):
        n = C.c_size_t()
        if not lib().oracle_gguf_arr_str_len(self.h, key.encode(), C.byref(n)):
            return None
        out = []
        for i in range(n.value):
            p, ln = C.c_void_p(), C.c_size_t()
            lib().oracle_gguf_arr_str_item(self.h, key.encode(), i, C.byref(p), C.byref(ln))
            out.append(C.string_at(p, ln.value).decode() if ln.value else "")
        return out

    def get_arr_i32(self, key):
        p, n = C.c_void_p(), C.c_size_t()
        if not lib().oracle_gguf_arr_i32(self.h, key.encode(), C.byref(p), C.byref(n)):
            return None
        if n.value == 0:
            return []
        return list(np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_int32)), (n.value,)))

    def tensors(self):
        out = []
        for i in range(lib().oracle_gguf_n_tensors(self.h)):
            nd, dims, ty, off = C.c_uint32(), (C.c_uint64 * 4)(), C.c_int(), C.c_uint64()
            lib().oracle_gguf_tensor_meta(self.h, i, C.byref(nd), dims, C.byref(ty), C.byref(off))
            out.append((lib().oracle_gguf_tensor_name(self.h, i).decode(),
                        [int(dims[d]) for d in range(min(nd.value, 4))], ty.value, off.value))
        return out

    def tensor_f32(self, name):
        p, n = C.c_void_p(), C.c_size_t()
        _check(lib().oracle_gguf_tensor_f32(self.h, name.encode(), C.byref(p), C.byref(n)))
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (n.value,)).copy()

    def tensor_raw(self, name):
        p, n, t = C.c_void_p(), C.c_size_t(), C.c_int()
        _check(lib().oracle_gguf_tensor_raw(self.h, name.encode(), C.byref(p), C.byref(n), C.byref(t)))
        return C.string_at(p, n.value), t.value


class Model:
    """The oracle's CPU `Model` (src/model/llama.rs:20-238): forward, forward_hidden, reset."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        h = C.c_void_p()
        if path is not None:
            _check(lib().oracle_model_open(path.encode(), C.byref(h)))
        else:
            buf = np.frombuffer(data, np.uint8)
            _check(lib().oracle_model_from_bytes(_ptr(buf), len(data), C.byref(h)))
        self.h = h
        c = Config()
        lib().oracle_model_config(h, C.byref(c))
        self.cfg = c

    def close(self):
        if getattr(self, "h", None):
            lib().oracle_model_free(self.h)
            self.h = None

    __del__ = close

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.cfg.vocab_size, np.float32)
        _check(lib().oracle_forward(self.h, int(token), int(pos), _ptr(out)))
        return out

    def forward_hidden(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.cfg.n_embd, np.float32)
        _check(lib().oracle_forward_hidden(self.h, int(token), int(pos), _ptr(out)))
        return out

    def reset(self):
        lib().oracle_model_reset(self.h)

    def set_kv_f16(self, on: bool = True):
        """The CUDA path's opt-in f16 KV cache (not in the reference): K/V are
        rounded to f16 when appended. Empties the cache."""
        lib().oracle_model_set_kv_f16(self.h, int(bool(on)))

    def cap_context(self, n: int):
        lib().oracle_model_cap_context(self.h, int(n))
        c = Config()
        lib().oracle_model_config(self.h, C.byref(c))
        self.cfg = c
