"""Pin the CPU oracle to the reference's own known-answer tests.

Each test restates a unit test of Tsuskov/talos (file:line given) and runs it
against oracle/talos_oracle.c. Tolerances are the reference's (abs 1e-5 for
CPU-to-CPU checks).
"""
import math

import numpy as np
import pytest

import oracle

TOL = 1e-5  # src/math/ops.rs:67-69, src/math/matmul.rs:77


def close(a, b, tol=TOL):
    assert abs(a - b) < tol, f"expected {b}, got {a}"


# ---------------------------------------------------------------- ops.rs:71-163

def test_rmsnorm_hand():  # ops.rs:71-83
    out = oracle.rmsnorm([1.0, 2.0, 3.0], [1.0, 1.0, 1.0], 0.0)
    scale = 1.0 / math.sqrt(14.0 / 3.0)
    for o, x in zip(out, [1, 2, 3]):
        close(o, x * scale)


def test_rmsnorm_weighted():  # ops.rs:85-95
    out = oracle.rmsnorm([2.0, 0.0], [3.0, 5.0], 0.0)
    close(out[0], 2.0 / math.sqrt(2.0) * 3.0)
    close(out[1], 0.0)


def test_softmax_sums_to_one_and_known():  # ops.rs:97-107
    x = oracle.softmax([1.0, 2.0, 3.0])
    close(float(np.sum(x)), 1.0)
    denom = math.exp(-2) + math.exp(-1) + 1.0
    close(x[0], math.exp(-2) / denom)
    close(x[1], math.exp(-1) / denom)
    close(x[2], 1.0 / denom)


def test_softmax_uniform():  # ops.rs:109-116
    for v in oracle.softmax([5.0] * 4):
        close(v, 0.25)


def test_silu():  # ops.rs:118-123
    close(oracle.silu(0.0), 0.0)
    close(oracle.silu(2.0), 2.0 / (1.0 + math.exp(-2.0)))


def test_swiglu_small():  # ops.rs:125-133
    out = oracle.swiglu([0.0, 2.0], [10.0, 3.0])
    close(out[0], 0.0)
    close(out[1], oracle.silu(2.0) * 3.0)


def test_rope_preserves_pair_norm():  # ops.rs:135-151
    n_head, hd = 2, 4
    v = np.arange(n_head * hd, dtype=np.float32) + 1.0
    r = oracle.rope(v, 7, n_head, hd, 10000.0)
    for h in range(n_head):
        for i in range(hd // 2):
            b = h * hd
            n0 = v[b + 2 * i] ** 2 + v[b + 2 * i + 1] ** 2
            n1 = r[b + 2 * i] ** 2 + r[b + 2 * i + 1] ** 2
            assert abs(n1 - n0) < 1e-4 * max(1.0, n0)


def test_rope_pos_zero_identity():  # ops.rs:153-163
    v = np.arange(18, dtype=np.float32) * 0.5 - 1.0
    r = oracle.rope(v, 0, 3, 6, 10000.0)
    np.testing.assert_allclose(r, v, atol=TOL)


def test_rope_interleaved_pairs_known_angle():
    # theta_i = pos * base^(-2i/hd) rotates the adjacent pair (2i, 2i+1) (ops.rs:39-61).
    hd, pos, base = 4, 3, 10000.0
    v = np.array([1.0, 0.0, 0.0, 1.0], np.float32)
    r = oracle.rope(v, pos, 1, hd, base)
    t0 = pos * base ** 0.0
    t1 = pos * base ** (-2.0 / hd)
    np.testing.assert_allclose(r, [math.cos(t0), math.sin(t0), -math.sin(t1), math.cos(t1)], atol=1e-5)


# ---------------------------------------------------------------- matmul.rs:54-97

def _naive(w, x, rows, cols):
    out = np.zeros(rows, np.float32)
    for m in range(rows):
        acc = np.float32(0)
        for k in range(cols):
            acc = np.float32(acc + np.float32(w[m * cols + k] * x[k]))
        out[m] = acc
    return out


@pytest.mark.parametrize("rows,cols", [(8, 8), (5, 13), (13, 5)])
def test_matvec_vs_naive(rows, cols):  # matmul.rs:66-87
    rng = np.random.default_rng(rows * 100 + cols)
    w = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    np.testing.assert_allclose(oracle.matvec_f32(w, x, rows, cols), _naive(w, x, rows, cols), atol=TOL)


def test_matvec_hand():  # matmul.rs:89-97
    out = oracle.matvec_f32([1, 2, 3, 4, 5, 6], [1, 1], 3, 2)
    assert list(out) == [3.0, 7.0, 11.0]


def test_dot_lanes_and_tail():
    # 8-lane accumulation + scalar tail (matmul.rs:15-30): exact on integers.
    a = np.arange(1, 20, dtype=np.float32)
    b = np.ones(19, np.float32)
    assert oracle.dot(a, b) == float(a.sum())


# ---------------------------------------------------------------- dtype.rs:124-167

def _sample_block():  # dtype.rs:128-130
    return np.array([(i - 16.0) * 0.37 + 0.1 for i in range(32)], np.float32)


def test_q8_0_round_trip():  # dtype.rs:132-146
    x = _sample_block()
    raw = oracle.quantize(oracle.Q8_0, x)
    out = oracle.dequant(oracle.Q8_0, raw, 32)
    d = np.abs(x).max() / 127.0
    assert np.all(np.abs(x - out) <= d + 1e-3)


def test_q4_0_round_trip():  # dtype.rs:148-167
    x = _sample_block()
    raw = oracle.quantize(oracle.Q4_0, x)
    out = oracle.dequant(oracle.Q4_0, raw, 32)
    mx = x[np.argmax(np.abs(x))]
    d = abs(mx / -8.0)
    assert np.all(np.abs(x - out) <= d + 1e-3)


def test_q4_0_quantizer_matches_reference_helper():
    # The unclamped helper of dtype.rs:149-160 and the clamped one of
    # metal/mod.rs:563-574 agree on finite input; restate the first in numpy.
    x = _sample_block()
    mx = 0.0
    for v in x:
        if abs(v) > abs(mx):
            mx = v
    d = np.float32(mx) / np.float32(-8.0)
    idv = np.float32(1.0) / d
    want = bytearray(np.float16(d).tobytes())
    for j in range(16):
        a = min(int(np.float32(x[j] * idv + np.float32(8.5))), 15)
        b = min(int(np.float32(x[j + 16] * idv + np.float32(8.5))), 15)
        want.append(a | (b << 4))
    assert bytes(oracle.quantize(oracle.Q4_0, x)) == bytes(want)


def test_q6_k_round_trip():
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.02, 512).astype(np.float32)
    raw = oracle.quantize(oracle.Q6_K, x)
    assert raw.size == 2 * 210
    out = oracle.dequant(oracle.Q6_K, raw, 512)
    # one 6-bit step of each 16-element sub-block
    for s in range(32):
        blk = x[16 * s:16 * s + 16]
        step = np.abs(blk).max() / 32.0 * 1.1 + 1e-6
        assert np.all(np.abs(blk - out[16 * s:16 * s + 16]) <= step)


# Independent numpy restatement of dtype.rs:64-121 (cross-checks the C oracle).
def _np_dequant(gtype, raw, n):
    raw = np.frombuffer(bytes(raw), np.uint8)
    out = np.empty(n, np.float32)
    if gtype == oracle.F32:
        return raw.view("<f4")[:n].copy()
    if gtype == oracle.Q8_0:
        b = raw.reshape(-1, 34)
        d = b[:, :2].copy().view("<f2").astype(np.float32)
        q = b[:, 2:].view(np.int8).astype(np.float32)
        return (d * q).reshape(-1)
    if gtype == oracle.Q4_0:
        b = raw.reshape(-1, 18)
        d = b[:, :2].copy().view("<f2").astype(np.float32)
        qs = b[:, 2:]
        lo = (qs & 0xF).astype(np.int32) - 8
        hi = (qs >> 4).astype(np.int32) - 8
        return (d * np.concatenate([lo, hi], 1).astype(np.float32)).reshape(-1)
    if gtype == oracle.Q6_K:
        b = raw.reshape(-1, 210)
        for sb in range(b.shape[0]):
            blk = b[sb]
            d = np.frombuffer(blk[208:210].tobytes(), "<f2").astype(np.float32)[0]
            for n_ in range(2):
                ql, qh = blk[n_ * 64:], blk[128 + n_ * 32:]
                sc = blk[192 + n_ * 8:].view(np.int8)
                y = out[sb * 256 + n_ * 128:]
                for l in range(32):
                    is_ = l // 16
                    q1 = int((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32
                    q2 = int((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32
                    q3 = int((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32
                    q4 = int((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32
                    y[l] = np.float32(d * np.float32(sc[is_])) * np.float32(q1)
                    y[l + 32] = np.float32(d * np.float32(sc[is_ + 2])) * np.float32(q2)
                    y[l + 64] = np.float32(d * np.float32(sc[is_ + 4])) * np.float32(q3)
                    y[l + 96] = np.float32(d * np.float32(sc[is_ + 6])) * np.float32(q4)
        return out
    raise ValueError(gtype)


@pytest.mark.parametrize("gtype,n", [(oracle.F32, 64), (oracle.Q8_0, 256), (oracle.Q4_0, 256),
                                     (oracle.Q6_K, 512)])
def test_dequant_matches_numpy_restatement(gtype, n):
    rng = np.random.default_rng(gtype + 1)
    nbytes = n // oracle.BLOCK_ELEMS[gtype] * oracle.BLOCK_BYTES[gtype]
    raw = rng.integers(0, 256, nbytes, dtype=np.uint8)
    if gtype == oracle.F32:
        raw = rng.normal(0, 1, n).astype(np.float32).view(np.uint8)
    else:  # keep the f16 scales finite
        bb = oracle.BLOCK_BYTES[gtype]
        off = 208 if gtype == oracle.Q6_K else 0
        for blk in range(nbytes // bb):
            raw[blk * bb + off:blk * bb + off + 2] = np.frombuffer(
                np.float16(rng.uniform(-0.05, 0.05)).tobytes(), np.uint8)
    got = oracle.dequant(gtype, raw, n)
    want = _np_dequant(gtype, raw, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_f16_exhaustive():
    # half::f16::to_f32 is exact: all 65536 patterns against numpy (NaN: any NaN).
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h], np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(11)
    vals = np.concatenate([
        rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 1000),
        [0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.9802322e-8, 6.1e-5]]).astype(np.float32)
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- sample.rs:7-14, 84-88

def test_argmax_picks_max():  # sample.rs:84-88
    assert oracle.argmax([0.1, 9.0, -3.0, 2.0]) == 1


def test_argmax_ties_take_last():
    # Iterator::max_by returns the last of equal maxima.
    assert oracle.argmax([1.0, 5.0, 5.0, 2.0]) == 2
    # total_cmp: +0.0 > -0.0, NaN above everything
    assert oracle.argmax([0.0, -0.0]) == 0
    assert oracle.argmax([1.0, float("nan"), 3.0]) == 1


# ---------------------------------------------------------------- perplexity (src/eval.rs)


def test_token_nll_uniform_is_ln_vocab():  # eval.rs: uniform_logits_score_ln_vocab
    v = 50
    for target in (0, 7, v - 1):
        assert abs(oracle.token_nll(np.zeros(v, np.float32), target) - np.log(v)) < 1e-4


def test_token_nll_confident_is_near_zero():  # eval.rs: confident_correct_prediction_scores_near_zero
    lg = np.zeros(16, np.float32)
    lg[5] = 100.0
    assert oracle.token_nll(lg, 5) < 1e-3


def test_token_nll_hand_softmax():  # eval.rs: nll_matches_hand_computed_softmax
    lg = np.array([1.0, 2.0, 3.0], np.float32)
    want = -np.log(np.exp(3.0) / (np.exp(1.0) + np.exp(2.0) + np.exp(3.0)))
    assert abs(oracle.token_nll(lg, 2) - want) < 1e-5


def test_perplexity_chunks_from_a_fresh_cache():
    """eval.rs:35-52: chunks of the context length, each scored from position 0."""
    from .helpers import prompt, tiny_model
    from talos_b200 import gguf

    m = oracle.Model(data=tiny_model(gguf.F32))
    m.cap_context(8)
    toks = prompt(19, 4096, 3)  # chunks of 8, 8, 3
    got = oracle.perplexity(m, toks)
    nll, n = 0.0, 0
    for c0 in (0, 8, 16):
        ch = toks[c0:c0 + 8]
        m.reset()
        for pos in range(len(ch) - 1):
            nll += oracle.token_nll(m.forward(ch[pos], pos), ch[pos + 1])
            n += 1
    assert n == 7 + 7 + 2
    assert got == np.float32(np.exp(nll / n))
