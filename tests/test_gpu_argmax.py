"""The greedy choice on the GPU follows sample::argmax (src/sample.rs:7-14): the
maximum under f32::total_cmp, and on ties the LAST maximal index (Rust's
Iterator::max_by keeps the last of equal elements).

* talos_argmax, the device argmax over a given vector, against the oracle's
  restatement on hand-made vectors: ties, -0.0 against +0.0, NaNs of both signs,
  infinities (the reference's own case is src/sample.rs:84-88).
* Exact ties made inside a decode step: output.weight gets a copy of the row that
  wins at a probe step, at a later (or earlier) row index. The two logits are then
  bit-identical, and talos_forward's logits, the device greedy loop
  (talos_generate_greedy) and the batched step all pick the later index, on both
  ways a step is launched.
"""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf, synth
from talos_b200.model import argmax as gpu_argmax

pytestmark = pytest.mark.gpu

NAN_P = np.frombuffer(np.uint32(0x7FC00000).tobytes(), np.float32)[0]
NAN_N = np.frombuffer(np.uint32(0xFFC00000).tobytes(), np.float32)[0]
INF = np.float32(np.inf)

CASES = [
    ([0.1, 9.0, -3.0, 2.0], 1),            # src/sample.rs:84-88
    ([1.0, 5.0, 5.0, 2.0], 2),             # tie: the last maximum
    ([5.0, 5.0, 5.0], 2),
    ([-0.0, 0.0], 1),                      # +0.0 > -0.0 under total_cmp
    ([0.0, -0.0], 0),
    ([-0.0, -0.0, -1.0], 1),
    ([1.0, NAN_P, 3.0], 1),                # +NaN above everything
    ([NAN_P, INF], 0),
    ([INF, NAN_P, NAN_P], 2),
    ([NAN_N, -INF], 1),                    # -NaN below everything
    ([NAN_N, NAN_N], 1),
    ([-INF, -INF, -3.0e38], 2),
]


@pytest.mark.parametrize("vals,want", CASES)
def test_device_argmax_total_order(vals, want):
    v = np.array(vals, np.float32)
    assert oracle.argmax(v) == want
    assert gpu_argmax(v) == want


def test_device_argmax_planted_ties_large():
    rng = np.random.default_rng(11)
    v = rng.normal(0, 1, 1_000_003).astype(np.float32)
    m = np.float32(v.max() + 1.0)
    for i in (17, 500_000, 999_999):
        v[i] = m
    assert oracle.argmax(v) == 999_999
    assert gpu_argmax(v) == 999_999


def tied_model(wtype, probe_pos, seed=42):
    """The tiny Llama with output.weight row b a byte copy of row a, where a is
    the oracle's choice at position probe_pos of the seeded prompt. Returns
    (gguf bytes, prompt, a, b, expected choice = max(a, b))."""
    shape = synth.TINY
    V, E = shape.vocab, shape.n_embd
    base = synth.llama_bytes(shape, seed, wtype=wtype)
    toks = synth.token_ids(seed, probe_pos + 1, V)
    cpu = oracle.Model(data=base)
    for p, t in enumerate(toks):
        lg = cpu.forward(t, p)
    cpu.close()
    a = oracle.argmax(lg)
    b = a + 1 + (a * 7919) % (V - 1 - a) if a < V - 1 else a - 3
    w = synth.llama_gguf(shape, seed, wtype=wtype)
    row = E // gguf.BLOCK_ELEMS[wtype] * gguf.BLOCK_BYTES[wtype]
    out = synth.tensor(seed, "output.weight", V, E, wtype).copy()
    out[b * row:(b + 1) * row] = out[a * row:(a + 1) * row]
    for t in w.tensors:
        if t.name == "output.weight":
            t.data = out.tobytes()
    return w.to_bytes(), toks, a, b, max(a, b)


@pytest.mark.parametrize("sk", ["fused", "layered"])
@pytest.mark.parametrize("wtype", [gguf.Q8_0, gguf.F32])
def test_tie_in_a_decode_step(wtype, sk):
    data, toks, a, b, want = tied_model(wtype, probe_pos=5)
    cpu = oracle.Model(data=data)
    for p, t in enumerate(toks):
        c = cpu.forward(t, p)
    assert c[a] == c[b] and oracle.argmax(c) == want
    gpu = Model.load_bytes(data, step_kernel=sk)
    for p, t in enumerate(toks):
        g = gpu.forward_gpu(t, p)
    assert g.view(np.uint32)[a] == g.view(np.uint32)[b], "tied rows gave different logits"
    assert oracle.argmax(g) == want and gpu_argmax(g) == want
    # the device greedy loop's choice at the same position
    gpu.reset()
    for p, t in enumerate(toks[:-1]):
        gpu.forward_gpu(t, p)
    got = gpu.generate_greedy(toks[-1], len(toks) - 1, 1)
    assert int(got[0]) == want
    gpu.close()


def test_tie_in_a_batched_step():
    data, toks, a, b, want = tied_model(gguf.Q8_0, probe_pos=5)
    gpu = Model.load_bytes(data)
    gpu.set_batch(2)
    other = synth.token_ids(3, len(toks), synth.TINY.vocab)
    for p, t in enumerate(toks):
        lg = gpu.forward_batch([t, other[p]], [p, p])
    g = lg[0]
    assert g.view(np.uint32)[a] == g.view(np.uint32)[b]
    assert oracle.argmax(g) == want
    gpu.close()
