"""The Llama-3-70B shape at reduced depth against the oracle: n_embd 8192,
n_ff 28672, 64 heads over 8 kv heads, the full 128,256-token vocabulary, one
layer (every per-layer kernel sees the 70B sizes: the per-token kernel's
8192-element staged inputs and 28672-element down-projection input, the GEMM's
224 K blocks of 128, the 1002 output tiles of the vocabulary). All Q4_0 like
the 70B benchmark model (seed 3). Covers the per-token kernel (prompt fed token
by token, then greedy tokens), the batched prefill and the batched decode of
independent sequences. Bar: 1e-3 absolute on the logits
(src/math/metal/mod.rs:527-531).
"""
import dataclasses

import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf, synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TOL = 1e-3
SHAPE = dataclasses.replace(synth.LLAMA3_70B, n_layer=1, ctx=64)


@pytest.fixture(scope="module")
def data():
    return synth.llama_bytes(SHAPE, 3, wtype=gguf.Q4_0)


@pytest.fixture(scope="module")
def cpu(data):
    m = oracle.Model(data=data)
    yield m
    m.close()


def test_llama70b_shape_per_token_and_prefill(data, cpu):
    V = SHAPE.vocab
    toks = synth.token_ids(3, 6, V)
    cpu.reset()
    ref = [cpu.forward(int(t), p) for p, t in enumerate(toks)]
    gpu = Model.load_bytes(data, step_kernel="fused")
    assert gpu.ctx.step_kernel() == "fused"
    for p, t in enumerate(toks):
        assert np.max(np.abs(gpu.forward_gpu(int(t), p) - ref[p])) <= TOL
    # greedy continuation on the device: the oracle's tokens
    t = oracle.argmax(ref[-1])
    gen = [int(x) for x in gpu.generate_greedy(t, len(toks), 3)]
    want, lg, pos = [], ref[-1], len(toks)
    for _ in range(3):
        lg = cpu.forward(oracle.argmax(lg), pos)
        pos += 1
        want.append(oracle.argmax(lg))
    assert gen == want
    # the same prompt through the batched prefill (one tensor-core pass)
    gpu.reset()
    last = gpu.prefill(toks, 0)
    assert np.max(np.abs(last - ref[-1])) <= TOL
    gpu.close()


def test_llama70b_shape_batched_decode(data, cpu):
    V = SHAPE.vocab
    S, P = 3, 3
    prompts = [synth.token_ids(40 + i, P, V) for i in range(S)]
    gpu = Model.load_bytes(data)
    gpu.set_batch(S)
    lgs = [gpu.forward_batch([pr[p] for pr in prompts], [p] * S) for p in range(P)]
    gpu.close()
    for i in range(S):
        cpu.reset()
        for p in range(P):
            r = cpu.forward(int(prompts[i][p]), p)
            assert np.max(np.abs(lgs[p][i] - r)) <= TOL, f"sequence {i} position {p}"
