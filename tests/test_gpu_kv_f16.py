"""The opt-in f16 KV cache (talos_ctx_set_kv_dtype) against the oracle run with
the same cache rounding (K after RoPE and V rounded to f16, ties to even, when
appended). Same bars as the f32 path: greedy tokens identical; logits within
1e-4 max-abs for F32 weights, 1e-3 for quantized weights; both launch paths."""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf, synth
from talos_b200._lib import TalosError

from .helpers import prompt, tiny_model

# the per-token kernel reads an f16 cache with head_dim 32, 64 or 128
HD_SHAPES = {
    32: synth.Shape(n_embd=128, n_layer=2, n_head=4, n_head_kv=2, n_ff=256, vocab=512, ctx=128),
    64: synth.Shape(n_embd=256, n_layer=2, n_head=4, n_head_kv=1, n_ff=512, vocab=512, ctx=128),
    128: synth.Shape(n_embd=512, n_layer=2, n_head=4, n_head_kv=2, n_ff=768, vocab=512, ctx=256),
}

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "layered"])
def sk(request):
    return request.param


def run_pair(data, n_prompt, n_gen, sk):
    cpu = oracle.Model(data=data)
    cpu.set_kv_f16(True)
    gpu = Model.load_bytes(data, step_kernel=sk, kv_dtype="f16")
    assert gpu.ctx.kv_dtype() == "f16"
    toks = prompt(n_prompt, cpu.cfg.vocab_size, 5)
    err, pos = 0.0, 0
    for t in toks:
        c, g = cpu.forward(t, pos), gpu.forward_gpu(t, pos)
        err = max(err, float(np.max(np.abs(g - c))))
        pos += 1
    cpu_tok, gpu_tok = [], []
    for _ in range(n_gen):
        ct, gt = oracle.argmax(c), oracle.argmax(g)
        assert ct == gt, f"greedy token differs at pos {pos}"
        cpu_tok.append(ct)
        gpu_tok.append(gt)
        c, g = cpu.forward(ct, pos), gpu.forward_gpu(gt, pos)
        err = max(err, float(np.max(np.abs(g - c))))
        pos += 1
    gpu.reset()
    last = gpu.prefill(toks, 0)
    first = oracle.argmax(last)
    dev = gpu.generate_greedy(first, n_prompt, n_gen - 1)
    assert [first] + [int(t) for t in dev] == cpu_tok
    gpu.close()
    return err


@pytest.mark.parametrize("hd", [32, 64, 128])
def test_kv_f16_f32_weights(hd, sk):
    err = run_pair(synth.llama_bytes(HD_SHAPES[hd], 9, wtype=gguf.F32), 12, 40, sk)
    assert err <= 1e-4, err


@pytest.mark.parametrize("wtype", [gguf.Q4_0, gguf.Q8_0])
def test_kv_f16_quant_weights(wtype, sk):
    err = run_pair(synth.llama_bytes(HD_SHAPES[128], 4, wtype=wtype), 12, 40, sk)
    assert err <= 1e-3, err


def test_kv_f16_long_sequence():
    # several rounds of positions per warp and split: 300 positions on hd 128
    data = synth.llama_bytes(HD_SHAPES[128], 6, wtype=gguf.Q8_0)
    cpu = oracle.Model(data=data)
    cpu.set_kv_f16(True)
    gpu = Model.load_bytes(data, step_kernel="fused", kv_dtype="f16")
    toks = prompt(250, 512, 2)
    last = gpu.prefill(toks, 0)
    for p, t in enumerate(toks):
        ref = cpu.forward(t, p)
    assert np.max(np.abs(last - ref)) <= 1e-3
    gpu.close()


def test_kv_f16_other_head_dims_use_the_layered_graph():
    # TINY has head_dim 48: AUTO takes the layered graph, FUSED is refused
    data = tiny_model(gguf.Q4_0)
    m = Model.load_bytes(data, kv_dtype="f16")
    assert m.ctx.step_kernel() == "layered"
    cpu = oracle.Model(data=data)
    cpu.set_kv_f16(True)
    for p, t in enumerate([3, 9, 27, 81]):
        assert np.max(np.abs(m.forward_gpu(t, p) - cpu.forward(t, p))) <= 1e-3
    m.ctx.set_step_kernel("fused")
    with pytest.raises(TalosError, match="UNSUPPORTED"):
        m.forward_gpu(1, 4)
    m.close()


def test_kv_dtype_switch_frees_half_and_empties():
    data = tiny_model(gguf.Q4_0)
    m = Model.load_bytes(data)
    toks = prompt(6, 4096, 8)
    ref = [m.forward_gpu(t, p) for p, t in enumerate(toks)]
    b32 = m.ctx.device_bytes()
    m.ctx.set_kv_dtype("f16")
    b16 = m.ctx.device_bytes()
    cfg = m.cfg
    kv_elems = 2 * cfg.n_layer * cfg.context_length * cfg.n_head_kv * (cfg.n_embd // cfg.n_head)
    assert b32 - b16 == kv_elems * 2
    m.ctx.set_kv_dtype("f32")  # back: the same logits as before the switches
    again = [m.forward_gpu(t, p) for p, t in enumerate(toks)]
    assert all(np.array_equal(a, b) for a, b in zip(ref, again))
    m.close()
