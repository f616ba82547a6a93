"""Whole decode steps on the GPU against the oracle's CPU forward.

Bars: greedy tokens identical; logits within 1e-4 max-abs
for F32 weights and 1e-3 max-abs for quantized weights; a re-run is bit-identical
(tests/forward_gpu.rs:183-190). The step tests run both ways a step can be
launched: the per-token kernel ("fused") and the layered kernel graph.
"""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf, synth
from talos_b200.model import weight_shapes
from talos_b200._lib import TalosError

from .helpers import forward_gpu_model, gqa_pair, prompt, tiny_model

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "layered"])
def sk(request):
    return request.param


def test_forward_gpu_matches_cpu(sk):  # tests/forward_gpu.rs:146-193
    data = forward_gpu_model(0)
    cpu = oracle.Model(data=data)
    gpu = Model.load_bytes(data, step_kernel=sk)
    assert gpu.ctx.step_kernel() == sk
    toks = [1, 3, 5, 7, 2, 4]
    max_rel, run1 = 0.0, None
    for pos, t in enumerate(toks):
        c = cpu.forward(t, pos)
        g = gpu.forward_gpu(t, pos)
        max_rel = max(max_rel, float(np.max(np.abs(g - c) / np.maximum(np.abs(c), 1.0))))
        run1 = g
    assert max_rel <= 1e-3
    gpu.reset()
    for pos, t in enumerate(toks):
        run2 = gpu.forward_gpu(t, pos)
    assert np.array_equal(run1, run2), "GPU forward is nondeterministic"


def test_forward_hidden_gpu_matches_cpu(sk):  # tests/forward_gpu.rs:197-228
    data = forward_gpu_model(1)
    cpu = oracle.Model(data=data)
    gpu = Model.load_bytes(data, step_kernel=sk)
    for pos, t in enumerate([1, 3, 5, 7, 2, 4]):
        c = cpu.forward_hidden(t, pos)
        g = gpu.forward_hidden_gpu(t, pos)
        assert g.shape == (16,)
        assert np.max(np.abs(g - c) / np.maximum(np.abs(c), 1.0)) <= 1e-3


def test_gqa_matches_replicated_mha_gpu(sk):  # tests/gqa.rs:194-227 on the GPU path
    g_bytes, m_bytes = gqa_pair(7)
    outs = []
    for data in (g_bytes, m_bytes):
        m = Model.load_bytes(data, step_kernel=sk)
        for pos, t in enumerate([1, 2, 3, 4, 5]):
            lg = m.forward_gpu(t, pos)
        outs.append(lg)
        m.close()
    assert np.max(np.abs(outs[0] - outs[1])) <= 1e-5


def greedy_parity(data, n_prompt, n_gen, tol, seed=42, sk="auto"):
    """Prompt token by token, then greedy decode; compare every step's logits and
    the chosen tokens with the oracle. Returns (max abs err, min top-2 gap)."""
    cpu = oracle.Model(data=data)
    gpu = Model.load_bytes(data, step_kernel=sk)
    vocab = cpu.cfg.vocab_size
    toks = prompt(n_prompt, vocab, seed)
    max_err, min_gap = 0.0, np.inf
    pos = 0
    for t in toks:
        c = cpu.forward(t, pos)
        g = gpu.forward_gpu(t, pos)
        max_err = max(max_err, float(np.max(np.abs(g - c))))
        pos += 1
    cpu_tokens, gpu_tokens = [], []
    for _ in range(n_gen):
        ct, gt = oracle.argmax(c), oracle.argmax(g)
        s = np.sort(c)
        min_gap = min(min_gap, float(s[-1] - s[-2]))
        cpu_tokens.append(ct)
        gpu_tokens.append(gt)
        assert ct == gt, f"greedy token differs at pos {pos}: cpu {ct} gpu {gt} (top-2 gap {s[-1] - s[-2]:.2e})"
        c = cpu.forward(ct, pos)
        g = gpu.forward_gpu(gt, pos)
        max_err = max(max_err, float(np.max(np.abs(g - c))))
        pos += 1
    assert max_err <= tol, f"max abs logit err {max_err:.3e} > {tol}"
    # the on-device greedy loop chooses the same tokens
    gpu.reset()
    last = gpu.prefill(toks, 0)
    first = oracle.argmax(last)
    dev = gpu.generate_greedy(first, n_prompt, n_gen - 1)
    assert [first] + [int(t) for t in dev] == cpu_tokens
    gpu.close()
    return max_err, min_gap


def test_tiny_f32_greedy_parity(sk):  # the tiny F32 benchmark model
    err, gap = greedy_parity(tiny_model(gguf.F32), 16, 64, 1e-4, sk=sk)
    print(f"tiny F32: max abs err {err:.2e}, min top-2 gap {gap:.2e}")


@pytest.mark.parametrize("wtype", [gguf.Q4_0, gguf.Q8_0])
def test_tiny_quant_greedy_parity(wtype, sk):  # the tiny quantized benchmark models
    err, gap = greedy_parity(tiny_model(wtype), 16, 64, 1e-3, sk=sk)
    print(f"tiny {gguf.TYPE_NAMES[wtype]}: max abs err {err:.2e}, min top-2 gap {gap:.2e}")


def test_argument_errors(sk):
    m = Model.load_bytes(forward_gpu_model(2), step_kernel=sk)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.forward_gpu(16, 0)  # token == vocab
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.forward_gpu(1, 8)  # pos == ctx
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.upload("blk.9.attn_q.weight", np.zeros(16 * 16, np.float32), gguf.F32, 16, 16)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.upload("blk.0.attn_q.weight", np.zeros(16 * 8, np.float32), gguf.F32, 8, 16)
    m.close()


def test_missing_weight_is_state_error():
    from talos_b200 import Context, Config

    ctx = Context(Config(1, 4, 2, 16, 32, 8, 16, 1e-5, 4, 1e4))
    with pytest.raises(TalosError, match="STATE"):
        ctx.forward(1, 0)
    ctx.close()


def test_cap_context(sk):
    m = Model.load_bytes(forward_gpu_model(3), step_kernel=sk)
    m.cap_context(4)
    assert m.cfg.context_length == 4
    m.forward_gpu(1, 3)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.forward_gpu(1, 4)
    m.close()


def test_step_kernel_choice():
    """AUTO takes the per-token kernel where the model fits it; head_dim 256 does
    not (attention keeps head_dim <= 128 in registers), so AUTO falls back to the
    layered graph and an explicit FUSED request fails as UNSUPPORTED."""
    wide = synth.Shape(n_embd=256, n_layer=1, n_head=1, n_head_kv=1, n_ff=64, vocab=32, ctx=8)
    data = synth.llama_bytes(wide, 5, wtype=gguf.F32)
    m = Model.load_bytes(data)
    assert m.ctx.step_kernel() == "layered"
    cpu = oracle.Model(data=data)
    assert np.max(np.abs(m.forward_gpu(3, 0) - cpu.forward(3, 0))) <= 1e-4
    m.ctx.set_step_kernel("fused")
    with pytest.raises(TalosError, match="UNSUPPORTED"):
        m.forward_gpu(3, 1)
    m.close()
    t = Model.load_bytes(tiny_model(gguf.Q4_0))
    assert t.ctx.step_kernel() == "fused"
    t.close()


def test_fused_and_layered_agree():
    """The two launch paths compute the same step: logits within 1e-5 of each
    other on the tiny Q4_0 model over a prompt."""
    data = tiny_model(gguf.Q4_0)
    a = Model.load_bytes(data, step_kernel="fused")
    b = Model.load_bytes(data, step_kernel="layered")
    for pos, t in enumerate(prompt(12, 4096, 9)):
        la, lb = a.forward_gpu(t, pos), b.forward_gpu(t, pos)
    assert np.max(np.abs(la - lb)) <= 1e-5
    a.close()
    b.close()


@pytest.mark.parametrize("second", [gguf.Q4_0, gguf.Q8_0])
def test_reupload_replaces_weights(second):
    """Uploading every tensor again into a loaded context (same shapes; the same
    type reuses each tensor's device range, Q8_0 after Q4_0 needs larger ones)
    gives the second model's logits, with the first model's forward steps run
    before the re-upload still in the stream's history."""
    a_bytes = tiny_model(gguf.Q4_0)
    b_bytes = synth.llama_bytes(synth.TINY, 23, wtype=second)
    m = Model.load_bytes(a_bytes)
    for pos, t in enumerate([5, 6, 7]):
        m.forward_gpu(t, pos)
    b = gguf.GgufFile.from_bytes(b_bytes)
    for name, (rows, cols) in weight_shapes(m.cfg).items():
        if rows == 1:
            m.ctx.upload(name, b.tensor_f32(name), gguf.F32, 1, cols)
        else:
            raw, gt = b.tensor_raw(name)
            m.ctx.upload(name, raw, gt, rows, cols)
    m.reset()
    cpu = oracle.Model(data=b_bytes)
    for pos, t in enumerate([5, 6, 7, 8]):
        assert np.max(np.abs(m.forward_gpu(t, pos) - cpu.forward(t, pos))) <= 1e-3
    m.close()


@pytest.mark.slow
@pytest.mark.parametrize("step_kernel", ["fused", "layered"])
def test_mistral_7b_shape_parity(tmp_path, step_kernel):
    """The Mistral-7B-shape benchmark model at full size: Q4_0 + Q6_K output; a short prompt and
    greedy steps against the oracle (the CPU forward reads 4 GB per token)."""
    path = str(tmp_path / "m7b.gguf")
    synth.write_llama(path, synth.with_ctx(synth.MISTRAL_7B, 64), 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    cpu = oracle.Model(path=path)
    gpu = Model.load(path, step_kernel=step_kernel)
    toks = prompt(4, 32000, 1)
    pos, max_err = 0, 0.0
    for t in toks:
        c, g = cpu.forward(t, pos), gpu.forward_gpu(t, pos)
        max_err = max(max_err, float(np.max(np.abs(g - c))))
        pos += 1
    for _ in range(4):
        ct, gt = oracle.argmax(c), oracle.argmax(g)
        assert ct == gt
        c, g = cpu.forward(ct, pos), gpu.forward_gpu(gt, pos)
        max_err = max(max_err, float(np.max(np.abs(g - c))))
        pos += 1
    print(f"7B: max abs logit err {max_err:.2e}")
    assert max_err <= 1e-3
    gpu.close()
