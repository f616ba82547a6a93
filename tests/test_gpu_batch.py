"""Batched steps on the tensor-core GEMM: batched decode (talos_ctx_set_batch /
talos_forward_batch, up to 64 sequences per step, each with its own cache slot
and position) against one oracle model per sequence, and prefill of up to 128
consecutive prompt positions per step. Bars as for one sequence: logits within
1e-3 max-abs (quantized weights), greedy tokens identical, reruns bit-identical."""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf, synth
from talos_b200._lib import TalosError

from .helpers import prompt, tiny_model

pytestmark = pytest.mark.gpu

SHAPE_Q6K = synth.Shape(n_embd=512, n_layer=2, n_head=4, n_head_kv=2, n_ff=768, vocab=512, ctx=128)


def run_batch(data, prompts, start, steps, m=None):
    """Slot i joins at step start[i] (position 0) and then takes one token per
    step: its prompt, then its greedy choice. Returns per-slot logits lists."""
    cpu = [oracle.Model(data=data) for _ in prompts]
    own = m is None
    if own:
        m = Model.load_bytes(data)
        m.ctx.set_batch(len(prompts))
    pos = [0] * len(prompts)
    nxt = [p[0] for p in prompts]
    gpu_out, cpu_out = [[] for _ in prompts], [[] for _ in prompts]
    for step in range(steps):
        live = [i for i in range(len(prompts)) if start[i] <= step]
        n = max(live) + 1  # slots 0 .. n-1; a slot that has not joined yet re-feeds position 0
        toks = [nxt[i] if start[i] <= step else prompts[i][0] for i in range(n)]
        ps = [pos[i] if start[i] <= step else 0 for i in range(n)]
        lg = m.ctx.forward_batch(toks, ps)
        for i in live:
            c = cpu[i].forward(toks[i], ps[i])
            gpu_out[i].append(lg[i])
            cpu_out[i].append(c)
            pos[i] += 1
            k = pos[i]
            nxt[i] = prompts[i][k] if k < len(prompts[i]) else oracle.argmax(c)
            if k >= len(prompts[i]):
                assert oracle.argmax(lg[i]) == nxt[i], f"slot {i} greedy token differs at pos {k}"
    if own:
        m.close()
    return gpu_out, cpu_out


def max_err(gpu_out, cpu_out):
    return max(float(np.max(np.abs(g - c))) for gs, cs in zip(gpu_out, cpu_out) for g, c in zip(gs, cs))


@pytest.mark.parametrize("wtype", [gguf.Q4_0, gguf.Q8_0])
def test_batch_matches_oracle_per_sequence(wtype):
    data = tiny_model(wtype)
    prompts = [prompt(n, 4096, 20 + i) for i, n in enumerate([6, 9, 4, 12])]
    g, c = run_batch(data, prompts, start=[0, 0, 0, 3], steps=16)
    assert max_err(g, c) <= 1e-3


def test_batch_q6_k_output_and_fewer_slots():
    data = synth.llama_bytes(SHAPE_Q6K, 8, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    prompts = [prompt(n, 512, 40 + i) for i, n in enumerate([5, 7])]
    g, c = run_batch(data, prompts, start=[0, 2], steps=12)
    assert max_err(g, c) <= 1e-3


def test_batch_rerun_bit_identical():
    data = tiny_model(gguf.Q4_0)
    prompts = [prompt(5, 4096, 60 + i) for i in range(4)]
    m = Model.load_bytes(data)
    m.ctx.set_batch(4)
    a, _ = run_batch(data, prompts, [0, 0, 1, 2], 8, m=m)
    b, _ = run_batch(data, prompts, [0, 0, 1, 2], 8, m=m)
    assert all(np.array_equal(x, y) for xs, ys in zip(a, b) for x, y in zip(xs, ys))
    m.close()


def test_batch_argument_errors():
    m = Model.load_bytes(tiny_model(gguf.Q4_0))
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.forward_batch([1], [0])  # no slots reserved
    m.ctx.set_batch(2)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.forward_batch([1, 2, 3], [0, 0, 0])
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.forward_batch([4096, 1], [0, 0])  # token == vocab
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.set_batch(65)
    m.close()
    f = Model.load_bytes(tiny_model(gguf.F32))
    f.ctx.set_batch(1)
    with pytest.raises(TalosError, match="UNSUPPORTED"):
        f.ctx.forward_batch([1], [0])
    f.close()


def test_batch_32_sequences():
    """32 sequences at once (the batch size of the 70B-shape benchmark), each
    joining at its own step with its own prompt length: every sequence's logits
    and greedy tokens against its own oracle model."""
    data = tiny_model(gguf.Q4_0)
    prompts = [prompt(2 + (7 * i) % 9, 4096, 100 + i) for i in range(32)]
    g, c = run_batch(data, prompts, start=[i % 5 for i in range(32)], steps=14)
    assert max_err(g, c) <= 1e-3


def test_batch_token_tile_sizes():
    """Step sizes around the 32 / 64-column tile boundaries (graphs per tile size)."""
    data = tiny_model(gguf.Q8_0)
    for nseq in (33, 64):
        prompts = [prompt(3, 4096, 300 + i) for i in range(nseq)]
        g, c = run_batch(data, prompts, start=[0] * nseq, steps=5)
        assert max_err(g, c) <= 1e-3


@pytest.mark.parametrize("n,pos0", [(1, 0), (5, 0), (11, 0), (6, 3), (128, 0), (150, 5), (249, 0)])
def test_prefill_in_batched_steps(n, pos0):
    """talos_prefill runs up to 128 consecutive prompt positions per weight pass
    on the main cache: the last logits and the decode steps after it match the
    oracle."""
    data = tiny_model(gguf.Q8_0)
    cpu = oracle.Model(data=data)
    gpu = Model.load_bytes(data)
    head = prompt(pos0, 4096, 70)
    toks = prompt(n, 4096, 71)
    if pos0:
        gpu.prefill(head, 0)
    for p, t in enumerate(head + toks):
        ref = cpu.forward(t, p)
    last = gpu.prefill(toks, pos0)
    assert np.max(np.abs(last - ref)) <= 1e-3
    pos = pos0 + n
    t = oracle.argmax(ref)
    for _ in range(6):  # the cache rows the batched steps wrote serve the per-token kernel
        g, c = gpu.forward_gpu(t, pos), cpu.forward(t, pos)
        assert np.max(np.abs(g - c)) <= 1e-3
        t, pos = oracle.argmax(c), pos + 1
    gpu.close()


def test_cap_context_releases_batch_slots():
    m = Model.load_bytes(tiny_model(gguf.Q4_0))
    m.ctx.set_batch(2)
    m.ctx.forward_batch([1, 2], [0, 0])
    m.cap_context(64)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        m.ctx.forward_batch([1, 2], [1, 1])
    m.ctx.set_batch(2)
    assert m.ctx.forward_batch([1, 2], [0, 0]).shape == (2, 4096)
    m.close()


def oracle_greedy(cpu, toks, n_gen):
    """Prompt then n_gen greedy tokens on one oracle model: (last prompt logits, tokens)."""
    cpu.reset()
    for p, t in enumerate(toks):
        lg = cpu.forward(int(t), p)
    last, gen, pos = lg, [], len(toks)
    t = oracle.argmax(lg)
    for _ in range(n_gen):
        gen.append(t)
        lg = cpu.forward(t, pos)
        pos += 1
        t = oracle.argmax(lg)
    return last, gen


@pytest.mark.parametrize("wtype", [gguf.Q4_0, gguf.Q8_0])
def test_prefill_slot_then_batch_greedy(wtype):
    """The multi-prompt workload: each sequence's prompt into its slot
    (talos_prefill_slot; 150 tokens take two passes), then every sequence's
    greedy tokens together on the device (talos_generate_batch_greedy). Tokens
    identical to one oracle run per sequence."""
    data = tiny_model(wtype)
    lens = [20, 7, 150, 33, 1]
    prompts = [prompt(n, 4096, 40 + i) for i, n in enumerate(lens)]
    n_gen = 12
    cpu = oracle.Model(data=data)
    want = [oracle_greedy(cpu, p, n_gen) for p in prompts]
    m = Model.load_bytes(data)
    m.ctx.set_batch(len(prompts))
    firsts = []
    for i, p in enumerate(prompts):
        last = m.ctx.prefill_slot(i, p, 0)
        assert np.max(np.abs(last - want[i][0])) <= 1e-3, f"sequence {i}"
        firsts.append(oracle.argmax(last))
    gen = m.ctx.generate_batch_greedy(firsts, lens, n_gen)  # [step, seq]
    for i in range(len(prompts)):
        assert [firsts[i]] + [int(x) for x in gen[:-1, i]] == want[i][1], f"sequence {i}"
    # a second call continues from where the first left every sequence
    more = m.ctx.generate_batch_greedy([int(x) for x in gen[-1]], [n + n_gen for n in lens], 2)
    for i, p in enumerate(prompts):
        _, longer = oracle_greedy(cpu, p, n_gen + 2)
        assert [int(x) for x in gen[-1:, i]] + [int(x) for x in more[:-1, i]] == longer[n_gen:], f"sequence {i}"
    m.close()


def test_prefill_slot_argument_errors():
    m = Model.load_bytes(tiny_model(gguf.Q4_0))
    with pytest.raises(TalosError):
        m.ctx.prefill_slot(0, [1, 2, 3])  # no slots reserved
    m.ctx.set_batch(2)
    with pytest.raises(TalosError):
        m.ctx.prefill_slot(2, [1, 2, 3])
    with pytest.raises(TalosError):
        m.ctx.generate_batch_greedy([1, 2], [250, 0], 10)  # positions past the 256-position context
    m.close()
