"""Tensor-parallel decode on 2 GPUs (one process per GPU, NCCL bootstrap, the
all-reduce inside the per-token kernel) against the single-device oracle.

Needs at least two GPUs; skipped otherwise. Ranks are never placed on one GPU
(ranks that wait on each other must run concurrently, and the context refuses
two ranks on one device)."""
import os
import queue as _queue

import numpy as np
import pytest

import oracle
from talos_b200 import gguf, synth

from .helpers import prompt, tiny_model
from .test_tp_cpu import TP_SHAPE

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        from talos_b200 import _lib
        import ctypes as C

        n = C.c_int()
        _lib.check(_lib.load().talos_device_count(C.byref(n)))
        return n.value
    except Exception:
        return 0


def _rank(rank, world, data, toks, n_gen, q_id, q_out):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        from talos_b200 import Model, nccl_unique_id

        if rank == 0:
            uid = nccl_unique_id()
            for _ in range(world - 1):
                q_id.put(uid)
        else:
            uid = q_id.get(timeout=120)
        m = Model.load_bytes(data, device=rank, tp_size=world, tp_rank=rank, nccl_id=uid)
        logits = [m.forward_gpu(int(t), pos) for pos, t in enumerate(toks)]
        first = oracle.argmax(logits[-1])  # sample::argmax: the last maximum on ties
        gen = m.generate_greedy(first, len(toks), n_gen) if n_gen else np.zeros(0, np.uint32)
        q_out.put((rank, np.stack(logits), [int(t) for t in gen], None))
        m.close()
    except Exception as e:  # reported to the parent, which fails the test
        q_out.put((rank, None, None, repr(e)))


def run_tp(data, toks, world, n_gen=0, timeout=300):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, data, toks, n_gen, q_id, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, lg, gen, err = q_out.get(timeout=timeout)
            res[r] = (lg, gen, err)
    except _queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    assert len(res) == world, f"ranks answered: {sorted(res)}"
    for r, (_, _, err) in res.items():
        assert err is None, f"rank {r}: {err}"
    return [res[r] for r in range(world)]


def oracle_run(data, toks, n_gen):
    cpu = oracle.Model(data=data)
    logits = [cpu.forward(int(t), pos) for pos, t in enumerate(toks)]
    gen, lg, pos = [], logits[-1], len(toks)
    t = oracle.argmax(lg)
    for _ in range(n_gen):
        lg = cpu.forward(t, pos)
        pos += 1
        t = oracle.argmax(lg)
        gen.append(t)
    return np.stack(logits), gen


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["tiny_f32", "tp_q4_0", "tp_q8_0"])
def test_tp2_matches_oracle(name):
    if name == "tiny_f32":
        data, vocab, tol = tiny_model(gguf.F32), 4096, 1e-4
    else:
        wt = gguf.Q4_0 if name == "tp_q4_0" else gguf.Q8_0
        data, vocab, tol = synth.llama_bytes(TP_SHAPE, 3, wtype=wt), TP_SHAPE.vocab, 1e-3
    toks = prompt(8, vocab, 11)
    n_gen = 12
    ranks = run_tp(data, toks, 2, n_gen)
    ref, ref_gen = oracle_run(data, toks, n_gen)
    for lg, gen, _ in ranks:
        assert np.max(np.abs(lg - ref)) <= tol
        assert gen == ref_gen
    assert np.array_equal(ranks[0][0], ranks[1][0]), "ranks disagree on the logits"


@pytest.mark.slow
@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp2_mistral_7b_shape(tmp_path):
    path = str(tmp_path / "m7b.gguf")
    synth.write_llama(path, synth.with_ctx(synth.MISTRAL_7B, 64), 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    with open(path, "rb") as f:
        data = f.read()
    toks = prompt(4, 32000, 1)
    ranks = run_tp(data, toks, 2, 4, timeout=600)
    ref, ref_gen = oracle_run(data, toks, 4)
    for lg, gen, _ in ranks:
        assert np.max(np.abs(lg - ref)) <= 1e-3
        assert gen == ref_gen
