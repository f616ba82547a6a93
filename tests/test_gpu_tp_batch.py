"""Batched steps under tensor parallelism on 2 GPUs (one process per GPU), against
the single-device oracle: batched decode of independent sequences, the batched
prefill and perplexity, and the bounded cross-rank waits (a rank that withholds
its step makes the other rank's step return TALOS_ERR_TIMEOUT; after
talos_ctx_tp_resync on both ranks the next steps match the oracle again).

Each rank keeps its shard of the q/k/v/gate/up/output rows and of the o/down
columns; the row-parallel o-proj and down GEMMs store their rows into every
rank's receive slots from the GEMM epilogue and a join kernel sums them in rank
order, so both ranks hold the same residual stream and the same gathered
logits. Needs at least two GPUs; skipped otherwise. NVLS is off in every rank
(nothing here uses multicast).
"""
import os
import queue as _queue
import time
import traceback

import numpy as np
import pytest

import oracle
from talos_b200 import gguf, synth

from .test_gpu_tp import _gpus
from .test_tp_cpu import TP_SHAPE

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")]

TOL = 1e-3  # src/math/metal/mod.rs:527-531, 1e-3 * max(|cpu|, 1), taken as an absolute bar on O(1) logits
SHAPE = synth.with_ctx(TP_SHAPE, 256)


def _model(wt):
    return synth.llama_bytes(SHAPE, 3, wtype=wt, out_type=gguf.Q6_K if wt == gguf.Q8_0 else None)


def _job_batch(m, rank, bar, a):
    """Sequences 0..S-1 from position 0, P prompt steps, then G greedy steps
    (fewer live sequences on the last steps: n shrinks to S-1)."""
    prompts = a["prompts"]
    S, P = len(prompts), len(prompts[0])
    m.set_batch(S)
    lg, out = None, []
    for p in range(P):
        lg = m.forward_batch([pr[p] for pr in prompts], [p] * S)
        out.append(lg)
    toks = [oracle.argmax(r) for r in lg]
    gen = [toks]
    for g in range(a["G"]):
        n = S if g < a["G"] - 1 else S - 1
        lg = m.forward_batch(toks[:n], [P + g] * n)
        out.append(np.concatenate([lg, np.zeros((S - n, lg.shape[1]), np.float32)]))
        toks = [oracle.argmax(r) for r in lg] + toks[n:]
        gen.append(toks)
    return np.stack(out), gen


def _job_prefill(m, rank, bar, a):
    last = m.prefill(a["prompt"], 0)
    t = oracle.argmax(last)
    nxt = m.forward_gpu(t, len(a["prompt"]))
    ppl = m.ctx.perplexity(a["ppl_tokens"])
    return last, nxt, ppl


def _job_timeout(m, rank, bar, a):
    """Rank 1 withholds a batched step, then a per-token step; rank 0's calls
    must fail with TALOS_ERR_TIMEOUT within the bound, and after a resync on
    both ranks the same steps match the oracle."""
    from talos_b200._lib import TalosError

    res = {}
    toks = a["toks"]
    m.set_batch(2)
    res["b0"] = m.forward_batch(toks[0], [0, 0])
    bar.wait(timeout=120)
    if rank == 0:
        t0 = time.time()
        try:
            m.forward_batch(toks[1], [1, 1])
            res["b_err"] = "no error"
        except TalosError as e:
            res["b_err"] = e.status
        res["b_secs"] = time.time() - t0
    bar.wait(timeout=120)
    m.ctx.tp_resync()
    bar.wait(timeout=120)
    res["b1"] = m.forward_batch(toks[1], [1, 1])
    # the per-token kernel: its in-kernel all-reduce waits for the peer as well
    res["t0"] = m.forward_gpu(toks[2], 0)
    bar.wait(timeout=120)
    if rank == 0:
        t0 = time.time()
        try:
            m.forward_gpu(toks[3], 1)
            res["t_err"] = "no error"
        except TalosError as e:
            res["t_err"] = e.status
        res["t_secs"] = time.time() - t0
    bar.wait(timeout=120)
    m.ctx.tp_resync()
    bar.wait(timeout=120)
    res["t1"] = m.forward_gpu(toks[3], 1)
    return res


def _job_greedy(m, rank, bar, a):
    """Prompts into the sequences' slots, then batched greedy on the device."""
    prompts = a["prompts"]
    m.set_batch(len(prompts))
    lasts = [m.ctx.prefill_slot(i, p, 0) for i, p in enumerate(prompts)]
    firsts = [oracle.argmax(x) for x in lasts]
    gen = m.ctx.generate_batch_greedy(firsts, [len(p) for p in prompts], a["G"])
    return np.stack(lasts), firsts, gen


JOBS = {"batch": _job_batch, "prefill": _job_prefill, "timeout": _job_timeout, "greedy": _job_greedy}


def _rank(rank, world, job, data, args, q_id, q_out, bar):
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
        out = JOBS[job](m, rank, bar, args)
        q_out.put((rank, out, None))
        m.close()
    except Exception:
        q_out.put((rank, None, traceback.format_exc()))


def run_job(job, data, args, world=2, timeout=300):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out, bar = ctx.Queue(), ctx.Queue(), ctx.Barrier(world)
    procs = [ctx.Process(target=_rank, args=(r, world, job, data, args, q_id, q_out, bar)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out, err = q_out.get(timeout=timeout)
            res[r] = (out, err)
    except _queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    assert len(res) == world, f"ranks answered: {sorted(res)}"
    for r, (_, err) in res.items():
        assert err is None, f"rank {r}: {err}"
    return [res[r][0] for r in range(world)]


def _oracle_seq(cpu, toks, pos0=0):
    return [cpu.forward(int(t), pos0 + i) for i, t in enumerate(toks)]


@pytest.mark.parametrize("wt", [gguf.Q4_0, gguf.Q8_0])
def test_tp2_batched_decode_matches_oracle(wt):
    data = _model(wt)
    S, P, G = 5, 4, 4
    prompts = [synth.token_ids(70 + i, P, SHAPE.vocab) for i in range(S)]
    ranks = run_job("batch", data, {"prompts": prompts, "G": G})
    (lg0, gen0), (lg1, gen1) = ranks
    assert np.array_equal(lg0, lg1), "ranks disagree on the gathered logits"
    assert gen0 == gen1
    cpu = oracle.Model(data=data)
    for i in range(S):
        cpu.reset()
        # the sequence's inputs: its prompt, then the tokens the GPU run chose
        n_live = G if i < S - 1 else G - 1
        feed = list(prompts[i]) + [gen0[g][i] for g in range(n_live)]
        ref = _oracle_seq(cpu, feed)
        for s, r in enumerate(ref):
            err = float(np.max(np.abs(lg0[s, i] - r)))
            assert err <= TOL, f"sequence {i} step {s}: {err:.3e}"
        # greedy choices equal the oracle's (sample::argmax, last maximum)
        for g in range(n_live):
            assert gen0[g][i] == oracle.argmax(ref[P - 1 + g])


def test_tp2_prefill_and_perplexity_match_oracle():
    data = _model(gguf.Q4_0)
    # 150 positions: a prefill step without logits, then one with them
    prompt = synth.token_ids(81, 150, SHAPE.vocab)
    ppl_toks = synth.token_ids(82, 300, SHAPE.vocab)  # chunks of the 256-position context
    ranks = run_job("prefill", data, {"prompt": prompt, "ppl_tokens": ppl_toks})
    cpu = oracle.Model(data=data)
    ref = _oracle_seq(cpu, prompt)[-1]
    t = oracle.argmax(ref)
    ref_next = cpu.forward(t, len(prompt))
    cpu.reset()
    want_ppl = oracle.perplexity(cpu, ppl_toks)
    for last, nxt, (ppl, nll, n) in ranks:
        assert np.max(np.abs(last - ref)) <= TOL
        assert np.max(np.abs(nxt - ref_next)) <= TOL
        assert n == 298  # chunks of 256 and 44 tokens score 255 + 43 positions
        assert abs(ppl - want_ppl) <= 1e-3 * want_ppl
    assert np.array_equal(ranks[0][0], ranks[1][0])


def test_tp2_withheld_step_times_out_and_resyncs():
    data = _model(gguf.Q4_0)
    V = SHAPE.vocab
    toks = [synth.token_ids(90, 2, V), synth.token_ids(91, 2, V), [int(synth.token_ids(92, 1, V)[0])],
            [int(synth.token_ids(93, 1, V)[0])]]
    args = {"toks": [toks[0], toks[1], toks[2][0], toks[3][0]]}
    r0, r1 = run_job("timeout", data, args)
    from talos_b200._lib import TIMEOUT

    assert r0["b_err"] == TIMEOUT, r0["b_err"]
    assert r0["t_err"] == TIMEOUT, r0["t_err"]
    assert r0["b_secs"] < 30 and r0["t_secs"] < 30, (r0["b_secs"], r0["t_secs"])
    cpu = oracle.Model(data=data)
    for i in range(2):
        cpu.reset()
        ref = _oracle_seq(cpu, [toks[0][i], toks[1][i]])
        for r in (r0, r1):
            assert np.max(np.abs(r["b0"][i] - ref[0])) <= TOL
            assert np.max(np.abs(r["b1"][i] - ref[1])) <= TOL
    cpu.reset()
    ref = _oracle_seq(cpu, [toks[2][0], toks[3][0]])
    for r in (r0, r1):
        assert np.max(np.abs(r["t0"] - ref[0])) <= TOL
        assert np.max(np.abs(r["t1"] - ref[1])) <= TOL


def test_tp2_prefill_slots_and_batch_greedy_match_oracle():
    data = _model(gguf.Q4_0)
    lens, G = [20, 3, 150, 9], 8  # 150: a fill step without logits, then one with them
    prompts = [synth.token_ids(100 + i, n, SHAPE.vocab) for i, n in enumerate(lens)]
    r0, r1 = run_job("greedy", data, {"prompts": prompts, "G": G})
    assert np.array_equal(r0[0], r1[0]) and np.array_equal(r0[2], r1[2]), "ranks disagree"
    cpu = oracle.Model(data=data)
    lasts, firsts, gen = r0
    for i, p in enumerate(prompts):
        cpu.reset()
        ref = _oracle_seq(cpu, p)[-1]
        assert np.max(np.abs(lasts[i] - ref)) <= TOL
        toks, t, pos = [], oracle.argmax(ref), len(p)
        for _ in range(G):
            toks.append(t)
            t = oracle.argmax(cpu.forward(t, pos))
            pos += 1
        assert [firsts[i]] + [int(x) for x in gen[:-1, i]] == toks, f"sequence {i}"
