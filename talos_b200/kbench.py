"""Kernel microbenchmarks.

Matvec microbenchmark:

    python -m talos_b200.kbench [--type q4_0|q8_0|q6_k|f32] [--rows R] [--cols C]
                                [--copies N] [--reps K] [--warmup W]

Packs N distinct copies of a seeded N(0, 0.02) weight [R, C] (N chosen so that
together they exceed twice the L2), then times K graph-captured launches of
talos_matvec_dev cycling through the copies. Reports microseconds per matvec
and algorithmic GB/s (packed weight bytes + x + y per launch). Default: the
4096 x 4096 Q4_0 microbench, seed 7, x ~ N(0, 1).

Decode step on a reduced-depth model (a small case of the same kernels, for
profiling; its weights still exceed the L2):

    python -m talos_b200.kbench --step [--layers L] [--steps K] [--step-kernel fused|layered]

builds the Mistral-7B shape (seed 1, Q4_0, Q6_K output) with L layers, feeds a
16-token prompt and times K device-side greedy steps.

Prefill on the same model (one batched tensor-core pass per 128 positions):

    python -m talos_b200.kbench --prefill N [--layers L] [--steps K]

times K talos_prefill calls of an N-token prompt at position 0 (CUDA events).

Batched decode on the same model:

    python -m talos_b200.kbench --batch N [--layers L] [--steps K]

times K talos_forward_batch steps of N sequences (each at its own position,
host logits out, wall clock per call) and reports the aggregate tokens/s.

The Llama-3-70B shape (the 70B benchmark model: all Q4_0, seed 3) on one GPU:

    python -m talos_b200.kbench --llama70b [--model-dir DIR]

writes the 39.7 GB GGUF file to DIR (default /dev/shm; about 95 s), loads it,
times a 32-token prefill, the per-token decode (device greedy loop, best of
3 x 48 tokens) and 12 batched steps of 4 sequences, then deletes the file.

Per-phase times of the per-token kernel, on 1, 2, 4 or 8 GPUs (tensor parallel):

    python -m talos_b200.kbench --phases --tp N [--layers L]

loads the 7B shape with L layers (default 4) on every rank, feeds a 16-token
prompt, and reads the kernel's device-timer stamps (talos_profile_phases) of
three steps: per phase kind the median over CTAs, layers and steps of the
input staging, the compute, the epilogue tail up to the CTA's arrival, and the
wait from the arrival to the next phase's start (the grid barrier; after the
o-proj and down phases under tensor parallelism the cross-rank barrier).

The 70B multi-prompt workload (32 sequences, each a 512-token uniform-random
prompt then 128 greedy tokens) on 1, 2, 4 or 8 GPUs, one process per GPU:

    python -m talos_b200.kbench --config5 --tp N [--seqs 32] [--prompt 512] [--gen 128]
                                [--model-dir DIR] [--layers L]

writes the same model file (kept when it exists; --layers L for a reduced
depth), loads it on every rank with a context of prompt + gen positions,
prefills each sequence's slot (talos_prefill_slot) and runs the greedy tokens
of all sequences together (talos_generate_batch_greedy). Both phases are timed
with CUDA events on each rank's context stream; the reported time is the max
over ranks. Reports tok/s and, for the decode, the fraction of the measured HBM
copy bandwidth that the bytes each rank must read per step (its weight shard
and its KV rows) need at that rate.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

TYPES = {"f32": 0, "q4_0": 2, "q8_0": 8, "q6_k": 14}
ALGO_BYTES_PER_ELEM = {0: 4.0, 2: 18 / 32, 8: 34 / 32, 14: 210 / 256}


def argmax_last(v) -> int:
    """sample::argmax (src/sample.rs:7-14): the last maximal element on ties."""
    v = np.asarray(v)
    return int(v.size - 1 - np.argmax(v[::-1]))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--type", default="q4_0", choices=sorted(TYPES))
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--copies", type=int, default=0)
    ap.add_argument("--reps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--step", action="store_true")
    ap.add_argument("--layers", type=int, default=None)  # --step / --batch: 2; --config5: 80
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--step-kernel", default="auto", choices=["auto", "fused", "layered"])
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--prefill", type=int, default=0)
    ap.add_argument("--llama70b", action="store_true")
    ap.add_argument("--model-dir", default="/dev/shm")
    ap.add_argument("--config5", action="store_true")
    ap.add_argument("--phases", action="store_true")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--seqs", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=128)
    a = ap.parse_args(argv)
    if a.config5:
        return config5_bench(a)
    if a.phases:
        return phases_bench(a)
    if a.llama70b:
        return llama70b_bench(a)
    if a.batch:
        return batch_bench(a)
    if a.prefill:
        return prefill_bench(a)
    if a.step:
        return step_bench(a)

    from talos_b200 import build

    build.build()
    print(json.dumps(matvec_bench(a.type, a.rows, a.cols, a.seed, a.reps, a.copies, a.device)), flush=True)
    return 0


def matvec_bench(type_name: str, rows: int, cols: int, seed: int = 7, reps: int = 200, copies: int = 0,
                 device: int = 0) -> dict:
    """a seeded N(0, 0.02) [rows, cols] weight of `type_name`
    and x ~ N(0, 1); `copies` packed copies (enough to exceed twice the L2 when
    0), cycled through by `reps` graph-captured talos_matvec_dev launches timed
    with CUDA events. Returns microseconds per matvec and algorithmic GB/s
    (weight bytes in the GGUF format + x + y)."""
    import ctypes as C

    import torch

    from talos_b200 import _lib, model, synth

    gt = TYPES[type_name]
    torch.cuda.set_device(device)
    raw = synth.tensor(seed, "bench.w", rows, cols, gt)
    x = synth.normal(seed, "bench.x", cols, 1.0)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    copies = copies or max(2, int(np.ceil(2 * l2 / raw.nbytes)) + 1)
    ws = [model.Weight(gt, raw, rows, cols, device) for _ in range(copies)]
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(rows, device="cuda")
    # talos_matvec_bench captures the launches into one CUDA graph and times a
    # replay with CUDA events, so the host's per-call cost is not measured.
    torch.cuda.synchronize()
    arr = (C.c_void_p * copies)(*[w.h.value for w in ws])
    us_c = C.c_float()
    _lib.check(_lib.load().talos_matvec_bench(arr, copies, C.c_void_p(xd.data_ptr()), C.c_void_p(yd.data_ptr()),
                                              reps, C.byref(us_c)))
    us = float(us_c.value)
    algo = rows * cols * ALGO_BYTES_PER_ELEM[gt] + 4 * (rows + cols)
    out = {"kernel": f"matvec_{type_name}", "rows": rows, "cols": cols, "copies": copies,
           "l2_bytes": l2, "us_per_matvec": us, "algo_bytes": algo, "gbs": algo / (us * 1e-6) / 1e9,
           "packed_bytes": ws[0].packed_bytes()}
    for w in ws:
        w.close()
    return out


def tiny_decode(wtype: int, device: int = 0) -> dict:
    """BASELINE configs 1 / 2: the tiny Llama (seed 42) with every 2-D weight in
    `wtype`, a 16-token prompt, then 64 greedy tokens decoded on the device
    (talos_generate_greedy), timed with CUDA events. The weights sit in L2
    (26 MB at most), so the step is latency-bound."""
    import torch

    from talos_b200 import Model, synth

    m = Model.load_bytes(synth.llama_bytes(synth.TINY, 42, wtype=wtype), device=device)
    prompt = synth.token_ids(42, 16, synth.TINY.vocab)
    tok = argmax_last(m.prefill(prompt, 0))
    m.generate_greedy(tok, 16, 8)  # warm-up (graph capture)
    stream = torch.cuda.ExternalStream(m.ctx.stream(), device=torch.device("cuda", device))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    m.generate_greedy(tok, 16, 64)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    m.close()
    return {"tokens": 64, "ms": ms, "tok_s": 64 / (ms / 1e3), "step_kernel": "fused"}


def step_bench(a) -> int:
    import dataclasses
    import time

    import torch

    from talos_b200 import Model, build, gguf, synth

    build.build()
    torch.cuda.set_device(a.device)
    layers = a.layers or 2
    shape = dataclasses.replace(synth.MISTRAL_7B, n_layer=layers, ctx=64)
    t0 = time.time()
    data = synth.llama_bytes(shape, 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    gen_s = time.time() - t0
    m = Model.load_bytes(data, device=a.device, step_kernel=a.step_kernel)
    del data
    prompt = synth.token_ids(1, 16, shape.vocab)
    last = m.prefill(prompt, 0)
    tok = argmax_last(last)
    m.generate_greedy(tok, 16, 2)
    stream = torch.cuda.ExternalStream(m.ctx.stream(), device=torch.device("cuda", a.device))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    m.generate_greedy(tok, 18, a.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    E, F, V = shape.n_embd, shape.n_ff, shape.vocab
    wbytes = layers * (2 * E * E + 2 * shape.kv_dim * E + 3 * E * F) * 18 // 32 + V * E * 210 // 256
    out = {"kernel": "decode_step", "step_kernel": m.ctx.step_kernel(), "layers": layers,
           "ms_per_step": ms, "weight_bytes": wbytes, "gbs": wbytes / (ms * 1e-3) / 1e9, "model_gen_s": gen_s}
    print(json.dumps(out), flush=True)
    m.close()
    return 0


def prefill_bench(a) -> int:
    import dataclasses

    import torch

    from talos_b200 import Model, build, gguf, synth

    build.build()
    torch.cuda.set_device(a.device)
    layers = a.layers or 2
    shape = dataclasses.replace(synth.MISTRAL_7B, n_layer=layers, ctx=max(256, a.prefill))
    data = synth.llama_bytes(shape, 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    m = Model.load_bytes(data, device=a.device, max_ctx=max(256, a.prefill))
    del data
    prompt = synth.token_ids(1, a.prefill, shape.vocab)
    m.prefill(prompt, 0)  # warm-up (graph capture)
    stream = torch.cuda.ExternalStream(m.ctx.stream(), device=torch.device("cuda", a.device))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        m.prefill(prompt, 0)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    E, F, V = shape.n_embd, shape.n_ff, shape.vocab
    params = layers * (2 * E * E + 2 * shape.kv_dim * E + 3 * E * F)
    out = {"kernel": "prefill", "layers": layers, "tokens": a.prefill, "ms": ms, "tok_s": a.prefill / (ms * 1e-3),
           "useful_tflops_layers": 2.0 * params * a.prefill / (ms * 1e-3) / 1e12}
    print(json.dumps(out), flush=True)
    m.close()
    return 0


def batch_bench(a) -> int:
    import dataclasses
    import time

    from talos_b200 import Model, build, gguf, synth

    build.build()
    shape = dataclasses.replace(synth.MISTRAL_7B, n_layer=a.layers or 2, ctx=1024)
    data = synth.llama_bytes(shape, 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    m = Model.load_bytes(data, device=a.device, max_ctx=1024)
    del data
    m.ctx.set_batch(a.batch)
    toks = synth.token_ids(3, a.batch, shape.vocab)
    pos = [128 + 17 * i for i in range(a.batch)]
    for i in range(3):
        m.ctx.forward_batch(toks, [p + i for p in pos])
    t0 = time.perf_counter()
    for i in range(a.steps):
        lg = m.ctx.forward_batch(toks, [p + 3 + i for p in pos])
        toks = [argmax_last(r) for r in lg]
    dt = time.perf_counter() - t0
    out = {"kernel": "decode_batch", "batch": a.batch, "layers": a.layers or 2, "steps": a.steps,
           "ms_per_step": dt / a.steps * 1e3, "tok_s": a.batch * a.steps / dt}
    print(json.dumps(out), flush=True)
    m.close()
    return 0


def llama70b_bench(a) -> int:
    import shutil
    import time

    from talos_b200 import Model, build, gguf, synth

    build.build()
    if shutil.disk_usage(a.model_dir).free < 42e9:
        print(json.dumps({"kernel": "decode_70b", "skipped": f"under 42 GB free in {a.model_dir}"}))
        return 0
    path = os.path.join(a.model_dir, "talos_kbench_llama70b_q4_0.gguf")
    shape = synth.with_ctx(synth.LLAMA3_70B, 1024)
    t = time.time()
    synth.write_llama(path, shape, 3, wtype=gguf.Q4_0)
    gen = time.time() - t
    try:
        t = time.time()
        m = Model.load(path, device=a.device, max_ctx=1024)
        load = time.time() - t
        prompt = synth.token_ids(3, 32, shape.vocab)
        t = time.perf_counter()
        last = m.prefill(prompt, 0)
        pf = time.perf_counter() - t
        tok = argmax_last(last)
        m.generate_greedy(tok, 32, 4)
        best = 1e9
        for _ in range(3):
            t = time.perf_counter()
            m.generate_greedy(tok, 36, 48)
            best = min(best, (time.perf_counter() - t) / 48)
        algo = 39_099_994_624  # weight bytes per token (all Q4_0 matrices + norms + one embedding row)
        m.ctx.set_batch(4)
        toks, pos = [1, 2, 3, 4], [100, 200, 300, 400]
        for i in range(2):
            m.ctx.forward_batch(toks, [p + i for p in pos])
        t = time.perf_counter()
        for i in range(12):
            lg = m.ctx.forward_batch(toks, [p + 2 + i for p in pos])
            toks = [argmax_last(r) for r in lg]
        bt = (time.perf_counter() - t) / 12
        m.close()
    finally:
        os.remove(path)
    out = {"kernel": "decode_70b", "step_kernel": "fused", "model_gen_s": gen, "load_s": load,
           "prefill_32_ms": pf * 1e3, "decode_ms_per_token": best * 1e3, "decode_tok_s": 1 / best,
           "algo_gbs": algo / best / 1e9, "batch4_ms_per_step": bt * 1e3, "batch4_tok_s": 4 / bt}
    print(json.dumps(out), flush=True)
    return 0


def _c5_rank(rank, tp, path, a, q_id, q_out):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch

        from talos_b200 import Model, nccl_unique_id, synth

        torch.cuda.set_device(rank)
        kw = {}
        if tp > 1:
            if rank == 0:
                uid = nccl_unique_id()
                for _ in range(tp - 1):
                    q_id.put(uid)
            else:
                uid = q_id.get(timeout=600)
            kw = dict(tp_size=tp, tp_rank=rank, nccl_id=uid)
        m = Model.load(path, device=rank, max_ctx=a.prompt + a.gen, **kw)
        V = m.ctx.cfg.vocab_size
        prompts = [synth.token_ids(3 + i, a.prompt, V) for i in range(a.seqs)]
        m.set_batch(a.seqs)
        stream = torch.cuda.ExternalStream(m.ctx.stream(), device=torch.device("cuda", rank))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        # warm-up: one sequence's prompt and two greedy steps (graph capture)
        m.ctx.prefill_slot(0, prompts[0][:256], 0, want_logits=True)
        m.ctx.generate_batch_greedy([1] * a.seqs, [256] * a.seqs, 2)
        torch.cuda.synchronize()
        ev[0].record(stream)
        firsts = [argmax_last(m.ctx.prefill_slot(i, p, 0)) for i, p in enumerate(prompts)]
        ev[1].record(stream)
        ev[2].record(stream)
        gen = m.ctx.generate_batch_greedy(firsts, [a.prompt] * a.seqs, a.gen)
        ev[3].record(stream)
        torch.cuda.synchronize()
        q_out.put((rank, ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3]), gen[:, :4].tolist(), None))
        m.close()
    except Exception:
        import traceback

        q_out.put((rank, None, None, None, traceback.format_exc()))


PHASE_KINDS = ("qkv", "attn", "oproj", "gateup", "down")


def _ph_rank(rank, tp, data, layers, q_id, q_out):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch

        from talos_b200 import Model, nccl_unique_id, synth

        torch.cuda.set_device(rank)
        kw = {}
        if tp > 1:
            if rank == 0:
                uid = nccl_unique_id()
                for _ in range(tp - 1):
                    q_id.put(uid)
            else:
                uid = q_id.get(timeout=600)
            kw = dict(tp_size=tp, tp_rank=rank, nccl_id=uid)
        m = Model.load_bytes(data, device=rank, **kw)
        V = m.ctx.cfg.vocab_size
        toks = synth.token_ids(1, 16, V)
        for p, t in enumerate(toks):
            m.forward_gpu(int(t), p)
        runs = []
        for i in range(5):
            st = m.ctx.profile_phases(int(toks[i]), 16 + i)
            if i >= 2:
                runs.append(st.astype(np.int64))
        q_out.put((rank, runs, None))
        m.close()
    except Exception:
        import traceback

        q_out.put((rank, None, traceback.format_exc()))


def phases_bench(a) -> int:
    import dataclasses
    import multiprocessing as mp

    from talos_b200 import build, gguf, synth

    build.build()
    layers = a.layers or 4
    shape = dataclasses.replace(synth.MISTRAL_7B, n_layer=layers, ctx=64)
    data = synth.llama_bytes(shape, 1, wtype=gguf.Q4_0, out_type=gguf.Q6_K)
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ph_rank, args=(r, a.tp, data, layers, q_id, q_out)) for r in range(a.tp)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(a.tp):
        r, runs, err = q_out.get(timeout=1800)
        res[r] = (runs, err)
    for p in procs:
        p.join(timeout=120)
    errs = {r: v[1] for r, v in res.items() if v[1]}
    if errs:
        print(json.dumps({"kernel": "phases", "tp": a.tp, "error": errs}))
        return 1
    out = {"kernel": "phases", "tp": a.tp, "layers": layers, "position": "16-18", "per_layer_us": {}}
    runs = res[0][0]
    parts = {k: {"staging": [], "compute": [], "tail": [], "wait": []} for k in PHASE_KINDS}
    for st in runs:  # [phase][cta][4] ns: entered, staged, computed, arrived
        nph = st.shape[0]
        for p in range(min(nph - 1, 5 * layers)):
            kind = PHASE_KINDS[p % 5]
            e, s_, c, ar = (st[p, :, k] for k in range(4))
            nxt = st[p + 1, :, 0]
            ok = lambda x, y: (x > 0) & (y > 0)
            for name, x, y in (("staging", e, s_), ("compute", s_, c), ("tail", c, ar), ("wait", ar, nxt)):
                m = ok(x, y)
                if m.any():
                    parts[kind][name].append(float(np.median((y - x)[m])) / 1e3)
    total = 0.0
    for k in PHASE_KINDS:
        d = {n: (round(float(np.median(v)), 2) if v else None) for n, v in parts[k].items()}
        out["per_layer_us"][k] = d
        total += sum(x for x in d.values() if x)
    out["layer_us"] = round(total, 1)
    print(json.dumps(out), flush=True)
    return 0


def config5_bench(a) -> int:
    import dataclasses
    import multiprocessing as mp
    import shutil
    import time

    from talos_b200 import build, gguf, synth

    build.build()
    shape = dataclasses.replace(synth.LLAMA3_70B, n_layer=a.layers or 80)
    path = os.path.join(a.model_dir, f"talos_kbench_llama70b_{shape.n_layer}l_q4_0.gguf")
    gen_s = 0.0
    if not os.path.exists(path):
        need = 42e9 * shape.n_layer / 80
        if shutil.disk_usage(a.model_dir).free < need:
            print(json.dumps({"kernel": "config5", "skipped": f"under {need / 1e9:.0f} GB free in {a.model_dir}"}))
            return 0
        t = time.time()
        synth.write_llama(path + ".tmp", shape, 3, wtype=gguf.Q4_0)
        os.replace(path + ".tmp", path)
        gen_s = time.time() - t
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_c5_rank, args=(r, a.tp, path, a, q_id, q_out)) for r in range(a.tp)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(a.tp):
        r, pf, dc, toks, err = q_out.get(timeout=3600)
        res[r] = (pf, dc, toks, err)
    for p in procs:
        p.join(timeout=120)
    errs = {r: v[3] for r, v in res.items() if v[3]}
    if errs:
        print(json.dumps({"kernel": "config5", "tp": a.tp, "error": errs}))
        return 1
    pf = max(v[0] for v in res.values()) / 1e3
    dc = max(v[1] for v in res.values()) / 1e3
    agree = all(v[2] == res[0][2] for v in res.values())
    E, F, V, L = shape.n_embd, shape.n_ff, shape.vocab, shape.n_layer
    kv = shape.n_head_kv * (E // shape.n_head)
    # bytes one rank reads per decode step: its Q4_0 shard of every matrix and
    # of the output, plus its KV rows of every sequence at the step's positions
    w_rank = (L * (2 * E * E + 2 * kv * E + 3 * E * F) + V * E) * 18 // 32 / a.tp
    mean_pos = a.prompt + (a.gen + 1) / 2
    kv_rank = a.seqs * mean_pos * L * (kv / a.tp) * 4 * 2
    step_s = dc / a.gen
    peak = None
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                               "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["hbm_gbs"])
    except Exception:
        peak = 6650.0
    gbs = (w_rank + kv_rank) / step_s / 1e9
    out = {"kernel": "config5", "model": f"llama3-70b-shape ({L} layers) q4_0 seed 3", "tp": a.tp,
           "seqs": a.seqs, "prompt": a.prompt, "gen": a.gen, "model_gen_s": round(gen_s, 1),
           "prefill_s": pf, "prefill_tok_s": a.seqs * a.prompt / pf,
           "decode_s": dc, "decode_tok_s": a.seqs * a.gen / dc, "decode_ms_per_step": step_s * 1e3,
           "decode_bytes_per_rank_step": w_rank + kv_rank, "decode_gbs_per_rank": gbs,
           "decode_frac_of_measured_hbm": gbs / peak, "ranks_agree": agree, "first_tokens": res[0][2][:2]}
    print(json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.exit(main())
