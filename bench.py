#!/usr/bin/env python
"""Decode benchmark for the Talos B200 path (the Mistral-7B-shape Q4_0 model).

Workload: Mistral-7B-shaped Llama (d 4096, 32 layers, 32/8 heads, ff 14336,
vocab 32000, RoPE theta 1e6), random N(0, 0.02) weights from seed 1, Q4_0 with
output.weight in Q6_K; a 128-token uniform-random prompt (prefill, untimed),
then batch-1 greedy decode. One step = one decoded token.

  value : K greedy tokens decoded on the GPU with the argmax fed back on the
          device (talos_generate_greedy: one CUDA graph replay per token, i.e. one
          per-token kernel launch), timed with CUDA events on the context's
          stream. Weights (4.03 GB/token) are far larger than L2, so every step
          streams them from HBM.
  e2e   : the same decode through the public per-token call talos_forward with
          host buffers: token/pos host->device, logits device->host and the argmax
          on the host every step (the reference's decode loop, src/main.rs:97-113).
  roofline: the dominant kernel: the per-token kernel k_token (one launch = one
          token; algorithmic bytes = the token's weights + KV rows read), timed per
          launch with CUDA events (the layered graph's gate/up kernel when steps
          run the layered graph).
  cpu_baseline: the CPU oracle (a C restatement of the reference's rayon CPU
          forward) on this host's cores, a bounded sample of tokens.

--impl reference times that CPU path alone, per token, on the same workload.
Multi-GPU (torchrun, N > 1): tensor parallel over the N GPUs (one process per
GPU; heads, ff rows and vocab split, the all-reduce after o-proj and down runs
inside the per-token kernel over peer memory). All ranks decode the same single
sequence, so the work is fixed as N grows (strong scaling); value = tokens /
max over ranks of the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

# Algorithmic bytes of one decode token (7B shape): every matvec weight once
# (6,979,321,856 Q4_0 elements x 18/32 B), the Q6_K output (131,072,000 x 210/256),
# 65 f32 norm vectors, one Q4_0 embedding row.
W_BYTES_7B = 6979321856 * 18 // 32 + 131072000 * 210 // 256 + 65 * 4096 * 4 + 4096 // 32 * 18
KV_BYTES_PER_POS = 2 * 32 * 1024 * 4  # K and V rows read per cached position (f32)
GATEUP_BYTES = 2 * 14336 * 4096 * 18 // 32 + 4096 * 4 * 2 + 14336 * 4  # weights + x + norm + out
# DRAM bytes (read + write) of one k_token launch on the 7B shape, from the ncu
# capture summarised in profiles/k_token_m7b.md (a 2-layer capture scaled to 32
# layers: the output projection once plus 32 x the per-layer bytes).
K_TOKEN_TRAFFIC = 4_140_000_000
PROMPT_LEN = 128
MODEL_SEED = 1
PROMPT_SEED = 1


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def argmax_last(v: np.ndarray) -> int:
    """sample::argmax (src/sample.rs:7-14): last maximal element on ties."""
    return int(v.size - 1 - np.argmax(v[::-1]))


def bench_config(world: int, seq_len: int) -> dict:
    return {"workload": "mistral-7b-shape Q4_0 (+Q6_K output), 128-token prompt then batch-1 greedy decode",
            "model": "llama d4096 L32 h32/8 ff14336 V32000", "global_batch": 1, "seq_len": seq_len,
            "parallelism": f"tp{world}" if world > 1 else "1 GPU",
            "l2": "inputs larger than L2 (4.03 GB of weights per step)"}


def model_path() -> str:
    return os.environ.get("TALOS_BENCH_MODEL", f"/dev/shm/talos_bench_m7b_q4_0_s{MODEL_SEED}.gguf")


def ensure_model(path: str, threads: int | None = None) -> float:
    from talos_b200 import gguf, synth

    if os.path.exists(path) and os.path.getsize(path) > 4_000_000_000:
        return 0.0
    t = time.time()
    synth.write_llama(path + ".tmp", synth.MISTRAL_7B, MODEL_SEED, wtype=gguf.Q4_0, out_type=gguf.Q6_K,
                      threads=threads)
    os.replace(path + ".tmp", path)
    return time.time() - t


class ClockSampler:
    """SM clock and throttle reasons from NVML while the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock"}

    def __init__(self, device: int):
        self.samples, self.reasons, self.ok = [], set(), False
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[device]) if vis else device
            self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self._stop = threading.Event()
        self._th = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._th:
            self._th.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_decode(path: str, warmup: int, steps: int, budget_s: float):
    """The reference's decode loop (src/main.rs:88-113) through the oracle's CPU
    forward on all host threads: the 128-token prompt fed token by token
    (untimed), `warmup` greedy steps (untimed), then up to `steps` timed greedy
    steps, stopping early once `budget_s` seconds have passed. The timed steps sit
    at the positions the GPU arm times (PROMPT_LEN + warmup onwards). Returns
    (tok/s, steps timed, threads, seconds, first timed position)."""
    import oracle
    from talos_b200 import synth

    oracle.build()
    threads = max(1, len(os.sched_getaffinity(0)))
    oracle.set_threads(threads)
    m = oracle.Model(path=path)
    prompt = synth.token_ids(PROMPT_SEED, PROMPT_LEN, m.cfg.vocab_size)
    lg = None
    for i, t in enumerate(prompt):
        lg = m.forward(t, i)
    tok, pos = argmax_last(lg), PROMPT_LEN
    for _ in range(warmup):
        tok = argmax_last(m.forward(tok, pos))
        pos += 1
    pos0, n, t0 = pos, 0, time.perf_counter()
    while n < steps:
        tok = argmax_last(m.forward(tok, pos))
        pos += 1
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    m.close()
    return n / dt, n, threads, dt, pos0


def extra_configs(model, prompt) -> dict:
    """The other BASELINE configurations, measured on this GPU after the headline
    run (rank 0 of a one-GPU run only):
      c1_c2_tiny: the tiny Llama (seed 42) in F32 / Q8_0 / Q4_0, 64 greedy tokens
          on the device after a 16-token prompt (tok/s; the weights sit in L2);
      c3_matvec_4096: the 4096 x 4096 Q4_0 / Q8_0 fused dequant-matvec (seed 7,
          x ~ N(0, 1)), us and algorithmic GB/s with L2 defeated by rotating copies;
      prefill_128: this model's 128-token prompt through talos_prefill (the
          tensor-core GEMM path, 128 positions per weight pass), host wall clock;
      batch32: 32 sequences decoded together through talos_forward_batch (host
          logits every step), aggregate tok/s."""
    from talos_b200 import gguf, kbench

    out = {}
    out["c1_c2_tiny"] = {name: kbench.tiny_decode(t) for name, t in
                         (("f32", gguf.F32), ("q8_0", gguf.Q8_0), ("q4_0", gguf.Q4_0))}
    out["c3_matvec_4096"] = {t: {k: v for k, v in kbench.matvec_bench(t, 4096, 4096).items()
                                 if k in ("us_per_matvec", "gbs", "copies", "algo_bytes")}
                             for t in ("q4_0", "q8_0")}
    best = 1e9
    for _ in range(3):
        t0 = time.perf_counter()
        model.prefill(prompt, 0)
        best = min(best, time.perf_counter() - t0)
    out["prefill_128"] = {"ms": best * 1e3, "tok_s": len(prompt) / best, "path": "tcgen05 GEMM, 128 positions per step"}
    nb, vocab = 32, model.cfg.vocab_size
    model.ctx.set_batch(nb)
    toks = synth_ids(nb, vocab)
    # each sequence at its own position: 13 steps from positions spread over 32
    # below the end of the context the model was loaded with (around the prompt)
    top = min(PROMPT_LEN + 32, model.cfg.context_length - 14)
    pos = [top - 32 + (7 * i) % 32 for i in range(nb)]
    for i in range(3):
        model.ctx.forward_batch(toks, [p + i for p in pos])
    steps, t0 = 10, time.perf_counter()
    for i in range(steps):
        lg = model.ctx.forward_batch(toks, [p + 3 + i for p in pos])
        toks = [argmax_last(r) for r in lg]
    dt = (time.perf_counter() - t0) / steps
    model.ctx.set_batch(0)
    out["batch32"] = {"seqs": nb, "ms_per_step": dt * 1e3, "tok_s": nb / dt,
                      "path": "tcgen05 GEMM, host logits every step"}
    return out


def synth_ids(n: int, vocab: int) -> list[int]:
    from talos_b200 import synth

    return synth.token_ids(3, n, vocab)


def run_reference(args):
    """--impl reference: the CPU restatement of the reference's forward on this
    host's cores, on the GPU arm's workload: the same 128-token prompt (fed
    untimed), the same warm-up steps, then timed greedy decode steps at the same
    positions."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    ensure_model(model_path())
    budget = float(os.environ.get("TALOS_REF_BUDGET_S", "150"))
    v, n, threads, dt, pos0 = cpu_decode(model_path(), args.warmup, args.steps, budget)
    sample = (f"128-token prompt fed untimed, {args.warmup} untimed greedy steps, then {n} timed greedy decode "
              f"tokens (positions {pos0}..{pos0 + n - 1}) of the 7B-shape Q4_0/Q6_K model, {threads} threads; "
              f"timed steps capped at {budget:.0f} s of CPU time")
    line = {
        "metric": "decode tok/s (batch 1, 7B-shape Q4_0)", "value": v, "unit": "tok/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": n, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * dt / max(n, 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q4_0 weights, f32 activations/KV", "data": "synthetic",
        "config": bench_config(args.gpus, PROMPT_LEN + args.warmup + args.steps),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="talos_b200", choices=["talos_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the other BASELINE configurations")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)

    from talos_b200 import Model, build, synth

    build.build()
    path = model_path()
    gen_s = 0.0
    if local == 0:
        gen_s = ensure_model(path)
    if dist:
        dist.barrier()

    K, W = args.steps, args.warmup
    uid = None
    if world > 1:  # rank 0's NCCL id bootstraps the tensor-parallel contexts
        from talos_b200 import nccl_unique_id

        t = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(t, src=0)
        uid = bytes(t.cpu().numpy().tobytes())
    t_load = time.time()
    model = Model.load(path, device=local, max_ctx=PROMPT_LEN + 2 * (K + W) + 16, tp_size=world, tp_rank=rank,
                       nccl_id=uid)
    load_s = time.time() - t_load
    ctx = model.ctx
    stream = torch.cuda.ExternalStream(ctx.stream(), device=torch.device("cuda", local))
    vocab = model.cfg.vocab_size
    prompt = synth.token_ids(PROMPT_SEED, PROMPT_LEN, vocab)

    # ---------------- device-resident greedy decode (value)
    last = model.prefill(prompt, 0)
    tok = argmax_last(last)
    pos = PROMPT_LEN
    out = model.generate_greedy(tok, pos, W)
    tok, pos = int(out[-1]), pos + W
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with clocks:
        e0.record(stream)
        out = model.generate_greedy(tok, pos, K)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = K / (ms / 1000.0)
    tok, pos = int(out[-1]), pos + K
    kv_avg_pos = PROMPT_LEN + W + K / 2

    # ---------------- end to end through talos_forward with host buffers (e2e)
    logits = np.empty(vocab, np.float32)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        ctx.forward(tok, pos, logits)
        tok = argmax_last(logits)
        pos += 1
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = K / e2e_s

    # ---------------- per-kernel times of eagerly launched steps (roofline)
    n_prof = 4
    tot_ms, tot_n = None, None
    for i in range(n_prof):
        ms_k, n_k = ctx.profile_step(tok, PROMPT_LEN + W + i)
        if tot_ms is None:
            tot_ms, tot_n = ms_k, n_k
        else:
            for k in tot_ms:
                tot_ms[k] += ms_k[k]
                tot_n[k] += n_k[k]
    peak, peak_kind = measured_peaks()
    step_kernel = ctx.step_kernel()
    step_ms = sum(tot_ms.values()) / n_prof
    breakdown = {k: {"ms_per_step": tot_ms[k] / n_prof, "count_per_step": tot_n[k] // n_prof}
                 for k in tot_ms}
    if step_kernel == "fused":
        # the dominant (only) kernel is k_token: one launch = one whole token
        prof_pos = PROMPT_LEN + W + (n_prof - 1) / 2
        dom_bytes = W_BYTES_7B + KV_BYTES_PER_POS * (prof_pos + 1)
        dom_ms = step_ms
        dom_name = "k_token (whole decode step: 32 layers + output, one launch)"
        traffic = K_TOKEN_TRAFFIC
        launches = 2  # k_token + the greedy-advance kernel
    else:
        dom_bytes = GATEUP_BYTES
        dom_ms = tot_ms["gateup"] / max(tot_n["gateup"], 1)
        dom_name = "gateup (RMSNorm + gate/up Q4_0 matvec + SwiGLU)"
        traffic = None  # no ncu capture of the layered graph's gate/up kernel
        launches = sum(tot_n.values()) // n_prof + 1  # + the greedy-advance kernel
    achieved = dom_bytes / (dom_ms / 1000.0) / 1e9

    # ---------------- the other BASELINE configurations (rank 0 at N=1 only)
    configs = extra_configs(model, prompt) if world == 1 and not args.no_extra else None

    # ---------------- CPU baseline (rank 0 at N=1 only)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, n, thr, dt, p0 = cpu_decode(path, W, min(K, 12), budget_s=20.0)
        cpu = {"value": v, "unit": "tok/s", "cores": thr, "kind": "port",
               "sample": f"128-token prompt and {W} greedy steps untimed, then {n} timed greedy decode tokens "
                         f"(positions {p0}..{p0 + n - 1}, the GPU arm's first timed positions) of the same "
                         f"7B-shape model through the oracle's CPU forward, {dt:.1f} s"}

    tok_bytes = W_BYTES_7B + KV_BYTES_PER_POS * kv_avg_pos
    ms_step = ms / K
    line = {
        "metric": "decode tok/s (batch 1, 7B-shape Q4_0)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_0 weights, f32 activations/KV", "data": "synthetic",
        "config": bench_config(world, PROMPT_LEN + W + K),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 24, "d2h_bytes_per_step": vocab * 4 + 24},
        "roofline": {"bound": "hbm", "kernel": dom_name,
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "traffic": traffic, "bytes_per_launch": dom_bytes,
                     "ms_per_launch": dom_ms},
        "token_roofline": {"bytes_per_token": tok_bytes, "achieved_gbs": tok_bytes / (ms_step / 1000) / 1e9,
                           "frac": tok_bytes / (ms_step / 1000) / 1e9 / peak, "peak_kind": peak_kind},
        "step_kernel": step_kernel, "parts": breakdown, "profiled_step_ms": step_ms,
        "gpu_launches": launches * K,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "configs": configs,
        "setup": {"model_gen_s": gen_s, "load_s": load_s},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
