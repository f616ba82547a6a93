"""Single-kernel microbenchmark of the fused dequant-matvec.

    python -m talos_b200.kbench [--type q4_0|q8_0|q6_k|f32] [--rows R] [--cols C]
                                [--copies N] [--reps K] [--warmup W]

Packs N distinct copies of a seeded N(0, 0.02) weight [R, C] (N chosen so that
together they exceed twice the L2), then times K launches of talos_matvec_dev
cycling through the copies, with CUDA events on one stream. Reports microseconds
per matvec and algorithmic GB/s (packed weight bytes + x + y per launch).
Default: the 4096 x 4096 Q4_0 microbench, seed 7, x ~ N(0, 1).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

TYPES = {"f32": 0, "q4_0": 2, "q8_0": 8, "q6_k": 14}
ALGO_BYTES_PER_ELEM = {0: 4.0, 2: 18 / 32, 8: 34 / 32, 14: 210 / 256}


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
    a = ap.parse_args(argv)

    import torch

    from talos_b200 import build, model, synth

    build.build()
    gt = TYPES[a.type]
    torch.cuda.set_device(a.device)
    raw = synth.tensor(a.seed, "bench.w", a.rows, a.cols, gt)
    x = synth.normal(a.seed, "bench.x", a.cols, 1.0)
    l2 = torch.cuda.get_device_properties(a.device).L2_cache_size
    copies = a.copies or max(2, int(np.ceil(2 * l2 / raw.nbytes)) + 1)
    ws = [model.Weight(gt, raw, a.rows, a.cols, a.device) for _ in range(copies)]
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(a.rows, device="cuda")
    # talos_matvec_bench captures the launches into one CUDA graph and times a
    # replay with CUDA events, so the host's per-call cost is not measured.
    import ctypes as C

    from talos_b200 import _lib

    torch.cuda.synchronize()
    arr = (C.c_void_p * copies)(*[w.h.value for w in ws])
    us_c = C.c_float()
    _lib.check(_lib.load().talos_matvec_bench(arr, copies, C.c_void_p(xd.data_ptr()), C.c_void_p(yd.data_ptr()),
                                              a.reps, C.byref(us_c)))
    us = float(us_c.value)
    algo = a.rows * a.cols * ALGO_BYTES_PER_ELEM[gt] + 4 * (a.rows + a.cols)
    out = {"kernel": f"matvec_{a.type}", "rows": a.rows, "cols": a.cols, "copies": copies,
           "l2_bytes": l2, "us_per_matvec": us, "algo_bytes": algo, "gbs": algo / (us * 1e-6) / 1e9,
           "packed_bytes": ws[0].packed_bytes()}
    print(json.dumps(out), flush=True)
    for w in ws:
        w.close()
    return 0


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.exit(main())
