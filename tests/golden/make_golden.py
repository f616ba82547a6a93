"""Generate the golden fixtures under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

The oracle is the C restatement of the reference's CPU path (oracle/), pinned by
the reference's own known-answer tests (tests/test_oracle_kat.py). The reference
itself (Rust) cannot be built in this image, so these fixtures are oracle
outputs; they freeze the oracle's answers so that the GPU tests compare against
fixed numbers and the CPU suite notices any drift of the oracle or of the
synthetic-input generator (each fixture stores the sha256 of its input bytes).

Fixtures (all inputs are regenerated from seeds, only outputs are stored):
  tiny_{f32,q8_0,q4_0}.npz   the tiny Llama benchmark models, seed 42, 16-token
                             prompt (seed 42), 64 greedy tokens, logits after the
                             prompt and after the last greedy step.
  matvec4096_{q4_0,q8_0}.npz config 3: 4096x4096 N(0,0.02) seed 7, x N(0,1);
                             y = W x and the dequantized first two rows.
  dequant_blocks.npz         seeded random blocks of every format (with the
                             edge scales 0, subnormal, max, -0, inf, nan) and
                             their dequantized values.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

N_PROMPT, N_GEN = 16, 64
TINY_TYPES = {"f32": 0, "q8_0": 8, "q4_0": 2}
MV_TYPES = {"q4_0": 2, "q8_0": 8}
BLOCK = {0: (4, 1), 2: (18, 32), 8: (34, 32), 14: (210, 256)}  # bytes, elements per block
EDGE_F16 = [0x0000, 0x0001, 0x03FF, 0x7BFF, 0x8000, 0x7C00, 0x7E00, 0xFBFF]


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def tiny_case(wtype: int):
    """Prompt + greedy run of the oracle; returns the fixture dict."""
    import oracle
    from tests.helpers import prompt, tiny_model

    data = tiny_model(wtype)
    m = oracle.Model(data=data)
    vocab = m.cfg.vocab_size
    toks = prompt(N_PROMPT, vocab, 42)
    pos = 0
    for t in toks:
        lg = m.forward(t, pos)
        pos += 1
    first = lg.copy()
    gen = []
    for _ in range(N_GEN):
        t = oracle.argmax(lg)
        gen.append(t)
        lg = m.forward(t, pos)
        pos += 1
    m.close()
    return dict(model_sha=np.array(sha(data)), prompt=np.array(toks, np.uint32), tokens=np.array(gen, np.uint32),
                logits_prompt=first.astype(np.float32), logits_last=lg.astype(np.float32))


def matvec_case(gtype: int):
    import oracle
    from talos_b200 import synth

    raw = synth.tensor(7, "bench.w", 4096, 4096, gtype)
    x = synth.normal(7, "bench.x", 4096, 1.0)
    y = oracle.matvec_quant(raw, gtype, x, 4096, 4096)
    bpr = raw.nbytes // 4096
    d2 = oracle.dequant(gtype, raw[:2 * bpr], 2 * 4096)
    return dict(w_sha=np.array(sha(raw.tobytes())), x_sha=np.array(sha(x.tobytes())), y=y.astype(np.float32),
                dequant_rows01=d2.astype(np.float32))


def random_blocks(gtype: int, n_blocks: int, rng) -> np.ndarray:
    """Random bytes per block with an f16 scale from EDGE_F16 or a normal value."""
    nb, _ = BLOCK[gtype]
    raw = rng.integers(0, 256, size=(n_blocks, nb), dtype=np.uint8)
    if gtype == 0:
        return raw.reshape(-1)
    off = 208 if gtype == 14 else 0
    for i in range(n_blocks):
        h = EDGE_F16[i] if i < len(EDGE_F16) else int(np.float16(rng.normal(0, 0.01)).view(np.uint16))
        raw[i, off] = h & 0xFF
        raw[i, off + 1] = h >> 8
    return raw.reshape(-1)


def dequant_case():
    import oracle

    rng = np.random.default_rng(20240917)
    out = {}
    for name, gtype in (("f32", 0), ("q4_0", 2), ("q8_0", 8), ("q6_k", 14)):
        nblk = 64 if gtype == 0 else 24
        if gtype == 0:
            vals = rng.normal(0, 1, 64).astype(np.float32)
            vals[:4] = [0.0, -0.0, np.inf, 1e-40]
            raw = vals.view(np.uint8)
        else:
            raw = random_blocks(gtype, nblk, rng)
        n = (raw.size // BLOCK[gtype][0]) * BLOCK[gtype][1]
        out[f"{name}_raw"] = raw
        out[f"{name}_out"] = oracle.dequant(gtype, raw, n).astype(np.float32)
    return out


def generate() -> dict[str, dict]:
    fx = {f"tiny_{k}": tiny_case(v) for k, v in TINY_TYPES.items()}
    fx.update({f"matvec4096_{k}": matvec_case(v) for k, v in MV_TYPES.items()})
    fx["dequant_blocks"] = dequant_case()
    return fx


def main() -> int:
    import oracle
    from talos_b200 import build

    oracle.build()
    build.build_synth()
    for name, d in generate().items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **d)
        print("wrote", name)
    return 0


if __name__ == "__main__":
    sys.exit(main())
