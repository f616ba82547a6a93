"""The committed golden fixtures (tests/golden/, made by make_golden.py).

CPU tests: the seeded inputs still hash to what the fixtures were made from, and
the oracle still reproduces every fixture exactly. GPU tests: the CUDA path
against the same fixtures, with the north-star bars (dequant bit-exact, greedy
tokens identical, logits within 1e-4 max-abs for F32 and 1e-3 for quantized
weights, matvec within 1e-3 max-abs).
"""
import os

import numpy as np
import pytest

import oracle
from talos_b200 import synth

from .golden import make_golden as mg
from .helpers import prompt, tiny_model

GOLDEN = os.path.dirname(mg.__file__)
LOGIT_TOL = {"f32": 1e-4, "q8_0": 1e-3, "q4_0": 1e-3}


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


# ------------------------------------------------------------------ CPU


@pytest.mark.parametrize("name", sorted(mg.TINY_TYPES))
def test_tiny_inputs_unchanged(name):
    g = load(f"tiny_{name}")
    assert mg.sha(tiny_model(mg.TINY_TYPES[name])) == str(g["model_sha"])
    assert list(g["prompt"]) == prompt(mg.N_PROMPT, 4096, 42)


@pytest.mark.parametrize("name", sorted(mg.TINY_TYPES))
def test_oracle_reproduces_tiny(name):
    g = load(f"tiny_{name}")
    now = mg.tiny_case(mg.TINY_TYPES[name])
    assert np.array_equal(now["tokens"], g["tokens"])
    assert np.array_equal(now["logits_prompt"], g["logits_prompt"])
    assert np.array_equal(now["logits_last"], g["logits_last"])


@pytest.mark.parametrize("name", sorted(mg.MV_TYPES))
def test_oracle_reproduces_matvec(name):
    g = load(f"matvec4096_{name}")
    now = mg.matvec_case(mg.MV_TYPES[name])
    assert str(now["w_sha"]) == str(g["w_sha"]) and str(now["x_sha"]) == str(g["x_sha"])
    assert np.array_equal(now["y"], g["y"])
    assert np.array_equal(now["dequant_rows01"].view(np.uint32), g["dequant_rows01"].view(np.uint32))


def test_oracle_reproduces_dequant_blocks():
    g = load("dequant_blocks")
    for name, gtype in (("f32", 0), ("q4_0", 2), ("q8_0", 8), ("q6_k", 14)):
        raw = g[f"{name}_raw"]
        out = oracle.dequant(gtype, raw, g[f"{name}_out"].size)
        assert np.array_equal(out.view(np.uint32), g[f"{name}_out"].view(np.uint32)), name


# ------------------------------------------------------------------ GPU


def same_bits_nan_as_class(got, want):
    """Bit-exact, except that a NaN matches any NaN: the payload of a NaN made by
    arithmetic (inf * 0, NaN scale * q) is the platform's, not the format's."""
    gn, wn = np.isnan(got), np.isnan(want)
    return np.array_equal(gn, wn) and np.array_equal(got[~gn].view(np.uint32), want[~wn].view(np.uint32))


@pytest.mark.gpu
def test_gpu_dequant_golden_bit_exact():
    from talos_b200 import dequant

    g = load("dequant_blocks")
    for name, gtype in (("f32", 0), ("q4_0", 2), ("q8_0", 8), ("q6_k", 14)):
        want = g[f"{name}_out"]
        got = dequant(gtype, g[f"{name}_raw"], want.size)
        assert same_bits_nan_as_class(got, want), name


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(mg.MV_TYPES))
def test_gpu_matvec_golden(name):
    from talos_b200 import matvec

    g = load(f"matvec4096_{name}")
    gtype = mg.MV_TYPES[name]
    raw = synth.tensor(7, "bench.w", 4096, 4096, gtype)
    x = synth.normal(7, "bench.x", 4096, 1.0)
    y = matvec(gtype, raw, x, 4096, 4096)
    assert np.max(np.abs(y - g["y"])) <= 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(mg.TINY_TYPES))
def test_gpu_tiny_golden(name):
    """Prompt through forward_gpu, then the device greedy loop; tokens must equal
    the fixture's and the two stored logit vectors must be within the bar."""
    from talos_b200 import Model

    g = load(f"tiny_{name}")
    m = Model.load_bytes(tiny_model(mg.TINY_TYPES[name]))
    pos = 0
    for t in g["prompt"]:
        lg = m.forward_gpu(int(t), pos)
        pos += 1
    tol = LOGIT_TOL[name]
    assert np.max(np.abs(lg - g["logits_prompt"])) <= tol
    first = int(oracle.argmax(lg))
    assert first == int(g["tokens"][0])
    toks = m.generate_greedy(first, pos, mg.N_GEN - 1)
    assert [first] + [int(t) for t in toks] == [int(t) for t in g["tokens"]]
    # logits of the last step: replay the sequence through forward_gpu
    m.reset()
    pos = 0
    for t in list(g["prompt"]) + list(g["tokens"]):
        lg = m.forward_gpu(int(t), pos)
        pos += 1
    assert np.max(np.abs(lg - g["logits_last"])) <= tol
    m.close()
