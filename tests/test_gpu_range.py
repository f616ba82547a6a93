"""Activations beyond f16 range. The tensor-core paths carry a matvec input as an
f16 hi + lo pair; an input element of magnitude 2^15 or more would overflow the
hi part, so the kernels stage such an input again scaled by a power of two and
scale the rows back (the per-token kernel and the layered matvec), or scale every
input column into range before the split (the batched GEMM). The reference
works in f32 throughout (src/math/quant.rs:35-45), so results must match it.

Bar: the reference's GPU tolerance scaled to the output's magnitude,
|gpu - cpu| <= 1e-3 * max(1, max |cpu|) (src/math/metal/mod.rs:527-531 use
1e-3 * max(|cpu|, 1) per element; with outputs in the tens of thousands the
per-element form would ask f32 for more than its rounding of sums this large).
"""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, Weight, gguf, model, synth

pytestmark = pytest.mark.gpu


def close(gpu, cpu, tol=1e-3):
    err = float(np.max(np.abs(gpu - cpu)))
    bar = tol * max(1.0, float(np.max(np.abs(cpu))))
    assert np.all(np.isfinite(gpu)), "non-finite output"
    assert err <= bar, f"max abs err {err:.3e} > {bar:.3e}"


def wild_x(n, seed):
    """N(0, 1) with planted +-1e5, +-3e4 and 1e-6 entries (and one 7e4 run)."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, n).astype(np.float32)
    idx = rng.choice(n, 64, replace=False)
    x[idx[:8]] = 1e5
    x[idx[8:16]] = -1e5
    x[idx[16:24]] = 3e4
    x[idx[24:32]] = -3e4
    x[idx[32:64]] = 1e-6
    x[: min(64, n)] = np.float32(7e4)
    return x


@pytest.mark.parametrize("gtype,rows,cols", [(gguf.Q4_0, 256, 4096), (gguf.Q8_0, 200, 2048),
                                             (gguf.Q6_K, 64, 4096), (gguf.F32, 96, 1024)])
def test_matvec_wide_range_inputs(gtype, rows, cols):
    raw = synth.tensor(5, "range.w", rows, cols, gtype)
    x = wild_x(cols, gtype)
    want = (oracle.matvec_f32(raw.view(np.float32), x, rows, cols) if gtype == gguf.F32
            else oracle.matvec_quant(raw, gtype, x, rows, cols))
    close(model.matvec(gtype, raw, x, rows, cols), want)


@pytest.mark.parametrize("gtype", [gguf.Q4_0, gguf.Q6_K])
def test_noalloc_matvec_wide_range_inputs(gtype):
    import torch

    rows, cols = 512, 4096
    raw = synth.tensor(6, "range.n", rows, cols, gtype)
    x = wild_x(cols, 11)
    w = Weight(gtype, raw, rows, cols)
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((rows,), float("nan"), device="cuda")
    w.matvec_dev_noalloc(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    close(yd.cpu().numpy(), oracle.matvec_quant(raw, gtype, x, rows, cols))
    w.close()


def loud_model(wtype):
    """The tiny Llama with every norm weight 300: the RMS-normed inputs are in
    the hundreds and SwiGLU's outputs (the down projection's input) reach 10^5
    to 10^6, beyond f16."""
    return synth.llama_bytes(synth.TINY, 42, wtype=wtype, norm_value=300.0)


@pytest.mark.parametrize("sk", ["fused", "layered"])
@pytest.mark.parametrize("wtype", [gguf.Q4_0, gguf.Q8_0])
def test_decode_step_with_large_activations(wtype, sk):
    data = loud_model(wtype)
    cpu = oracle.Model(data=data)
    gpu = Model.load_bytes(data, step_kernel=sk)
    toks = synth.token_ids(42, 6, synth.TINY.vocab)
    pos = 0
    for t in toks:
        c, g = cpu.forward(t, pos), gpu.forward_gpu(t, pos)
        close(g, c)
        pos += 1
    for _ in range(6):  # greedy continuation: identical tokens
        ct, gt = oracle.argmax(c), oracle.argmax(g)
        assert ct == gt
        c, g = cpu.forward(ct, pos), gpu.forward_gpu(gt, pos)
        close(g, c)
        pos += 1
    gpu.close()


def test_batched_and_prefill_with_large_activations():
    data = loud_model(gguf.Q4_0)
    V = synth.TINY.vocab
    prompts = [synth.token_ids(50 + i, 5, V) for i in range(3)]
    cpus = [oracle.Model(data=data) for _ in prompts]
    gpu = Model.load_bytes(data)
    gpu.set_batch(3)
    for p in range(5):
        lg = gpu.forward_batch([pr[p] for pr in prompts], [p] * 3)
        for i, pr in enumerate(prompts):
            close(lg[i], cpus[i].forward(pr[p], p))
    # a 40-token prompt in one batched prefill step, then the per-token kernel
    cpu = oracle.Model(data=data)
    toks = synth.token_ids(77, 40, V)
    for p, t in enumerate(toks):
        ref = cpu.forward(t, p)
    last = gpu.prefill(toks, 0)
    close(last, ref)
    t = oracle.argmax(ref)
    close(gpu.forward_gpu(t, 40), cpu.forward(t, 40))
    gpu.close()
