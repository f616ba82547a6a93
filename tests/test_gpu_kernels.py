"""GPU kernels against the CPU oracle, through the C ABI.

* talos_dequant is bit-exact with GgmlType::dequantize (src/gguf/dtype.rs:64-121).
* talos_matvec matches the oracle's quant::matvec / matmul::matvec within the
  reference's GPU tolerance, |gpu - cpu| <= 1e-3 * max(|cpu|, 1)
  (src/math/metal/mod.rs:527-531), on the reference's own test shapes
  (src/math/metal/mod.rs:533-685) and on the 4096x4096 microbench shape.
"""
import numpy as np
import pytest

import oracle
from talos_b200 import Context, Config, gguf, model, synth

pytestmark = pytest.mark.gpu


def rel_close(gpu, cpu, tol=1e-3):
    err = np.abs(gpu - cpu) / np.maximum(np.abs(cpu), 1.0)
    assert np.all(err <= tol), f"max rel err {err.max():.3e} at {int(err.argmax())}"
    return float(err.max())


def random_blocks(gtype, n, rng, scale_lo=-0.05, scale_hi=0.05):
    """Random valid blocks: random quant bytes, finite f16 scales (as in
    src/math/metal/mod.rs:657-668 for Q6_K)."""
    be, bb = gguf.BLOCK_ELEMS[gtype], gguf.BLOCK_BYTES[gtype]
    if gtype == gguf.F32:
        return rng.normal(0, 1, n).astype(np.float32).view(np.uint8)
    raw = rng.integers(0, 256, n // be * bb, dtype=np.uint8)
    off = 208 if gtype == gguf.Q6_K else 0
    d = rng.uniform(scale_lo, scale_hi, n // be).astype(np.float16)
    special = np.array([0.0, 6e-8, -6.1e-5], np.float16)  # zero and subnormal scales
    k = min(3, d.size - 1)
    d[:k] = special[:k]
    for i, v in enumerate(d):
        raw[i * bb + off:i * bb + off + 2] = np.frombuffer(v.tobytes(), np.uint8)
    return raw


@pytest.mark.parametrize("gtype,n", [(gguf.F32, 1000), (gguf.Q8_0, 32 * 257), (gguf.Q4_0, 32 * 513),
                                     (gguf.Q6_K, 256 * 37), (gguf.Q4_0, 4096 * 4096)])
def test_dequant_bit_exact(gtype, n):
    rng = np.random.default_rng(n + gtype)
    raw = random_blocks(gtype, n, rng)
    gpu = model.dequant(gtype, raw, n)
    cpu = oracle.dequant(gtype, raw, n)
    assert np.array_equal(gpu.view(np.uint32), cpu.view(np.uint32))


def test_dequant_quantized_weights_bit_exact():
    for gtype in (gguf.Q4_0, gguf.Q8_0, gguf.Q6_K):
        raw = synth.tensor(7, "w", 64, 4096, gtype)
        n = 64 * 4096
        assert np.array_equal(model.dequant(gtype, raw, n).view(np.uint32),
                              oracle.dequant(gtype, raw, n).view(np.uint32))


F32_SHAPES = [(64, 128), (200, 257), (1, 64), (333, 32)]      # metal/mod.rs:536
QUANT_SHAPES = [(64, 128), (200, 256), (1, 64), (129, 32)]    # metal/mod.rs:580
Q6K_SHAPES = [(64, 256), (200, 512), (1, 256), (3, 768)]      # metal/mod.rs:672


@pytest.mark.parametrize("rows,cols", F32_SHAPES)
def test_matvec_f32(rows, cols):
    rng = np.random.default_rng(rows * cols)
    w = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    rel_close(model.matvec(gguf.F32, w.view(np.uint8), x, rows, cols), oracle.matvec_f32(w, x, rows, cols))


@pytest.mark.parametrize("gtype", [gguf.Q8_0, gguf.Q4_0])
@pytest.mark.parametrize("rows,cols", QUANT_SHAPES)
def test_matvec_quant(gtype, rows, cols):
    rng = np.random.default_rng(rows * cols + gtype)
    w = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    raw = oracle.quantize(gtype, w)
    rel_close(model.matvec(gtype, raw, x, rows, cols), oracle.matvec_quant(raw, gtype, x, rows, cols))


@pytest.mark.parametrize("rows,cols", Q6K_SHAPES)
def test_matvec_q6_k(rows, cols):
    rng = np.random.default_rng(rows * cols + 14)
    raw = random_blocks(gguf.Q6_K, rows * cols, rng)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    rel_close(model.matvec(gguf.Q6_K, raw, x, rows, cols), oracle.matvec_quant(raw, gguf.Q6_K, x, rows, cols))


@pytest.mark.parametrize("gtype", [gguf.Q4_0, gguf.Q8_0])
def test_matvec_4096_microbench_shape(gtype):
    # The 4096 x 4096 microbenchmark case: W N(0, 0.02) seed 7, x N(0, 1).
    raw = synth.tensor(7, "bench.w", 4096, 4096, gtype)
    x = synth.normal(7, "bench.x", 4096, 1.0)
    gpu = model.matvec(gtype, raw, x, 4096, 4096)
    cpu = oracle.matvec_quant(raw, gtype, x, 4096, 4096)
    assert np.max(np.abs(gpu - cpu)) <= 1e-3


@pytest.mark.parametrize("gtype,rows,cols", [(gguf.Q4_0, 48, 14336), (gguf.Q4_0, 40, 288),
                                             (gguf.Q8_0, 48, 14336), (gguf.Q6_K, 40, 8192),
                                             (gguf.F32, 24, 768)])
def test_matvec_long_and_ragged_rows(gtype, rows, cols):
    raw = synth.tensor(3, "w", rows, cols, gtype)
    x = synth.normal(3, "x", cols, 1.0)
    rel_close(model.matvec(gtype, raw, x, rows, cols), oracle.matvec_quant(raw, gtype, x, rows, cols))


def test_matvec_upload_spans_staging_chunks():
    # 38.3 MB of Q8_0: more than one 32 MB pinned staging chunk, with a ragged tail
    rows, cols = 1100, 32768
    raw = synth.tensor(5, "big", rows, cols, gguf.Q8_0)
    assert len(raw) > 32 << 20 and len(raw) % (32 << 20)
    x = synth.normal(5, "x", cols, 1.0)
    rel_close(model.matvec(gguf.Q8_0, raw, x, rows, cols), oracle.matvec_quant(raw, gguf.Q8_0, x, rows, cols))


def test_resident_weight_is_cached():
    # src/math/metal/mod.rs:602-625: same key, different bytes -> cached result.
    rng = np.random.default_rng(1)
    rows, cols = 64, 128
    wa = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    wb = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    cfg = Config(1, 4, 2, 16, 32, 8, 16, 1e-5, 4, 1e4)
    ctx = Context(cfg)
    cpu_a = oracle.matvec_f32(wa, x, rows, cols)
    g1 = ctx.matvec_resident("test::resident", wa.view(np.uint8), gguf.F32, x, rows, cols)
    g2 = ctx.matvec_resident("test::resident", wb.view(np.uint8), gguf.F32, x, rows, cols)
    rel_close(g1, cpu_a)
    rel_close(g2, cpu_a)
    ctx.close()


def test_matvec_quant_resident():  # metal/mod.rs:627-642
    rng = np.random.default_rng(2)
    rows, cols = 96, 128
    w = rng.uniform(-1, 1, rows * cols).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    raw = oracle.quantize(gguf.Q8_0, w)
    ctx = Context(Config(1, 4, 2, 16, 32, 8, 16, 1e-5, 4, 1e4))
    rel_close(ctx.matvec_resident("test::quant_resident", raw, gguf.Q8_0, x, rows, cols),
              oracle.matvec_quant(raw, gguf.Q8_0, x, rows, cols))
    ctx.close()


def test_matvec_device_entry_point():
    import torch

    raw = synth.tensor(5, "w", 512, 1024, gguf.Q4_0)
    x = synth.normal(5, "x", 1024, 1.0)
    w = model.Weight(gguf.Q4_0, raw, 512, 1024)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(512, device="cuda")
    torch.cuda.synchronize()
    w.matvec_dev(xd.data_ptr(), yd.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    rel_close(yd.cpu().numpy(), oracle.matvec_quant(raw, gguf.Q4_0, x, 512, 1024))
    w.close()
