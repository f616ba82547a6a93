"""talos_matvec_dev_noalloc, the split-K matvec whose scratch is static device
memory (no allocation in the call). The file name sorts last, so the GPU suite
also runs it after every other test; it passes alone as well.

Checks: two calls in a row give identical results (the per-tile arrival
counters are back at zero after each call) that agree with talos_matvec_dev,
the existing entry point, to rounding, and with the CPU oracle's
quant::matvec / matmul::matvec (src/math/quant.rs:18-51, src/math/matmul.rs:34-47)
within the reference's GPU tolerance |gpu - cpu| <= 1e-3 * max(|cpu|, 1)
(src/math/metal/mod.rs:527-531); weights over the scratch's row limit are
refused."""
import numpy as np
import pytest

import oracle
from talos_b200 import Weight, synth
from talos_b200._lib import TalosError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gtype,rows,cols", [(2, 4096, 14336), (2, 28672, 4096), (8, 4096, 4096),
                                             (14, 32000, 4096), (0, 288, 768), (2, 96, 288)])
def test_noalloc_matches_matvec_dev_twice(gtype, rows, cols):
    import torch

    raw = synth.tensor(3, "noalloc.w", rows, cols, gtype)
    x = synth.normal(3, "noalloc.x", cols, 1.0)
    w = Weight(gtype, raw, rows, cols)
    xd = torch.from_numpy(x).cuda()
    y0, y1, y2 = (torch.full((rows,), float("nan"), device="cuda") for _ in range(3))
    w.matvec_dev(xd.data_ptr(), y0.data_ptr())
    w.matvec_dev_noalloc(xd.data_ptr(), y1.data_ptr())
    w.matvec_dev_noalloc(xd.data_ptr(), y2.data_ptr())
    torch.cuda.synchronize()
    a, b, c = y0.cpu().numpy(), y1.cpu().numpy(), y2.cpu().numpy()
    w.close()
    assert np.array_equal(b, c), "second call differs from the first"
    assert np.all(np.isfinite(b))
    assert np.max(np.abs(b - a)) <= 1e-3
    if gtype == 0:
        cpu = oracle.matvec_f32(raw.view(np.float32), x, rows, cols)
    else:
        cpu = oracle.matvec_quant(raw, gtype, x, rows, cols)
    err = np.abs(b - cpu) / np.maximum(np.abs(cpu), 1.0)
    assert err.max() <= 1e-3, f"max rel err vs oracle {err.max():.3e}"


def test_noalloc_refuses_rows_over_the_scratch():
    import torch

    rows, cols = 65536 + 16, 32
    raw = synth.tensor(4, "noalloc.big", rows, cols, 2)
    w = Weight(2, raw, rows, cols)
    xd = torch.zeros(cols, device="cuda")
    yd = torch.zeros(rows, device="cuda")
    with pytest.raises(TalosError, match="UNSUPPORTED"):
        w.matvec_dev_noalloc(xd.data_ptr(), yd.data_ptr())
    w.close()
