"""talos_perplexity (src/eval.rs:35-52 on the GPU) against the oracle's
restatement: the same chunking (context length 8 here, so three chunks) and the
same f64 log-sum-exp NLL; perplexity within 1e-4 relative for F32 weights and
1e-3 for Q4_0, on both step kernels."""
import numpy as np
import pytest

import oracle
from talos_b200 import Model, gguf

from .helpers import prompt, tiny_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wtype,tol", [(gguf.F32, 1e-4), (gguf.Q4_0, 1e-3)])
@pytest.mark.parametrize("sk", ["fused", "layered"])
def test_perplexity_matches_oracle(wtype, tol, sk):
    data = tiny_model(wtype)
    toks = prompt(19, 4096, 3)
    cpu = oracle.Model(data=data)
    cpu.cap_context(8)
    want = oracle.perplexity(cpu, toks)
    gpu = Model.load_bytes(data, step_kernel=sk, max_ctx=8)
    ppl, nll, n = gpu.ctx.perplexity(toks)
    gpu.close()
    assert n == 16
    assert abs(ppl - want) / want <= tol, (ppl, want)


def test_perplexity_needs_two_tokens():
    from talos_b200._lib import TalosError

    gpu = Model.load_bytes(tiny_model(gguf.F32), max_ctx=8)
    with pytest.raises(TalosError, match="INVALID_ARG"):
        gpu.ctx.perplexity([5])
    gpu.close()
