"""Tensor-parallel restatement of the decode step, for CPU tests. TEST
INFRASTRUCTURE ONLY (like the rest of oracle/).

The reference is single-device; this module checks the partition the CUDA path
uses for tp ranks (one per GPU) against the oracle's single-device forward
(src/model/llama.rs:96-183), with torch.distributed (gloo) standing in for the
GPUs' all-reduce:

* column-parallel (each rank keeps a row range): attn_q by query heads,
  attn_k / attn_v by kv heads (rank r: kv heads [r*nkv/tp, (r+1)*nkv/tp) and
  their query-head groups, so GQA stays inside a rank), ffn_gate / ffn_up by
  ff rows, output by vocab rows (ceil(V/tp) per rank, the last rank shorter);
* row-parallel (each rank keeps a column range): attn_output over the rank's
  query-head columns, ffn_down over its ff columns; their partial outputs are
  summed over ranks (the all-reduce), in rank order;
* replicated: norms, token embedding, the residual stream.

The same ranges are what talos_weight_upload keeps on each rank.
"""
from __future__ import annotations

import numpy as np

from . import Gguf, argmax, dequant, rmsnorm, rope, softmax, swiglu


def shard_range(kind: str, rows: int, cols: int, tp: int, rank: int, cfg) -> tuple[int, int, int, int]:
    """(r0, r1, c0, c1) of a weight's shard on `rank` (talos_weight_upload's rule)."""
    hd = cfg.n_embd // cfg.n_head
    q_rows = cfg.n_head // tp * hd
    kv_l = cfg.n_head_kv // tp * hd
    ff_l = cfg.n_ff // tp
    vchunk = -(-cfg.vocab_size // tp)
    r0, r1, c0, c1 = 0, rows, 0, cols
    if kind == "attn_q":
        r0, r1 = rank * q_rows, (rank + 1) * q_rows
    elif kind in ("attn_k", "attn_v"):
        r0, r1 = rank * kv_l, (rank + 1) * kv_l
    elif kind in ("ffn_gate", "ffn_up"):
        r0, r1 = rank * ff_l, (rank + 1) * ff_l
    elif kind == "output":
        r0, r1 = rank * vchunk, min(cfg.vocab_size, (rank + 1) * vchunk)
    elif kind == "attn_output":
        c0, c1 = rank * q_rows, (rank + 1) * q_rows
    elif kind == "ffn_down":
        c0, c1 = rank * ff_l, (rank + 1) * ff_l
    return r0, r1, c0, c1


class TPModel:
    """One rank's shard of a GGUF model and its decode step; `allreduce(v)` sums
    a float32 vector over the ranks (in rank order) and `allgather(v)` joins the
    ranks' vocab shards."""

    def __init__(self, data: bytes, tp: int, rank: int, allreduce, allgather):
        from . import Model

        self.cfg = Model(data=data).cfg
        self.tp, self.rank = tp, rank
        self.allreduce, self.allgather = allreduce, allgather
        g = Gguf(data=data)
        c = self.cfg
        self.hd = c.n_embd // c.n_head

        def full(name, rows, cols):
            raw, t = g.tensor_raw(name)
            return dequant(t, np.frombuffer(raw, np.uint8), rows * cols).reshape(rows, cols)

        def shard(name, kind, rows, cols):
            r0, r1, c0, c1 = shard_range(kind, rows, cols, tp, rank, c)
            return np.ascontiguousarray(full(name, rows, cols)[r0:r1, c0:c1])

        E, F, KV, V = c.n_embd, c.n_ff, c.n_head_kv * self.hd, c.vocab_size
        self.embd = full("token_embd.weight", V, E)
        self.out_norm = g.tensor_f32("output_norm.weight")
        self.out = shard("output.weight", "output", V, E)
        self.layers = []
        for l in range(c.n_layer):
            p = f"blk.{l}."
            self.layers.append(dict(
                attn_norm=g.tensor_f32(p + "attn_norm.weight"), ffn_norm=g.tensor_f32(p + "ffn_norm.weight"),
                q=shard(p + "attn_q.weight", "attn_q", E, E), k=shard(p + "attn_k.weight", "attn_k", KV, E),
                v=shard(p + "attn_v.weight", "attn_v", KV, E),
                o=shard(p + "attn_output.weight", "attn_output", E, E),
                gate=shard(p + "ffn_gate.weight", "ffn_gate", F, E), up=shard(p + "ffn_up.weight", "ffn_up", F, E),
                down=shard(p + "ffn_down.weight", "ffn_down", E, F)))
        g.close()
        self.kv = [([], []) for _ in range(c.n_layer)]

    def forward(self, token: int, pos: int) -> np.ndarray:
        c, hd = self.cfg, self.hd
        nh, nkv = c.n_head // self.tp, c.n_head_kv // self.tp
        group = nh // nkv
        x = self.embd[token].astype(np.float32).copy()
        for l, ly in enumerate(self.layers):
            h = rmsnorm(x, ly["attn_norm"], c.rms_eps)
            q = rope((ly["q"] @ h).astype(np.float32), pos, nh, hd, c.rope_freq_base)
            k = rope((ly["k"] @ h).astype(np.float32), pos, nkv, hd, c.rope_freq_base)
            v = (ly["v"] @ h).astype(np.float32)
            kc, vc = self.kv[l]
            kc.append(k)
            vc.append(v)
            K, Vv = np.stack(kc), np.stack(vc)
            att = np.empty(nh * hd, np.float32)
            for i in range(nh):
                kh = i // group
                s = (K[:, kh * hd:(kh + 1) * hd] @ q[i * hd:(i + 1) * hd]) * np.float32(1.0 / np.sqrt(hd))
                p = softmax(s.astype(np.float32))
                att[i * hd:(i + 1) * hd] = p @ Vv[:, kh * hd:(kh + 1) * hd]
            x = x + self.allreduce((ly["o"] @ att).astype(np.float32))
            h = rmsnorm(x, ly["ffn_norm"], c.rms_eps)
            f = swiglu((ly["gate"] @ h).astype(np.float32), (ly["up"] @ h).astype(np.float32))
            x = x + self.allreduce((ly["down"] @ f).astype(np.float32))
        h = rmsnorm(x, self.out_norm, c.rms_eps)
        return self.allgather((self.out @ h).astype(np.float32))


__all__ = ["TPModel", "shard_range", "argmax"]
