"""Tensor parallelism on the CPU: two gloo ranks run the partition the CUDA path
uses (oracle/tp.py) and must reproduce the single-device oracle forward; the
shard ranges must tile every weight exactly once."""
import os
import socket

import numpy as np
import pytest

import oracle
from oracle.tp import shard_range
from talos_b200 import gguf, synth

from .helpers import prompt, tiny_model

KINDS = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down", "output"]
TP_SHAPE = synth.Shape(n_embd=256, n_layer=2, n_head=8, n_head_kv=4, n_ff=512, vocab=500, ctx=32)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, data, toks, out_dir):
    import torch
    import torch.distributed as dist

    from oracle.tp import TPModel

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def allreduce(v):
            parts = [torch.empty(v.size) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(v))
            acc = parts[0].numpy().copy()
            for p in parts[1:]:  # rank order, as the CUDA path sums its receive slots
                acc = acc + p.numpy()
            return acc.astype(np.float32)

        def allgather(v):
            n = torch.tensor([v.size])
            sizes = [torch.empty_like(n) for _ in range(world)]
            dist.all_gather(sizes, n)
            m = int(max(s.item() for s in sizes))
            pad = np.zeros(m, np.float32)
            pad[: v.size] = v
            parts = [torch.empty(m) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(pad))
            return np.concatenate([p.numpy()[: int(s.item())] for p, s in zip(parts, sizes)]).astype(np.float32)

        m = TPModel(data, world, rank, allreduce, allgather)
        logits = [m.forward(t, pos) for pos, t in enumerate(toks)]
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack(logits))
    finally:
        dist.destroy_process_group()


def _run_tp(data, toks, world, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(world, _free_port(), data, toks, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    return [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]


@pytest.mark.parametrize("tp", [2, 4])
def test_shard_ranges_tile_each_weight(tp):
    cfg = oracle.Model(data=synth.llama_bytes(TP_SHAPE, 1)).cfg
    E, F, V = cfg.n_embd, cfg.n_ff, cfg.vocab_size
    KV = cfg.n_head_kv * (E // cfg.n_head)
    dims = {"attn_q": (E, E), "attn_k": (KV, E), "attn_v": (KV, E), "attn_output": (E, E),
            "ffn_gate": (F, E), "ffn_up": (F, E), "ffn_down": (E, F), "output": (V, E)}
    for kind, (rows, cols) in dims.items():
        cover = np.zeros((rows, cols), np.int32)
        for r in range(tp):
            r0, r1, c0, c1 = shard_range(kind, rows, cols, tp, r, cfg)
            assert (c0 == 0 and c1 == cols) or (r0 == 0 and r1 == rows), kind  # one axis only
            cover[r0:r1, c0:c1] += 1
        assert (cover == 1).all(), kind


def test_tp2_gloo_matches_single_device_f32(tmp_path):
    data = tiny_model(gguf.F32)
    toks = prompt(6, 4096, 5)
    ranks = _run_tp(data, toks, 2, tmp_path)
    cpu = oracle.Model(data=data)
    ref = np.stack([cpu.forward(t, pos) for pos, t in enumerate(toks)])
    for r in ranks:
        assert np.max(np.abs(r - ref)) <= 1e-4
    assert np.array_equal(ranks[0], ranks[1])  # every rank holds the same logits


def test_tp4_gloo_matches_single_device_q4_0(tmp_path):
    data = synth.llama_bytes(TP_SHAPE, 3, wtype=gguf.Q4_0)
    toks = prompt(4, TP_SHAPE.vocab, 8)
    ranks = _run_tp(data, toks, 4, tmp_path)
    cpu = oracle.Model(data=data)
    ref = np.stack([cpu.forward(t, pos) for pos, t in enumerate(toks)])
    for r in ranks:
        assert np.max(np.abs(r - ref)) <= 1e-4
        assert [oracle.argmax(v) for v in r] == [oracle.argmax(v) for v in ref]
