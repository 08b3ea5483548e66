"""Multi-process sequence sharding on CPU (gloo, world size 2).

The multi-GPU path gives each rank a full model replica and a contiguous
slice of independent sequences, with no collective while decoding.  These
tests run two `gloo` ranks on the CPU: the slices cover every sequence
exactly once, the max-over-ranks timing reduction agrees on every rank, and
greedy streams decoded rank by rank (with the CPU oracle standing in for the
device) equal the streams of a single process.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from runtime_b200.sharding import max_over_ranks, shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _tiny():
    from runtime_b200 import lfm2 as M

    cfg = M.tiny_config(max_tokens=64)
    return cfg, M.synthetic_weights(cfg, 21)


def _decode(cfg, weights, prompt, steps):
    from oracle import oracle

    ref = oracle.Lfm2Oracle(cfg, weights, threads=1)
    tok = int(np.argmax(ref.append(prompt)))
    out = []
    for _ in range(steps):
        out.append(tok)
        s, _ = ref.append_argmax(tok)
        tok = int(s)
    return out


def _prompts(cfg, n):
    rng = np.random.default_rng(5)
    return [rng.integers(0, cfg.vocab, size=6 + i % 3) for i in range(n)]


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        # 1. partition
        parts = {}
        for n in (0, 1, 2, 5, 512, 513):
            mine = list(shard(n, world, rank))
            got = [None] * world
            dist.all_gather_object(got, mine)
            parts[n] = got
        # 2. max over ranks
        m = max_over_ranks(float(rank + 1) * 1.5, dist)
        # 3. sharded decoding of independent sequences
        cfg, w = _tiny()
        prompts = _prompts(cfg, 5)
        streams = {i: _decode(cfg, w, prompts[i], 4) for i in shard(len(prompts), world, rank)}
        allst = [None] * world
        dist.all_gather_object(allst, streams)
        dist.barrier()
        q.put((rank, parts, m, allst))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_shard_partitions_locally():
    for n in (0, 1, 7, 512, 65536):
        for world in (1, 2, 3, 4, 8):
            slices = [shard(n, world, r) for r in range(world)]
            items = [i for s in slices for i in s]
            assert items == list(range(n))
            sizes = [len(s) for s in slices]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def test_two_gloo_ranks_shard_and_decode():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg, w = _tiny()
    prompts = _prompts(cfg, 5)
    single = {i: _decode(cfg, w, prompts[i], 4) for i in range(len(prompts))}
    for rank, parts, m, allst in results:
        for n, got in parts.items():
            flat = [i for g in got for i in g]
            assert flat == list(range(n)), (n, got)
        assert m == 3.0
        merged = {}
        for d in allst:
            assert not (set(d) & set(merged))
            merged.update(d)
        assert merged == single
