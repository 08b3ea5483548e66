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


# ---------------------------------------------------------------------------
# LM-head row split (mf_lfm2_set_head_split): shard rows, the NCCL id handed
# out over the host group, and the candidate pick, with gloo ranks on CPU.
# The device side (NCCL all-gather, pick kernel) runs in
# tests/test_head_split_gpu.py on two GPUs.
# ---------------------------------------------------------------------------
from runtime_b200.sharding import head_shard_rows  # noqa: E402


def _shard_candidate(row, rows):
    """(max, first index of it, poisoned) of row[rows], as the head's argmax
    epilogue writes it for its shard (dense.rs:369-411 within the shard)."""
    part = row[rows.start:rows.stop]
    if not np.all(np.isfinite(part)):
        return (float("-inf"), -1.0, 1.0)
    i = int(np.argmax(part))
    return (float(part[i]), float(rows.start + i), 0.0)


def _pick(cands):
    """The pick over ranks in order: first strict maximum, NaN if poisoned."""
    bv, bi, poisoned = float("-inf"), -1.0, False
    for v, i, pz in cands:
        if pz:
            poisoned = True
        elif i >= 0 and (bi < 0 or v > bv):
            bv, bi = v, i
    return float("nan") if poisoned or bi < 0 else bi


def _head_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from runtime_b200.sharding import head_split_id

        uid = head_split_id(dist)
        ids = [None] * world
        dist.all_gather_object(ids, uid)
        rng = np.random.default_rng(77)
        picks = []
        for case in range(4):
            row = rng.normal(size=1000).astype(np.float32)
            if case == 1:   # tie across shards: the lower index wins
                row[:] = -5.0
                row[10] = row[990] = 3.0
            if case == 2:   # tie inside the higher shard
                row[:] = -5.0
                row[700] = row[800] = 4.0
            if case == 3:   # a NaN in one shard poisons the id
                row[600] = np.nan
            mine = _shard_candidate(row, head_shard_rows(len(row), world, rank))
            cands = [None] * world
            dist.all_gather_object(cands, mine)
            picks.append(_pick(cands))
        dist.barrier()
        q.put((rank, ids, picks))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_head_shard_rows_partition():
    for vocab in (1000, 1024, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            rows = [head_shard_rows(vocab, world, r) for r in range(world)]
            assert [i for r in rows for i in r] == list(range(vocab))
            assert all(r.start % 16 == 0 for r in rows)
    with pytest.raises(ValueError):
        head_shard_rows(40, 4, 0)   # 16-row shards leave the last rank nothing


def test_two_gloo_ranks_head_split_pick():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(77)
    want = []
    for case in range(4):
        row = rng.normal(size=1000).astype(np.float32)
        if case == 1:
            row[:] = -5.0
            row[10] = row[990] = 3.0
        if case == 2:
            row[:] = -5.0
            row[700] = row[800] = 4.0
        if case == 3:
            row[600] = np.nan
        want.append(float("nan") if not np.all(np.isfinite(row)) else float(np.argmax(row)))
    assert want[1] == 10.0 and want[2] == 700.0
    for rank, ids, picks in results:
        assert len(ids[0]) == 128 and ids[0] == ids[1]
        assert picks[:3] == want[:3] and np.isnan(picks[3]) and np.isnan(want[3])
