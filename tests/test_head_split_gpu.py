"""The LM-head row split over NCCL on two GPUs (mf_lfm2_set_head_split).

Each rank holds a full replica on its own GPU and runs the same greedy steps
on the same tokens; the head's rows are split in two, each rank scores its
shard, the candidates are all-gathered over NCCL and every rank picks the
same greedy id.  The stream must equal the one-GPU stream of the same model
(which the other tests hold to the CPU oracle), through the captured decode
graph and through the host form of the generation loop, for an INT8 head,
a ternary head and a dense F32 head.  Skipped with fewer than two GPUs.
NVLS stays off (NCCL_NVLS_ENABLE=0): the exchange is 12 bytes per rank.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HEADS = ("int8", "ternary", "dense")


def _model(be, head):
    from runtime_b200 import lfm2 as M

    fmts = {r: "ternary" for r in M.ROLES}
    fmts["embedding"] = head
    cfg = M.tiny_config(fmts, layers=("conv", "attention", "conv"), vocab=2048, max_tokens=96)
    return cfg, M.Lfm2Model(be, cfg, M.synthetic_weights(cfg, 41))


def _child(rank, world, uids, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from runtime_b200.backend import CudaBackend

        be = CudaBackend(rank)
        out = {}
        for head, uid in zip(HEADS, uids):   # a fresh NCCL id per communicator
            cfg, model = _model(be, head)
            prompt = np.random.default_rng(9).integers(0, cfg.vocab, size=11)
            ref = model.new_state()
            ref.append(prompt)
            first = int(np.argmax(ref.logits()))
            want, _ = ref.generate(20, first_token=first)
            ref.close()
            model.set_head_split(uid, rank, world)
            st = model.new_state()
            st.append(prompt)
            got, _ = st.generate(20, first_token=first)        # host loop
            g2 = model.new_state()
            g2.append(prompt)
            g2.append_argmax(first)
            g2.decode(18)                                     # captured graph
            last = int(g2.read_sampled())
            out[head] = (want, got, last)
            for s in (st, g2):
                s.close()
            model.close()
        be.close()
        q.put((rank, out, None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, None, repr(e)))


def test_head_split_two_gpus_matches_one():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from runtime_b200 import lfm2 as M

    uids = [M.nccl_unique_id() for _ in HEADS]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_child, args=(r, 2, uids, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=300) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, out, err in results:
        assert err is None, f"rank {rank}: {err}"
        for head, (want, got, last) in out.items():
            assert got == want, (rank, head)
            assert last == want[19], (rank, head)
    assert results[0][1] == results[1][1]
