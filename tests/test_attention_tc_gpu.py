"""Many-token causal GQA on the tcgen05 tensor cores (attention_tc.cu).

Head dimension 64 and 64 or more tokens take this kernel by default; it
splits every F32 operand of Q K^T and P V into a BF16 hi/lo pair (three
MMAs per product, F32 accumulators) and runs the online softmax in F32, the
reference's attention (crates/backend-cpu/src/attention_convolution.rs:
11-187) up to summation order.  Covered: the oracle at query groups 1 to
32, ragged token counts, a cached prefix before the call (keys visible to
every row, tiles that start mid-prefix), the F32 kernel on the same inputs
(`mf_set_attention_tc(0)`), and the batched many-sequence form through the
model's batch pass.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def close(got, exp, atol, rtol):
    got = np.asarray(got, np.float64).ravel()
    exp = np.asarray(exp, np.float64).ravel()
    assert got.shape == exp.shape
    err = np.abs(got - exp)
    assert np.all(err <= atol + rtol * np.abs(exp)), float(err.max())


def _gqa_run(be, qh, kvh, steps, seed):
    """Runs the calls of `steps` tokens in turn on one cache; returns the
    inputs and the device outputs."""
    d = 64
    rng = np.random.default_rng(seed)
    kvw = kvh * d
    cap = sum(steps) + 5
    bkc, bvc = be.allocate_f32((cap, kvw)), be.allocate_f32((cap, kvw))
    n = 0
    calls = []
    for t in steps:
        q = rng.normal(size=(t, qh * d)).astype(np.float32)
        k = rng.normal(size=(t, kvw)).astype(np.float32)
        v = rng.normal(size=(t, kvw)).astype(np.float32)
        out = be.allocate_f32(q.shape)
        n = be.causal_gqa(out, be.upload_f32(q), be.upload_f32(k), be.upload_f32(v), bkc, bvc, n, (qh, kvh, d))
        calls.append((q, k, v, be.read_f32(out)))
    return calls, cap


@pytest.mark.parametrize("qh,kvh,steps", [
    (32, 8, [300]),            # the bench model's heads, one call
    (32, 8, [37, 1, 130]),     # a cached prefix, then a ragged call
    (16, 8, [64, 600]),        # group 2, tiles starting mid-prefix
    (8, 1, [200]),             # group 8
    (64, 2, [129]),            # group 32: 4 tokens per CTA
    (8, 8, [77]),              # group 1
])
def test_tc_attention_matches_oracle(be, oracle, qh, kvh, steps):
    calls, cap = _gqa_run(be, qh, kvh, steps, seed=qh * 7 + kvh + len(steps))
    d, kvw = 64, kvh * 64
    kc = np.zeros((cap, kvw), np.float32)
    vc = np.zeros((cap, kvw), np.float32)
    n = 0
    for q, k, v, got in calls:
        ref, n = oracle.causal_gqa(q, k, v, qh, kvh, d, kc, vc, n, threads=8)
        close(got, ref, 1e-5, 1e-4)


def test_tc_and_f32_kernels_agree(be):
    from runtime_b200 import _lib

    lib = _lib.load()
    outs = []
    try:
        for on in (1, 0):
            assert lib.mf_set_attention_tc(on) == 0
            calls, _ = _gqa_run(be, 32, 8, [100, 400], seed=5)
            outs.append([c[3] for c in calls])
    finally:
        lib.mf_set_attention_tc(1)
    for tc, f32 in zip(*outs):
        close(tc, f32, 1e-5, 1e-4)
    assert not np.array_equal(outs[0][1], outs[1][1])   # two different kernels ran


def test_batched_many_token_attention_matches_f32(be):
    """The batch pass appends 70 tokens to each of 4 forked sequences
    (seq_tokens >= 64: the tensor-core kernel over all sequences in one
    launch); the greedy continuation must equal the F32 kernel's."""
    from runtime_b200 import _lib
    from runtime_b200 import lfm2 as M

    lib = _lib.load()
    cfg = M.tiny_config(None, layers=("conv", "attention", "conv", "attention"), max_tokens=160)
    w = M.synthetic_weights(cfg, 61)
    prefix = np.random.default_rng(6).integers(0, cfg.vocab, size=30)
    suffix = np.random.default_rng(7).integers(0, cfg.vocab, size=(4, 70))
    outs = []
    try:
        for on in (1, 0):
            assert lib.mf_set_attention_tc(on) == 0
            model = M.Lfm2Model(be, cfg, w)
            pre = model.new_state()
            pre.append(prefix, want_logits=False)
            batch = model.new_batch(4)
            batch.fork(pre)
            batch.append_argmax(suffix)
            outs.append(batch.decode(8, want_ids=True))
            batch.close()
            pre.close()
            model.close()
    finally:
        lib.mf_set_attention_tc(1)
    assert np.array_equal(outs[0], outs[1])


def test_no_fault_recorded(be):
    """The waits of every launch above completed: no fault bit."""
    import ctypes

    from runtime_b200 import _lib

    flags = ctypes.c_uint32(7)
    assert _lib.load().mf_device_faults(ctypes.byref(flags)) == 0
    assert flags.value == 0
