"""Batched multi-sequence LFM2 execution on the GPU vs the oracle, sequence by sequence.

A batch forks S sequences from one prefix state, appends a different suffix
to each (one pass over all of them, rows sequence-major, in row-bounded
groups of sequences), then decodes greedy steps for all of them together
(one captured pass per step, every matmul at S rows).  Each sequence must
give the oracle's logits within the logit gate (1e-2 absolute) and the
oracle's greedy stream, as if it had run alone.  Covered: format mixes,
the integer-MMA GEMV (S < 48) and the tcgen05 GEMM (S >= 48) at decode,
suffixes long enough to split into several sequence groups, and agreement
with the single-sequence fused decode step.
"""
import numpy as np
import pytest

from runtime_b200 import lfm2 as M

pytestmark = pytest.mark.gpu

CONFIG4_LIKE = {"embedding": "int8", "conv_in": "nf4", "conv_out": "nf4", "q": "nf4", "k": "nf4",
                "v": "nf4", "o": "nf4", "w1": "ternary", "w2": "ternary", "w3": "ternary"}
CONFIG3_LIKE = {**{r: "ternary" for r in M.ROLES}, "embedding": "dense"}
ALL_INT8 = {**{r: "int8" for r in M.ROLES}}


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def run_case(be, oracle, formats, seqs, prefix_len, suffix_len, steps, seed, max_tokens=96):
    cfg = M.tiny_config(formats, max_tokens=max_tokens)
    w = M.synthetic_weights(cfg, seed)
    model = M.Lfm2Model(be, cfg, w)
    ref = oracle.Lfm2Oracle(cfg, w, threads=8)
    rng = np.random.default_rng(seed)
    prefix = rng.integers(0, cfg.vocab, size=prefix_len)
    suffixes = rng.integers(0, cfg.vocab, size=(seqs, suffix_len))

    st = model.new_state()
    st.append(prefix)
    ref.append(prefix)
    batch = model.new_batch(seqs)
    batch.fork(st)
    batch.append_argmax(suffixes)
    ids, logits = batch.read()
    ids_steps = batch.decode(steps, want_ids=True)

    refs = []
    for s in range(seqs):
        o = ref.fork()
        lg = o.append(suffixes[s])
        assert np.max(np.abs(logits[s] - lg)) <= 1e-2, s
        tok = int(np.argmax(lg))
        assert int(ids[s]) == tok, s
        stream = []
        for _ in range(steps):
            sampled, _ = o.append_argmax(tok)
            tok = int(sampled)
            stream.append(tok)
        assert list(ids_steps[:, s]) == stream, s
        refs.append(stream)
    _, last_logits = batch.read()
    batch.close()
    st.close()
    model.close()
    return refs, last_logits


@pytest.mark.parametrize("formats", [None, CONFIG4_LIKE, CONFIG3_LIKE, ALL_INT8],
                         ids=["ternary-int8head", "config4-like", "config3-like", "int8"])
def test_batch_suffix_and_decode_match_oracle(be, oracle, formats):
    run_case(be, oracle, formats, seqs=5, prefix_len=11, suffix_len=7, steps=6, seed=41)


def test_batch_single_token_suffix(be, oracle):
    """A one-token suffix takes the decode-shaped pass (fused attention)."""
    run_case(be, oracle, CONFIG4_LIKE, seqs=4, prefix_len=9, suffix_len=1, steps=5, seed=43)


def test_batch_of_many_sequences_uses_the_gemm(be, oracle):
    """50 sequences: every decode-step matmul runs at 50 rows (tcgen05 GEMM)."""
    run_case(be, oracle, CONFIG4_LIKE, seqs=50, prefix_len=6, suffix_len=3, steps=4, seed=47)


def test_batch_long_suffix_runs_in_sequence_groups(be, oracle):
    """3 x 1500-token suffixes exceed one pass's row budget: sequences are
    appended in groups, with the tiled prefill attention per sequence."""
    run_case(be, oracle, None, seqs=3, prefix_len=5, suffix_len=1500, steps=3, seed=53, max_tokens=1536)


def test_batch_matches_single_sequence_decode(be, oracle):
    """Each batched stream equals the single-sequence fused decode's stream."""
    cfg = M.tiny_config(CONFIG4_LIKE, max_tokens=64)
    w = M.synthetic_weights(cfg, 59)
    model = M.Lfm2Model(be, cfg, w)
    rng = np.random.default_rng(59)
    prefix = rng.integers(0, cfg.vocab, size=8)
    suffixes = rng.integers(0, cfg.vocab, size=(3, 4))
    st = model.new_state()
    st.append(prefix)
    batch = model.new_batch(3)
    batch.fork(st)
    batch.append_argmax(suffixes)
    ids, _ = batch.read()
    got = batch.decode(6, want_ids=True)
    for s in range(3):
        one = st.fork()
        one.append(suffixes[s])
        tok = int(ids[s])
        stream = []
        for _ in range(6):
            one.append_argmax(tok)
            tok = int(one.read_sampled())
            stream.append(tok)
        assert list(got[:, s]) == stream
        one.close()
    batch.close()
    st.close()
    model.close()
