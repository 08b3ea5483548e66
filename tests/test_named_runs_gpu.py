"""The named benchmark runs at full shape, token for token against the CPU
oracle's fixtures (tests/golden/make_named_runs.py writes them; the seeds
are bench.py's).

North-star gates: final logits within 1e-2 absolute, greedy token streams
identical.  Each run goes through the product path the benchmark times:
bulk prefill (`mf_lfm2_append`, tcgen05 GEMMs above 48 rows), then the
greedy loop of `mf_lfm2_generate` (the device-side loop over the captured
fused decode step), or for config 5 the batched sequence API over all 512
sequences with the stated subset checked.  Reference order:
crates/executor-core/src/lfm2/executor/execution.rs:35-627 and
`sample_epilogue` :591-614.

Should a stream ever diverge, the assertion message carries the oracle's
top-1 minus top-2 logit margin at that step (a near tie is the only way
reordered F32 sums can flip an argmax).
"""
import os

import numpy as np
import pytest

from runtime_b200 import lfm2 as M

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
NAMED = os.path.join(HERE, "golden", "named_runs")
LOGIT_ATOL = 1e-2


def load(name):
    path = os.path.join(NAMED, f"{name}.npz")
    assert os.path.exists(path), f"missing fixture {path} (tests/golden/make_named_runs.py)"
    return np.load(path)


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def stream_check(got, want, margins):
    got, want = list(got), list(want)
    assert len(got) == len(want), (len(got), len(want))
    for i, (g, w) in enumerate(zip(got, want)):
        assert g == w, (f"greedy stream diverges at step {i}: device {g}, oracle {w}; "
                        f"oracle top-2 margin there {margins[i]:.3g}")


@pytest.mark.parametrize("name,steps", [("lfm2-350m", 128), ("lfm2-1.2b", 256)])
def test_named_single_sequence_run(be, name, steps):
    fx = load(name)
    prompt = fx["prompt"]
    cfg = M.PRESETS[name].with_(max_tokens=len(prompt) + steps + 8)
    model = M.Lfm2Model(be, cfg, M.synthetic_weights(cfg, int(fx["weight_seed"])))
    st = model.new_state()
    st.append(prompt, want_logits=True)
    logits = st.logits()
    err = float(np.max(np.abs(logits - fx["prompt_logits"])))
    assert err <= LOGIT_ATOL, f"prompt logits differ by {err}"
    assert int(np.argmax(logits)) == int(fx["ids"][0])
    ids, stopped = st.generate(steps + 1, first_token=int(fx["ids"][0]))
    assert not stopped
    stream_check(ids, fx["ids"], fx["margins"])
    assert st.length == len(prompt) + steps
    err = float(np.max(np.abs(st.logits() - fx["final_logits"])))
    assert err <= LOGIT_ATOL, f"final-step logits differ by {err}"
    st.close()
    model.close()


def test_named_batched_run_subset(be):
    """Config 5: 512 sequences fork the 512-token prefix and append their
    64-token suffixes in one batch, then decode greedily; the fixture's
    subset of sequences must match the oracle token for token."""
    from tests.golden.make_named_runs import C5_SEQS, C5_STEPS, c5_inputs

    fx = load("lfm2-2.6b")
    cfg, seed, prefix, suffixes = c5_inputs()
    assert int(fx["weight_seed"]) == seed and np.array_equal(fx["prefix"], prefix)
    subset = [int(s) for s in fx["subset"]]
    assert np.array_equal(fx["suffixes"], suffixes[subset])
    model = M.Lfm2Model(be, cfg, M.synthetic_weights(cfg, seed))
    pre = model.new_state()
    pre.append(prefix, want_logits=False)
    batch = model.new_batch(C5_SEQS)
    batch.fork(pre)
    batch.append_argmax(suffixes)
    sampled, logits = batch.read()
    for j, s in enumerate(subset):
        row = logits[s]
        err = float(np.max(np.abs(row[fx["top_idx"][j]] - fx["top_val"][j])))
        assert err <= LOGIT_ATOL, f"sequence {s}: top logits differ by {err}"
        assert float(row.max()) <= float(fx["top_val"][j][0]) + LOGIT_ATOL
        assert abs(float(row.astype(np.float64).sum()) - fx["sums"][j][0]) <= LOGIT_ATOL * row.size
    ids = batch.decode(C5_STEPS, want_ids=True)       # [steps, sequences]
    for j, s in enumerate(subset):
        got = [int(sampled[s])] + [int(v) for v in ids[:, s]]
        stream_check(got, fx["ids"][j], fx["margins"][j])
    batch.close()
    pre.close()
    model.close()
