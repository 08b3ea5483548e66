"""The persistent single-token decode step against the CPU oracle.

One launch per greedy token runs every stage of the step
(crates/executor-core/src/lfm2/executor/execution.rs:35-627 for one row,
then sample_epilogue :591-614).  North-star gates: logits within 1e-2
absolute, greedy streams identical to the oracle's, token for token.
Covered: every packed format in every role family, the dense F32 tied head,
conv and attention layers, contexts that leave attention chunks empty, the
captured decode graph, the device generation loop, and the comparison with
the separate-launch fused step.
"""
import numpy as np
import pytest

from runtime_b200 import lfm2 as M

pytestmark = pytest.mark.gpu

CONFIG3_LIKE = {**{r: "ternary" for r in M.ROLES}, "embedding": "dense"}
CONFIG4_LIKE = {"embedding": "int8", "conv_in": "nf4", "conv_out": "nf4", "q": "nf4", "k": "nf4",
                "v": "nf4", "o": "nf4", "w1": "ternary", "w2": "ternary", "w3": "ternary"}
ALL_NF4 = {r: "nf4" for r in M.ROLES}
ALL_INT8 = {r: "int8" for r in M.ROLES}
TERNARY_NF4_HEAD = {**{r: "ternary" for r in M.ROLES}, "embedding": "nf4"}


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def faults():
    import ctypes as C

    from runtime_b200 import _lib

    v = C.c_uint32(0)
    assert _lib.load().mf_device_faults(C.byref(v)) == 0
    return v.value


def run_stream(model, prompt, steps):
    st = model.new_state()
    st.append(prompt)
    first = int(np.argmax(st.logits()))
    ids, stopped = st.generate(steps + 1, first_token=first)
    assert not stopped
    return st, ids


@pytest.mark.parametrize("formats,layers", [
    (None, ("conv", "attention", "conv", "attention")),
    (CONFIG4_LIKE, ("conv", "attention", "conv", "attention")),
    (CONFIG3_LIKE, ("conv", "conv", "attention")),
    (ALL_NF4, ("attention", "conv")),
    (ALL_INT8, ("conv", "attention")),
    (TERNARY_NF4_HEAD, ("attention", "attention", "conv")),
])
def test_persistent_stream_matches_oracle(be, oracle, formats, layers):
    cfg = M.tiny_config(formats, layers=layers, max_tokens=96)
    w = M.synthetic_weights(cfg, 21)
    model = M.Lfm2Model(be, cfg, w)
    model.set_persistent(True)
    ref = oracle.Lfm2Oracle(cfg, w, threads=8)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, size=9)
    ref_logits = ref.append(prompt)
    st, ids = run_stream(model, prompt, 40)
    assert st.persistent_active
    want = [int(np.argmax(ref_logits))]
    for _ in range(40):
        s, logits = ref.append_argmax(want[-1])
        want.append(int(s))
    assert ids == want
    assert np.max(np.abs(st.logits() - logits)) <= 1e-2
    assert st.length == len(prompt) + 40
    assert faults() == 0
    st.close()
    model.close()


def test_persistent_single_steps_and_graph_replays_agree(be, oracle):
    """append_argmax (one launch at a time), the captured decode graph and
    decode_host give the oracle's ids, and each step is one launch."""
    cfg = M.tiny_config(CONFIG4_LIKE, max_tokens=64)
    w = M.synthetic_weights(cfg, 4)
    model = M.Lfm2Model(be, cfg, w)
    model.set_persistent(True)
    ref = oracle.Lfm2Oracle(cfg, w, threads=8)
    prompt = np.random.default_rng(9).integers(0, cfg.vocab, size=5)
    st = model.new_state()
    st.append(prompt)
    tok = int(np.argmax(ref.append(prompt)))
    want = []
    t = tok
    for _ in range(20):
        s, _ = ref.append_argmax(t)
        t = int(s)
        want.append(t)
    st.append_argmax(tok)                 # host token, one launch
    assert st.persistent_active
    assert model.kernels_per_decode_step == 1
    assert int(st.read_sampled()) == want[0]
    st.decode(11)                         # graph replays (8-step graph + singles)
    assert int(st.read_sampled()) == want[11]
    got = [int(st.decode_host(None)) for _ in range(8)]
    assert got == want[12:20]
    assert faults() == 0
    st.close()
    model.close()


def test_persistent_matches_separate_launch_step(be):
    """Same greedy stream and logits within rounding as the fused
    separate-launch step (config-4 widths, two layers)."""
    cfg = M.PRESETS["lfm2-1.2b"].with_(layer_types=["conv", "attention"], max_tokens=160)
    w = M.synthetic_weights(cfg, 8)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, size=100)
    streams, logits = [], []
    for persistent in (True, False):
        model = M.Lfm2Model(be, cfg, w)
        model.set_persistent(persistent)
        st, ids = run_stream(model, prompt, 24)
        assert st.persistent_active == persistent
        streams.append(ids)
        logits.append(st.logits())
        st.close()
        model.close()
    assert streams[0] == streams[1]
    assert np.max(np.abs(logits[0] - logits[1])) <= 1e-3
    assert faults() == 0


def test_persistent_state_copy_restarts_stream(be):
    """Restoring a state from its prefix (device copies) replays the same
    stream: the step's tagged exchange words carry a per-state epoch that
    only moves forward."""
    cfg = M.tiny_config(None, max_tokens=80)
    model = M.Lfm2Model(be, cfg, M.synthetic_weights(cfg, 2))
    model.set_persistent(True)
    prefix = model.new_state()
    prefix.append(np.arange(7) * 31 % cfg.vocab)
    prefix.append_argmax(3)
    work = model.new_state()
    runs = []
    for _ in range(3):
        work.copy_from(prefix)
        ids, _ = work.generate(16)
        runs.append(ids)
    assert runs[0] == runs[1] == runs[2]
    assert work.persistent_active
    assert faults() == 0
    for s in (work, prefix):
        s.close()
    model.close()
