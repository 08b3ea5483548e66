"""The non-allocating causal GQA entry point.

`mfk_causal_gqa_noalloc` serves callers that cannot call cudaMalloc (a host
whose memory manager already owns the device's memory, or a decode loop that
must not make a call that may synchronize the device): its split-key
partials live in a static device array instead of backend scratch.

Each case here runs the same attention through the CPU oracle
(`oracle.causal_gqa`, the restatement of
crates/backend-cpu/src/attention_convolution.rs:11-187) and through the
non-allocating entry point, and the first case also through `mf_causal_gqa`
(handle tier, backend scratch) on an identical copy of the caches, two calls
in a row.  Outputs agree within the GQA tolerance of the other tests; the
appended cache rows are bit-exact copies.  The cases cover each path
causal_gqa takes: single-token and 2-16-token decode (partials in the static
array), 17-63 tokens at head_dim 64 (the tiled prefill kernel, no partials,
so a long cache is no reason to refuse), and the split-key chunk kernel at
another head dimension (partials again).

This file is named to be collected last, and it builds its own backend, so
it passes alone in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-5, 1e-4  # the GQA tolerance of tests/test_layer_gpu.py
RESOURCE_LIMIT = 8


def close(got, exp):
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    assert got.shape == exp.shape
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - exp) <= ATOL + RTOL * np.abs(exp)), float(np.max(np.abs(got - exp)))


@pytest.fixture(scope="module")
def be():
    from runtime_b200.backend import CudaBackend

    b = CudaBackend(0)
    yield b
    b.close()


def noalloc(be, out, q, k, v, kc, vc, cap, start, t, spec):
    from runtime_b200 import _lib

    L = _lib.load()
    return L.mfk_causal_gqa_noalloc(out.ptr, q.ptr, k.ptr, v.ptr, kc.ptr, vc.ptr, cap, start, t,
                                    spec[0], spec[1], spec[2], C.c_void_p(be.stream))


def test_noalloc_gqa_matches_oracle_and_allocating_entry_point_twice(be, oracle):
    from runtime_b200 import _lib

    L = _lib.load()
    qh, kvh, d = 32, 8, 64
    cap, start = 1024, 700   # 700+ visible rows: the split-key path, so the scratch is used
    rng = np.random.default_rng(17)
    kc0 = rng.normal(size=(cap, kvh * d)).astype(np.float32)
    vc0 = rng.normal(size=(cap, kvh * d)).astype(np.float32)
    kc_ref, vc_ref = kc0.copy(), vc0.copy()               # oracle caches
    kc_a, vc_a = be.upload_f32(kc0), be.upload_f32(vc0)   # allocating path's caches
    kc_b, vc_b = be.upload_f32(kc0), be.upload_f32(vc0)   # non-allocating path's caches
    n_ref, n_a, n_b = start, start, start
    for call in range(2):
        q = rng.normal(size=(1, qh * d)).astype(np.float32)
        k = rng.normal(size=(1, kvh * d)).astype(np.float32)
        v = rng.normal(size=(1, kvh * d)).astype(np.float32)
        ref, n_ref = oracle.causal_gqa(q, k, v, qh, kvh, d, kc_ref, vc_ref, n_ref, threads=8)
        bq, bk, bv = be.upload_f32(q), be.upload_f32(k), be.upload_f32(v)
        out_a = be.allocate_f32((1, qh * d))
        out_b = be.allocate_f32((1, qh * d))
        n_a = be.causal_gqa(out_a, bq, bk, bv, kc_a, vc_a, n_a, (qh, kvh, d))
        st = noalloc(be, out_b, bq, bk, bv, kc_b, vc_b, cap, n_b, 1, (qh, kvh, d))
        assert st == 0, L.mf_last_error().decode()
        n_b += 1
        assert n_a == n_b == n_ref == start + call + 1
        got = be.read_f32(out_b)
        close(got, ref)
        close(got, be.read_f32(out_a))
        assert np.array_equal(be.read_f32(kc_b), kc_ref)
        assert np.array_equal(be.read_f32(vc_b), vc_ref)


@pytest.mark.parametrize("qh,kvh,d,start,t", [
    (32, 8, 64, 300, 5),      # 2-16 tokens: decode kernel, partials in the static array
    (32, 8, 64, 2048 - 63, 63),  # 17-63 tokens at head_dim 64: tiled prefill kernel, no partials
    (8, 2, 128, 580, 20),     # split-key chunk kernel (head_dim 128), partials in the static array
])
def test_noalloc_gqa_paths_match_oracle(be, oracle, qh, kvh, d, start, t):
    from runtime_b200 import _lib

    L = _lib.load()
    rng = np.random.default_rng(qh * 1000 + d * 10 + t)
    cap = start + t
    kvw = kvh * d
    kc = np.zeros((cap, kvw), np.float32)
    vc = np.zeros((cap, kvw), np.float32)
    kc[:start] = rng.normal(size=(start, kvw))
    vc[:start] = rng.normal(size=(start, kvw))
    bkc, bvc = be.upload_f32(kc), be.upload_f32(vc)
    q = rng.normal(size=(t, qh * d)).astype(np.float32)
    k = rng.normal(size=(t, kvw)).astype(np.float32)
    v = rng.normal(size=(t, kvw)).astype(np.float32)
    ref, n_ref = oracle.causal_gqa(q, k, v, qh, kvh, d, kc, vc, start, threads=8)
    out = be.allocate_f32(q.shape)
    st = noalloc(be, out, be.upload_f32(q), be.upload_f32(k), be.upload_f32(v), bkc, bvc, cap, start, t,
                 (qh, kvh, d))
    assert st == 0, L.mf_last_error().decode()
    assert n_ref == start + t
    close(be.read_f32(out), ref)
    assert np.array_equal(be.read_f32(bkc), kc)
    assert np.array_equal(be.read_f32(bvc), vc)


def test_noalloc_gqa_rejects_partials_beyond_static_scratch(be):
    from runtime_b200 import _lib

    L = _lib.load()
    # 16 tokens take the decode kernel: 16 tokens x 32 heads x ceil(4096/64)
    # key chunks x 66 floats x 4 B = 8.8 MB of partials > 4 MiB.
    qh, kvh, d, t, cap = 32, 8, 64, 16, 4096
    q = be.allocate_f32((t, qh * d))
    kv = be.allocate_f32((t, kvh * d))
    kc, vc = be.allocate_f32((cap, kvh * d)), be.allocate_f32((cap, kvh * d))
    out = be.upload_f32(np.full((t, qh * d), 7.0, np.float32))
    st = noalloc(be, out, q, kv, kv, kc, vc, cap, cap - t, t, (qh, kvh, d))
    assert st == RESOURCE_LIMIT, st
    assert b"static scratch" in L.mf_last_error()
    # Refused before any work: output and caches untouched.
    assert np.all(be.read_f32(out) == 7.0)
    assert not be.read_f32(kc).any()
