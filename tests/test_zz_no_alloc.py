"""The non-allocating causal GQA entry point against the allocating one.

`mfk_causal_gqa_noalloc` serves callers that cannot call cudaMalloc (a host
whose memory manager already owns the device's memory, or a decode loop that
must not make a call that may synchronize the device): its split-key
partials live in a static device array instead of backend scratch.  Each
call here runs the same decode-shaped attention through `mf_causal_gqa`
(handle tier, backend scratch) and through the non-allocating entry point
on an identical copy of the caches, twice in a row, and requires equal
outputs and caches within the GQA tolerance of the other tests.

This file is named to be collected last, and it builds its own backend, so
it passes alone in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-5, 1e-4  # the GQA tolerance of tests/test_layer_gpu.py


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


def test_noalloc_gqa_matches_allocating_entry_point_twice(be):
    from runtime_b200 import _lib

    L = _lib.load()
    qh, kvh, d = 32, 8, 64
    cap, start = 1024, 700   # 700+ visible rows: the split-key path, so the scratch is used
    rng = np.random.default_rng(17)
    kc0 = rng.normal(size=(cap, kvh * d)).astype(np.float32)
    vc0 = rng.normal(size=(cap, kvh * d)).astype(np.float32)
    kc_a, vc_a = be.upload_f32(kc0), be.upload_f32(vc0)   # allocating path's caches
    kc_b, vc_b = be.upload_f32(kc0), be.upload_f32(vc0)   # non-allocating path's caches
    n_a, n_b = start, start
    for call in range(2):
        q = rng.normal(size=(1, qh * d)).astype(np.float32)
        k = rng.normal(size=(1, kvh * d)).astype(np.float32)
        v = rng.normal(size=(1, kvh * d)).astype(np.float32)
        bq, bk, bv = be.upload_f32(q), be.upload_f32(k), be.upload_f32(v)
        out_a = be.allocate_f32((1, qh * d))
        out_b = be.allocate_f32((1, qh * d))
        n_a = be.causal_gqa(out_a, bq, bk, bv, kc_a, vc_a, n_a, (qh, kvh, d))
        st = L.mfk_causal_gqa_noalloc(out_b.ptr, bq.ptr, bk.ptr, bv.ptr, kc_b.ptr, vc_b.ptr, cap, n_b, 1,
                                      qh, kvh, d, C.c_void_p(be.stream))
        assert st == 0, L.mf_last_error().decode()
        n_b += 1
        assert n_a == n_b == start + call + 1
        close(be.read_f32(out_b), be.read_f32(out_a))
        close(be.read_f32(kc_b), be.read_f32(kc_a))
        close(be.read_f32(vc_b), be.read_f32(vc_a))


def test_noalloc_gqa_rejects_partials_beyond_static_scratch(be):
    from runtime_b200 import _lib

    L = _lib.load()
    # 63 tokens x 32 heads x ceil(4096/256) chunks x 66 floats x 4 B = 8.5 MB > 4 MiB
    qh, kvh, d, t, cap = 32, 8, 64, 63, 4096
    q = be.allocate_f32((t, qh * d))
    kv = be.allocate_f32((t, kvh * d))
    kc, vc = be.allocate_f32((cap, kvh * d)), be.allocate_f32((cap, kvh * d))
    out = be.allocate_f32((t, qh * d))
    st = L.mfk_causal_gqa_noalloc(out.ptr, q.ptr, kv.ptr, kv.ptr, kc.ptr, vc.ptr, cap, cap - t, t, qh, kvh, d,
                                  C.c_void_p(be.stream))
    assert st == 8, st  # MF_RESOURCE_LIMIT
    assert b"static scratch" in L.mf_last_error()
