"""Boundary semantics of the handle tier on a device: injected failures,
resource limits, pollable fences, the lease and the fence-retirement queue.

The reference pins these in its deferred test backend
(crates/executor-core/tests/model_executor.rs:369, `inject_copy_failure`)
and in the engine-api contract: limits and admission before any mutation
(crates/engine-api/src/resources.rs:6-11, crates/backend-cpu/src/storage.rs),
nonblocking completions (resources.rs:89-99), BackendLease
(crates/engine-api/src/backend.rs:25-62) and FenceRetirement
(resources.rs:143-185).  Every failure here is made on the host (an injected
status or a refused admission); no device fault is provoked.
"""
import numpy as np
import pytest

from runtime_b200.backend import CudaBackend, ExecutorError

pytestmark = pytest.mark.gpu

MiB = 1 << 20


def kinds(fn):
    with pytest.raises(ExecutorError) as e:
        fn()
    return e.value.kind


def busy(be, src, dst, copies=40):
    """Queue enough device work that a fence submitted after it is pending
    when first polled (each copy moves 2 x 256 MiB)."""
    for _ in range(copies):
        be.copy(dst, src)


@pytest.fixture(scope="module")
def be():
    b = CudaBackend(0)
    yield b
    b.close()


def test_injected_fence_failure_then_next_fence_succeeds(be):
    be.inject_failure("fence")
    f = be.fence()
    assert kinds(lambda: f.wait()) == "BackendFailure"
    f.release()
    g = be.fence()
    assert g.wait() == ()
    g.release()


def test_injected_allocation_failure_allocates_nothing(be):
    before = be.resource_report()
    be.inject_failure("allocation")
    assert kinds(lambda: be.allocate_f32((1024,))) == "BackendFailure"
    assert be.resource_report() == before
    buf = be.allocate_f32((1024,))           # the next allocation succeeds
    assert be.resource_report()["scratch_bytes"] == before["scratch_bytes"] + 4096
    buf.release()
    assert be.resource_report() == before


def test_injected_readback_failure_then_next_readback_succeeds(be):
    x = np.arange(64, dtype=np.float32)
    buf = be.upload_f32(x)
    be.inject_failure("readback")
    r = be.read_f32_async(buf)
    assert kinds(lambda: r.wait()) == "BackendFailure"
    r.release()
    assert np.array_equal(be.read_f32(buf), x)


def test_unknown_failure_kind_is_rejected(be):
    from runtime_b200 import _lib

    assert _lib.load().mf_inject_failure(be.handle, 9) == 1  # InvalidArgument


def test_allocation_limits_are_resource_limits_and_allocate_nothing():
    with CudaBackend(0, limits={"max_allocation_bytes": MiB, "max_total_bytes": 3 * MiB}) as b:
        empty = b.resource_report()
        assert kinds(lambda: b.allocate_f32((MiB // 4 + 1,))) == "ResourceLimit"
        assert b.resource_report() == empty and b.peak_accounted_bytes() == 0
        bufs = [b.allocate_f32((MiB // 4,)) for _ in range(3)]   # 3 MiB: at the total cap
        assert kinds(lambda: b.allocate_f32((1,))) == "ResourceLimit"
        assert kinds(lambda: b.upload_u8(np.zeros(16, np.uint8))) == "ResourceLimit"
        assert b.resource_report()["scratch_bytes"] == 3 * MiB
        bufs[0].release()
        b.allocate_f32((MiB // 4,))                                # room again
        assert b.peak_accounted_bytes() == 3 * MiB
        assert b.capabilities().max_allocation_bytes == MiB


def test_pending_operation_limit():
    with CudaBackend(0, limits={"max_pending_operations": 2}) as b:
        f1, f2 = b.fence(), b.fence()
        assert b.resource_report()["pending_operations"] == 2
        assert kinds(lambda: b.fence()) == "ResourceLimit"
        buf = b.allocate_f32((4,))
        assert kinds(lambda: b.read_f32_async(buf)) == "ResourceLimit"
        f1.wait()
        f1.release()
        f3 = b.fence()                                   # a slot is free again
        for f in (f2, f3):
            f.wait()
            f.release()
        assert b.resource_report()["pending_operations"] == 0


def test_fence_is_pending_then_ready(be):
    src = be.allocate_f32((64 * MiB,))
    dst = be.allocate_f32((64 * MiB,))
    busy(be, src, dst)
    f = be.fence()
    assert f.poll() is None          # the copies are still running
    assert f.wait() == ()
    assert f.poll() == ()            # a fence stays ready
    f.release()
    src.release()
    dst.release()


def test_lease_distinguishes_instances_with_equal_identity():
    with CudaBackend(0, owner=7) as a, CudaBackend(0, owner=7) as b:
        ia, ta = a.lease()
        ib, tb = b.lease()
        assert ia == ib == a.identity()
        assert ta != tb
        assert a.lease()[1] == ta    # stable for one instance
        a.advance_generation()
        assert a.lease()[0].generation == ia.generation + 1 and a.lease()[1] == ta


def test_retired_fence_keeps_buffers_until_terminal(be):
    from runtime_b200 import _lib

    base = be.resource_report()["scratch_bytes"]
    src = be.allocate_f32((64 * MiB,))
    dst = be.allocate_f32((64 * MiB,))
    busy(be, src, dst)
    f = be.fence()
    src_h, dst_h, f_h = src.handle, dst.handle, f.handle
    be.retire_fence(f, [src, dst])
    assert be.retired_fences_unresolved() == 1
    L = _lib.load()
    # The queue owns them now: the caller can release neither.
    assert L.mf_buffer_release(be.handle, src_h) == 1
    assert L.mf_fence_release(f_h) == 1
    assert L.mf_fence_retire(be.handle, f_h, None, 0) == 1      # already retired
    assert be.resource_report()["scratch_bytes"] == base + 2 * 256 * MiB
    for _ in range(100000):
        be.poll_retired_fences()
        if be.retired_fences_unresolved() == 0:
            break
    assert be.retired_fences_unresolved() == 0
    assert be.resource_report()["scratch_bytes"] == base
    assert be.resource_report()["pending_operations"] == 0
    assert L.mf_buffer_release(be.handle, dst_h) == 9           # released: no longer this backend's


def test_retirement_rejects_foreign_payload_without_change(be):
    with CudaBackend(0) as other:
        foreign = other.allocate_f32((16,))
        mine = be.allocate_f32((16,))
        f = be.fence()
        assert kinds(lambda: be.retire_fence(f, [mine, foreign])) == "WrongBackend"
        assert be.retired_fences_unresolved() == 0
        g = other.fence()
        assert kinds(lambda: be.retire_fence(g, [])) == "WrongBackend"
        # The caller still owns everything it offered.
        assert f.handle and g.handle and mine.handle and foreign.handle
        assert f.wait() == () and g.wait() == ()
        f.release()
        g.release()
        mine.release()
        foreign.release()
