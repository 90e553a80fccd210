"""aem_capacity_route_static: capacity routing that allocates no device memory.

Some callers cannot call cudaMalloc while they run (a serving loop that
reserves its device budget up front, or one that cannot afford the
device-wide synchronisation of cudaFree mid-step).  This entry point keeps
its scratch in a fixed array inside the library instead.  These tests call it
through the C ABI and check it against the allocating entry point
(aem_capacity_route) -- routing is integer work, so the tolerance is zero --
on two calls in a row with different sizes, so that anything the first call
leaves in the shared array and the second call fails to reset would show.
The file sorts last so a run that stops at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _route(cuda, name, prim, sec, pos, cap, e):
    import torch
    from aethermoe_b200 import _lib
    L = _lib.lib()
    n = len(prim)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(cuda)  # noqa: E731
    p, s, q = t(prim), t(sec), t(pos)
    out = torch.full((max(n, 1),), -1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    c = _lib.CAPACITY_UNLIMITED if cap is None else cap
    if name == "static":
        st = L.aem_capacity_route_static(p.data_ptr(), s.data_ptr(), q.data_ptr(), n, e, c,
                                         out.data_ptr(), stream)
    else:
        st = L.aem_capacity_route(p.data_ptr(), s.data_ptr(), q.data_ptr(), n, e, c,
                                  out.data_ptr(), None, 0, stream)
    torch.cuda.synchronize()
    return st, out[:n].cpu().numpy()


def _batch(seed, n, e):
    rng = np.random.default_rng(seed)
    prim = (rng.zipf(1.3, size=n) - 1) % e
    return prim, rng.integers(0, e, size=n), rng.permutation(n)


def test_static_matches_allocating_entry_point_on_two_calls(cuda):
    from aethermoe_b200 import _lib
    for seed, n, e, cap in [(1, 250_000, 64, 2500), (2, 1_000, 8, 40)]:
        prim, sec, pos = _batch(seed, n, e)
        st, got = _route(cuda, "static", prim, sec, pos, cap, e)
        assert st == _lib.AEM_OK, _lib.last_error()
        st, want = _route(cuda, "alloc", prim, sec, pos, cap, e)
        assert st == _lib.AEM_OK, _lib.last_error()
        np.testing.assert_array_equal(got, want)
        assert (got != prim).any()  # the capacity ceiling rerouted something


def test_static_rejects_sizes_beyond_its_scratch(cuda):
    from aethermoe_b200 import _lib
    L = _lib.lib()
    n = 262_144 + 1  # AEM_ROUTE_STATIC_MAX_UNITS + 1
    st = L.aem_capacity_route_static(None, None, None, n, 8, 10, None, None)
    assert st == _lib.AEM_EINVAL
    assert "maximum" in _lib.last_error()


def test_static_reports_a_bad_permutation_then_recovers(cuda):
    from aethermoe_b200 import _lib
    prim, sec, pos = _batch(3, 5_000, 16)
    bad = pos.copy()
    bad[10] = bad[11]
    st, _ = _route(cuda, "static", prim, sec, bad, 100, 16)
    assert st == _lib.AEM_EDEVICE
    st, got = _route(cuda, "static", prim, sec, pos, 100, 16)
    assert st == _lib.AEM_OK
    _, want = _route(cuda, "alloc", prim, sec, pos, 100, 16)
    np.testing.assert_array_equal(got, want)
