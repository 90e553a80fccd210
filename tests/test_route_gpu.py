"""Capacity-ceiling routing on the GPU vs the reference Router (golden) and
the C oracle -- bit-exact.  Mirrors tests/test_orchestration.cpp's Phase B
(capacity 20 with 400 of 500 tokens on expert 0 -> exactly 380 reroutes;
unlimited capacity never reroutes; a 90%-on-one-expert stress batch)."""
import numpy as np
import pytest

import aem_oracle as O
import cases
import native

pytestmark = pytest.mark.gpu


def _route(cuda, prim, sec, pos, cap, e, workspace=True):
    import torch
    from aethermoe_b200 import _lib
    n = len(prim)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(cuda)  # noqa: E731
    p, s, q = t(prim), t(sec), t(pos)
    out = torch.full((max(n, 1),), -1, dtype=torch.int32, device=cuda)
    ws_bytes = _lib.lib().aem_capacity_route_workspace(n, e)
    ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=cuda) if workspace else None
    st = _lib.lib().aem_capacity_route(
        p.data_ptr(), s.data_ptr(), q.data_ptr(), n, e,
        _lib.CAPACITY_UNLIMITED if cap is None else cap, out.data_ptr(),
        ws.data_ptr() if workspace else None, ws_bytes if workspace else 0,
        torch.cuda.current_stream().cuda_stream)
    return st, out[:n].cpu().numpy()


@pytest.mark.parametrize("name", sorted(cases.routing_cases()))
def test_matches_reference_router(cuda, golden, name):
    prim, sec, pos, cap, e, shards = cases.routing_cases()[name]
    st, eff = _route(cuda, prim, sec, pos, cap, e)
    assert st == 0
    np.testing.assert_array_equal(eff, golden["routing"][f"{name}/effective"])


def test_overflow_exactly_380(cuda):
    prim, sec, pos, cap, e, _ = cases.routing_cases()["overflow_400_of_500"]
    st, eff = _route(cuda, prim, sec, pos, cap, e, workspace=False)
    assert st == 0
    assert int((eff != prim).sum()) == 380
    assert np.all(eff[eff != prim] == sec[eff != prim])


def test_unlimited_capacity_never_reroutes(cuda):
    prim, sec, pos, _, e, _ = cases.routing_cases()["unlimited_random"]
    st, eff = _route(cuda, prim, sec, pos, None, e)
    assert st == 0
    np.testing.assert_array_equal(eff, prim)


@pytest.mark.parametrize("n,e,cap", [(0, 4, 3), (1, 1, 0), (2049, 7, 100), (100_000, 64, 1500),
                                     (300_000, 256, 900), (98_304, 64, 1920)])
def test_random_batches_vs_c_oracle(cuda, n, e, cap):
    rng = np.random.default_rng(n + e)
    prim = (rng.zipf(1.3, size=n) - 1) % e
    sec = rng.integers(0, e, size=n)
    pos = rng.permutation(n)
    st, eff = _route(cuda, prim, sec, pos, cap, e)
    assert st == 0
    np.testing.assert_array_equal(eff, native.capacity_assign(prim, sec, pos, cap))


def test_duplicate_position_is_reported(cuda):
    from aethermoe_b200 import _lib
    prim = np.zeros(10, np.int32)
    pos = np.arange(10)
    pos[3] = 7
    st, _ = _route(cuda, prim, prim, pos, 2, 4)
    assert st == _lib.AEM_EDEVICE
    assert "permutation" in _lib.last_error()
    # the library stays usable afterwards
    st, eff = _route(cuda, prim, prim, np.arange(10), 2, 4)
    assert st == 0


def test_expert_out_of_range_is_reported(cuda):
    from aethermoe_b200 import _lib
    prim = np.array([0, 1, 9, 2], np.int32)
    st, _ = _route(cuda, prim, prim, np.arange(4), 2, 4)
    assert st == _lib.AEM_EDEVICE
