"""The expert-parallel step plan computed on the device (one thread block,
parallel over ranks and experts) equals the host plan ``aem_ep_plan_peer``
field by field -- the host plan is the one the gloo replays verify -- on
payloads from real routings, with ranks left out, and on inconsistent or
over-capacity payloads that must be rejected."""
import ctypes

import numpy as np
import pytest

import aem_oracle as O

pytestmark = pytest.mark.gpu


def _payloads(rng, R, E, k, tl, live):
    from aethermoe_b200.moe import ep_payload
    rows = []
    for s in range(R):
        logits = rng.normal(size=(tl, E)).astype(np.float32) + O.zipf_bias(E)
        idx = O.topk_strict(logits, k + 1).astype(np.int32)
        eff = O.moe_route(idx, k, E, O.default_capacity(tl * R, k, E))
        rows.append(ep_payload(eff, tl, E, R, live))
    return np.stack(rows)


def _device_plan(cuda, pay, rank, live, caps):
    import torch
    from aethermoe_b200 import _lib
    R = pay.shape[0]
    E = _width_to_experts(pay.shape[1], R)
    all_d = torch.from_numpy(pay).to(cuda)
    plan_d = torch.zeros(ctypes.sizeof(_lib.EpPeerPlan), dtype=torch.uint8, device=cuda)
    groups_d = torch.full((2 * (E + 1),), -7, dtype=torch.int32, device=cuda)
    _lib.check(_lib.lib().aem_ep_plan_peer_device(all_d.data_ptr(), R, E, rank, live, *caps,
                                                  plan_d.data_ptr(), groups_d.data_ptr(), None),
               "aem_ep_plan_peer_device")
    torch.cuda.synchronize()
    raw = bytes(plan_d.cpu().numpy())
    return _lib.EpPeerPlan.from_buffer_copy(raw), groups_d.cpu().numpy()


def _host_plan(pay, rank, live, caps):
    from aethermoe_b200 import _lib
    R = pay.shape[0]
    E = _width_to_experts(pay.shape[1], R)
    plan = _lib.EpPeerPlan()
    groups = np.full(2 * (E + 1), -7, np.int32)
    p = np.ascontiguousarray(pay)
    _lib.check(_lib.lib().aem_ep_plan_peer(p.ctypes.data, R, E, rank, live, *caps,
                                           ctypes.byref(plan), groups.ctypes.data))
    return plan, groups


def _width_to_experts(w, R):
    from aethermoe_b200 import _lib
    return next(e for e in range(R, 257, R) if _lib.ep_payload_words(e, R) == w)


def _same(a, b, ga, gb, el):
    assert bytes(a) == bytes(b)
    np.testing.assert_array_equal(ga[:2 * (el + 1)], gb[:2 * (el + 1)])


@pytest.mark.parametrize("R,E,k", [(2, 8, 2), (4, 64, 6), (8, 64, 6), (8, 256, 8), (64, 256, 4)])
def test_device_plan_equals_host_plan(cuda, R, E, k):
    rng = np.random.default_rng(R * 1000 + E)
    tl = 96
    caps = (R * tl * k, R * tl, tl * min(R, k))
    for live in ((1 << R) - 1, ((1 << R) - 1) & ~(1 << (R // 2))):
        pay = _payloads(rng, R, E, k, tl, live)
        for rank in sorted({0, R - 1, R // 3}):
            if not (live >> rank) & 1:
                continue
            hp, hg = _host_plan(pay, rank, live, caps)
            assert hp.ok == 1
            dp, dg = _device_plan(cuda, pay, rank, live, caps)
            _same(dp, hp, dg, hg, E // R)


def test_device_plan_rejects_what_the_host_rejects(cuda):
    rng = np.random.default_rng(9)
    R, E, k, tl = 4, 16, 3, 50
    live = (1 << R) - 1
    pay = _payloads(rng, R, E, k, tl, live)
    caps = (R * tl * k, R * tl, tl * min(R, k))
    bads = []
    b = pay.copy(); b[1, E + 1] += 1_000_000; bads.append((b, caps))   # more pairs than units
    b = pay.copy(); b[2, 3] = b[2, 2] - 1; bads.append((b, caps))         # starts decrease
    b = pay.copy(); b[0, 0] = 5; bads.append((b, caps))                   # starts not at 0
    b = pay.copy(); b[3, E + 3 + R] += 1000; bads.append((b, caps))       # half-A units > units
    b = pay.copy(); b[1, 2 * E + 3 + R] += 1000; bads.append((b, caps))   # half-A pairs > pairs
    bads.append((pay, (10, caps[1], caps[2])))                            # units over capacity
    bads.append((pay, (caps[0], 10, caps[2])))                            # pairs over capacity
    bads.append((pay, (caps[0], caps[1], 10)))                            # returns over capacity
    for bp, cp in bads:
        for rank in range(R):
            hp, hg = _host_plan(bp, rank, live, cp)
            dp, dg = _device_plan(cuda, bp, rank, live, cp)
            assert hp.ok == 0 and dp.ok == 0
            _same(dp, hp, dg, hg, E // R)
