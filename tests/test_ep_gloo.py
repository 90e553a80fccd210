"""The expert-parallel host plumbing on CPU ranks (gloo, world size 2 and 4).

Each rank gates its own token slice (oracle), all-gathers its per-(slot,
expert) primary counts, plans its global rank offsets with the library's
``aem_ep_plan_bases``, routes its units locally, all-gathers its expert
starts and plans the exchange with ``aem_ep_plan_exchange``.  Rank 0 checks
that the distributed decision equals the capacity rule on the whole batch
(bit-exact) and that every rank's receive segments are exactly the peers'
send segments.  It then replays one peer-memory exchange with the plans of
``aem_ep_plan_peer`` (the function the layer runs on the device): every
pushed pair and unit lands on a distinct row inside the destination's
received range, every unit row of the destination's grouped GEMM holds a unit
of that row group's expert pointing at its token's pair, and every
pair sum returned lands on the row the source's combine reads for that
(token, destination).  No GPU involved.
"""
import os
import socket
import tempfile

import numpy as np
import pytest

import aem_oracle as O

T, E, K_TOP = 1200, 16, 3


def _inputs():
    rng = np.random.default_rng(21)
    logits = rng.normal(size=(T, E)).astype(np.float32) + O.zipf_bias(E)
    return O.topk_strict(logits, K_TOP + 1).astype(np.int32)


def _rank(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    from aethermoe_b200.moe import ep_plan_bases, ep_plan_exchange, ep_plan_peer, ep_payload
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    idx = _inputs()
    tl = T // world
    cap = O.default_capacity(T, K_TOP, E)
    loc = idx[rank * tl:(rank + 1) * tl]
    counts = torch.from_numpy(O.ep_local_counts(loc, K_TOP, E))
    allc = [torch.zeros_like(counts) for _ in range(world)]
    dist.all_gather(allc, counts)
    base = ep_plan_bases(torch.stack(allc).numpy(), rank)
    prim, sec, _, _, slot = O.moe_units(loc, K_TOP, E)
    eff = np.empty_like(prim)
    seen = {}
    for u in range(len(prim)):  # local stable rank within (slot, primary) in position order
        key = (int(slot[u]), int(prim[u]))
        rk = int(base[key]) + seen.get(key, 0)
        seen[key] = seen.get(key, 0) + 1
        eff[u] = prim[u] if rk < cap else sec[u]
    starts = np.zeros(E + 1, np.int32)
    starts[1:] = np.cumsum(np.bincount(eff, minlength=E))
    alls = [torch.zeros(E + 1, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(alls, torch.from_numpy(starts))
    plan = ep_plan_exchange(torch.stack(alls).numpy(), rank)
    # peer-memory exchange plan: starts, pair counts, half-A counts per rank
    payload = torch.from_numpy(ep_payload(eff, tl, E, world))
    allp = [torch.zeros_like(payload) for _ in range(world)]
    dist.all_gather(allp, payload)
    caps = (world * tl * K_TOP, world * tl, tl * min(world, K_TOP))
    pp, pg = ep_plan_peer(torch.stack(allp).numpy(), rank, *caps)  # every rank live
    np.savez(os.path.join(outdir, f"r{rank}.npz"), eff=eff, starts=starts,
             so=plan[0], sc=plan[1], ro=plan[2], rc=plan[3], groups=plan[4], pgroups=pg,
             payload=payload.numpy(), **{"p_" + key: np.asarray(v) for key, v in pp.items()})
    dist.barrier()
    dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_distributed_routing_and_exchange_plan(world):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as outdir:
        mp.start_processes(_rank, args=(world, _port(), outdir), nprocs=world, join=True,
                           start_method="spawn")
        res = [dict(np.load(os.path.join(outdir, f"r{r}.npz"))) for r in range(world)]
    idx = _inputs()
    tl = T // world
    want = O.moe_route(idx, K_TOP, E, O.default_capacity(T, K_TOP, E))
    got = np.concatenate([r["eff"].reshape(K_TOP, tl) for r in res], axis=1).reshape(-1)
    np.testing.assert_array_equal(got, want)
    el = E // world
    for r in range(world):
        for p in range(world):
            # what r receives from p is what p sends to r, in the same segment layout
            assert res[r]["rc"][p] == res[p]["sc"][r]
            seg = res[p]["starts"][(r + 1) * el] - res[p]["starts"][r * el]
            assert res[p]["sc"][r] == seg
        assert res[r]["groups"][-1] == res[r]["rc"].sum()
        assert np.all(np.diff(res[r]["groups"]) >= 0)


def _half_major_order(eff, tl):
    """The source's expert-sorted units, half A (tokens < ceil(tl/2)) first
    inside every expert, each part in unit order u = j*tl + t."""
    half = (tl + 1) // 2
    u = np.arange(len(eff))
    return np.lexsort((u, (u % tl) >= half, eff))


def _replay(res, world, tl, live):
    """Simulates the pushes of one step from the saved per-rank plans: every
    pair and unit lands on a distinct row of the destination's received range
    for its half, every unit row lies in its half's row group of its expert and
    points at its token's pair, and every returned pair sum lands on the row
    the source's combine reads for that (token, destination)."""
    el = E // world
    half_t = (tl + 1) // 2
    ranks = [r for r in range(world) if (live >> r) & 1]
    xpair = {r: {} for r in ranks}  # row -> (source, token)
    units = {r: {} for r in ranks}  # row -> (source, unit)
    failed = 0
    for s_ in ranks:
        p = res[s_]["plan"]
        eff = res[s_]["eff"]
        order = _half_major_order(eff, tl)
        starts = np.zeros(E + 1, np.int64)
        starts[1:] = np.cumsum(np.bincount(eff, minlength=E))
        dest = eff.reshape(K_TOP, tl) // el
        pl = np.full((world, tl), -1)
        for r in range(world):
            if not (live >> r) & 1:
                failed += int((dest == r).sum())
                continue
            has = (dest == r).any(axis=0)
            pl[r, has] = np.arange(has.sum())
            assert has[:half_t].sum() == p["send_pair_a"][r]
            for t in np.nonzero(has)[0]:
                row = int(p["dst_pair_off"][r]) + pl[r, t]
                assert row not in xpair[r]
                xpair[r][row] = (s_, t)
            for e in range(r * el, (r + 1) * el):
                seg = order[starts[e]:starts[e + 1]]
                in_a = (seg % tl) < half_t
                for h, part in ((0, seg[in_a]), (1, seg[~in_a])):
                    for q, u in enumerate(part):
                        pos = int(p["dst_unit_off"][h][e]) + q
                        assert pos not in units[r]
                        units[r][pos] = (s_, u, h)
        res[s_]["_pl"] = pl
    ret = {r: {} for r in ranks}
    for r in ranks:
        p = res[r]["plan"]
        g = res[r]["groups"]
        na = int(p["units_in_a"])
        assert sorted(xpair[r]) == list(range(int(p["pairs_in"])))
        assert sorted(units[r]) == list(range(int(p["units_in"])))
        assert g[0][0] == 0 and g[0][-1] == na == g[1][0] and g[1][-1] == p["units_in"]
        for pos, (s_, u, h) in units[r].items():
            e = int(res[s_]["eff"][u])
            assert (pos < na) == (h == 0)
            grp = np.searchsorted(g[h], pos, side="right") - 1
            assert grp == e - r * el                      # the local expert's row group
            prow = int(res[s_]["plan"]["dst_pair_off"][r]) + res[s_]["_pl"][r, u % tl]
            assert xpair[r][prow] == (s_, u % tl)         # the unit's token
        roff, pa = p["recv_pair_off"], p["recv_pair_a"]
        for prow, (s_, t) in xpair[r].items():
            assert roff[s_] <= prow < roff[s_ + 1]
            assert (prow - roff[s_] < pa[s_]) == (t < half_t)  # the pair's half
            row = int(p["ret_off"][s_]) + prow - int(roff[s_])
            assert row not in ret[s_]
            ret[s_][row] = (r, t)
    for s_ in ranks:
        p = res[s_]["plan"]
        assert sorted(ret[s_]) == list(range(int(p["pairs_out"])))
        for row, (r, t) in ret[s_].items():  # the combine reads send_pair_off[r] + pl[r][t]
            assert int(p["send_pair_off"][r]) + res[s_]["_pl"][r, t] == row
    return failed


def _replay_peer_exchange(res, world, tl):
    from aethermoe_b200.moe import ep_plan_peer
    pay = np.stack([r["payload"] for r in res])
    caps = (world * tl * K_TOP, world * tl, tl * min(world, K_TOP))
    for rank, r in enumerate(res):
        plan, groups = ep_plan_peer(pay, rank, *caps)
        assert plan["ok"] == 1
        r["plan"], r["groups"] = plan, groups
    _replay(dict(enumerate(res)), world, tl, (1 << world) - 1)


@pytest.mark.parametrize("world", [2, 4])
def test_peer_exchange_plan_replay(world):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as outdir:
        mp.start_processes(_rank, args=(world, _port(), outdir), nprocs=world, join=True,
                           start_method="spawn")
        res = [dict(np.load(os.path.join(outdir, f"r{r}.npz"))) for r in range(world)]
    _replay_peer_exchange(res, world, T // world)


def test_peer_plan_rejects_overflow():
    """Counts beyond a receive capacity give ok = 0 on every rank."""
    from aethermoe_b200.moe import ep_plan_peer
    R, E_ = 2, 4
    # rank 0 sends 5 units / 3 pairs to rank 1, rank 1 sends 4 units / 2 pairs to itself
    pay = np.array([[0, 1, 2, 4, 7, 1, 3],
                    [0, 0, 0, 2, 4, 0, 2]], np.int32)
    for rank in range(R):
        ok, _ = ep_plan_peer(pay, rank, 100, 100, 100)
        assert ok["ok"] == 1
        bad, groups = ep_plan_peer(pay, rank, 8, 100, 100)  # rank 1 receives 9 units
        assert bad["ok"] == 0 and bad["units_in"] == 0 and not groups.any()
    # a pair count larger than the unit count is inconsistent
    pay2 = pay.copy()
    pay2[0, E_ + 1] = 3  # 2 units to rank 0 but 3 pairs
    assert ep_plan_peer(pay2, 0, 100, 100, 100)[0]["ok"] == 0


def test_peer_exchange_plan_with_a_rank_left_out():
    """A rank marked unhealthy takes no part: its tokens leave the batch, the
    capacity rule runs over the live ranks' tokens only, units whose expert
    lives on the dead rank fail, and the live ranks' pushes still tile every
    receive range exactly (host replay of the plans for live mask 0b1011)."""
    from aethermoe_b200.moe import ep_plan_peer, ep_payload
    world, dead = 4, 2
    live_ranks = [r for r in range(world) if r != dead]
    mask = sum(1 << r for r in live_ranks)
    idx = _inputs()
    tl = T // world
    cap = O.default_capacity(T, K_TOP, E)
    # the distributed rule with the dead rank's counts absent == the rule on the live tokens
    sub = np.concatenate([idx[r * tl:(r + 1) * tl] for r in live_ranks])
    eff_all = O.moe_route(sub, K_TOP, E, cap).reshape(K_TOP, len(live_ranks) * tl)
    res = {}
    payload = np.full((world, ep_payload(np.zeros(K_TOP * tl, np.int64), tl, E, world).size),
                      12345, np.int32)  # whatever a dead rank left behind is ignored
    for i, r in enumerate(live_ranks):
        eff = eff_all[:, i * tl:(i + 1) * tl].reshape(-1)
        payload[r] = ep_payload(eff, tl, E, world, mask)
        res[r] = dict(eff=eff)
    caps = (world * tl * K_TOP, world * tl, tl * min(world, K_TOP))
    for r in live_ranks:
        plan, groups = ep_plan_peer(payload, r, *caps, live=mask)
        assert plan["ok"] == 1
        res[r]["plan"], res[r]["groups"] = plan, groups
    assert _replay(res, world, tl, mask) > 0  # the dead rank's experts had units: they fail


def test_peer_plan_rejects_overflow():
    """Counts beyond a receive capacity or inconsistent counts give ok = 0."""
    from aethermoe_b200.moe import ep_plan_peer, ep_payload
    R, E_, tl, k = 2, 4, 6, 2
    rng = np.random.default_rng(5)
    effs = [rng.integers(0, E_, size=k * tl) for _ in range(R)]
    pay = np.stack([ep_payload(e, tl, E_, R) for e in effs])
    units_to = [sum(int((e // 2 == r).sum()) for e in effs) for r in range(R)]
    for rank in range(R):
        assert ep_plan_peer(pay, rank, 100, 100, 100)[0]["ok"] == 1
        bad, groups = ep_plan_peer(pay, rank, max(units_to) - 1, 100, 100)
        assert bad["ok"] == 0 and bad["units_in"] == 0 and not groups.any()
    for col, delta in ((E_ + 1, 1000), (2 * E_ + 3 + R, 1000), (E_ + 3 + R, 1000), (0, 1)):
        p2 = pay.copy()
        p2[0, col] += delta  # too many pairs / half-A pairs / half-A units; starts not at 0
        assert ep_plan_peer(p2, 0, 100, 100, 100)[0]["ok"] == 0
