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
    from aethermoe_b200.moe import ep_plan_bases, ep_plan_exchange, ep_plan_peer
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
    # peer-memory exchange plan: starts + pair counts per destination rank
    el = E // world
    dest = (eff.reshape(K_TOP, tl) // el)  # destination rank of every unit
    pcnt = np.array([(dest == r).any(axis=0).sum() for r in range(world)], np.int32)
    payload = torch.from_numpy(np.concatenate([starts, pcnt]).astype(np.int32))
    allp = [torch.zeros_like(payload) for _ in range(world)]
    dist.all_gather(allp, payload)
    caps = (world * tl * K_TOP, world * tl, tl * min(world, K_TOP))
    pp, pg = ep_plan_peer(torch.stack(allp).numpy(), rank, *caps)  # every rank live
    np.savez(os.path.join(outdir, f"r{rank}.npz"), eff=eff, starts=starts,
             so=plan[0], sc=plan[1], ro=plan[2], rc=plan[3], groups=plan[4], pgroups=pg,
             **{"p_" + key: np.asarray(v) for key, v in pp.items()})
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


def _replay_peer_exchange(res, world, tl):
    """Simulates the pushes of one step from the saved per-rank plans."""
    el = E // world
    plans = [{k[2:]: r[k] for k in r if k.startswith("p_")} for r in res]
    assert all(int(p["ok"]) == 1 for p in plans)
    # destination-side arrays, filled by the sources' pushes
    xpair = [dict() for _ in range(world)]  # row -> (source, token)
    units = [dict() for _ in range(world)]  # row -> (source, unit, pair row)
    for s_ in range(world):
        eff = res[s_]["eff"]
        order = np.argsort(eff, kind="stable")  # expert-grouped units, position order inside
        starts = res[s_]["starts"]
        dest = eff.reshape(K_TOP, tl) // el
        pl = np.full((world, tl), -1)
        for r in range(world):
            has = (dest == r).any(axis=0)
            pl[r, has] = np.arange(has.sum())
            for t in np.nonzero(has)[0]:
                row = int(plans[s_]["dst_pair_off"][r]) + pl[r, t]
                assert row not in xpair[r]
                xpair[r][row] = (s_, t)
            for e in range(r * el, (r + 1) * el):
                for i in range(starts[e], starts[e + 1]):
                    u = order[i]
                    pos = int(plans[s_]["dst_unit_off"][e]) + (i - starts[e])
                    assert pos not in units[r]
                    units[r][pos] = (s_, u, int(plans[s_]["dst_pair_off"][r]) + pl[r, u % tl])
        res[s_]["_pl"] = pl
    ret = [dict() for _ in range(world)]  # source-side return rows
    for r in range(world):
        p = plans[r]
        assert sorted(xpair[r]) == list(range(int(p["pairs_in"])))
        assert sorted(units[r]) == list(range(int(p["units_in"])))
        g = res[r]["pgroups"]
        for pos, (s_, u, prow) in units[r].items():
            e = int(res[s_]["eff"][u])
            grp = np.searchsorted(g, pos, side="right") - 1
            assert grp == e - r * el                        # the local expert's row group
            assert xpair[r][prow] == (s_, u % tl)           # the unit's token
        roff = p["recv_pair_off"]
        for prow, (s_, t) in xpair[r].items():
            assert roff[s_] <= prow < roff[s_ + 1]
            row = int(p["ret_off"][s_]) + prow - int(roff[s_])
            assert row not in ret[s_]
            ret[s_][row] = (r, t)
    for s_ in range(world):
        p = plans[s_]
        assert sorted(ret[s_]) == list(range(int(p["pairs_out"])))
        pl = res[s_]["_pl"]
        for row, (r, t) in ret[s_].items():  # the combine reads send_pair_off[r] + pl[r][t]
            assert int(p["send_pair_off"][r]) + pl[r, t] == row


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
    from aethermoe_b200.moe import ep_plan_peer
    world, dead = 4, 2
    live = [r for r in range(world) if r != dead]
    mask = sum(1 << r for r in live)
    idx = _inputs()
    tl = T // world
    el = E // world
    cap = O.default_capacity(T, K_TOP, E)
    # the distributed rule with the dead rank's counts absent == the rule on the live tokens
    sub = np.concatenate([idx[r * tl:(r + 1) * tl] for r in live])
    eff_all = O.moe_route(sub, K_TOP, E, cap).reshape(K_TOP, len(live) * tl)
    res = {}
    payload = np.zeros((world, E + 1 + world), np.int32)
    for i, r in enumerate(live):
        eff = eff_all[:, i * tl:(i + 1) * tl].reshape(-1)
        starts = np.zeros(E + 1, np.int32)
        starts[1:] = np.cumsum(np.bincount(eff, minlength=E))
        dest = eff.reshape(K_TOP, tl) // el
        pcnt = np.array([(dest == q).any(axis=0).sum() if q != dead else 0 for q in range(world)])
        payload[r] = np.concatenate([starts, pcnt])
        res[r] = dict(eff=eff, starts=starts)
    payload[dead] = 12345  # whatever a dead rank left behind is ignored
    caps = (world * tl * K_TOP, world * tl, tl * min(world, K_TOP))
    for r in live:
        pp, pg = ep_plan_peer(payload, r, *caps, live=mask)
        assert pp["ok"] == 1
        res[r].update(pgroups=pg, **{"p_" + key: np.asarray(v) for key, v in pp.items()})
    # replay the pushes of the live ranks
    xpair = {r: {} for r in live}
    units = {r: {} for r in live}
    ret = {r: {} for r in live}
    failed = 0
    for s_ in live:
        eff, starts = res[s_]["eff"], res[s_]["starts"]
        order = np.argsort(eff, kind="stable")
        dest = eff.reshape(K_TOP, tl) // el
        pl = np.full((world, tl), -1)
        for r in live:
            has = (dest == r).any(axis=0)
            pl[r, has] = np.arange(has.sum())
            for t in np.nonzero(has)[0]:
                row = int(res[s_]["p_dst_pair_off"][r]) + pl[r, t]
                assert row not in xpair[r]
                xpair[r][row] = (s_, t)
            for e in range(r * el, (r + 1) * el):
                for i in range(starts[e], starts[e + 1]):
                    pos = int(res[s_]["p_dst_unit_off"][e]) + (i - starts[e])
                    assert pos not in units[r]
                    units[r][pos] = (s_, order[i])
        failed += int((dest == dead).sum())
        res[s_]["_pl"] = pl
    assert failed > 0  # the dead rank's experts had units: those fail
    for r in live:
        p = res[r]
        assert sorted(xpair[r]) == list(range(int(p["p_pairs_in"])))
        assert sorted(units[r]) == list(range(int(p["p_units_in"])))
        for pos, (s_, u) in units[r].items():
            e = int(res[s_]["eff"][u])
            grp = np.searchsorted(p["pgroups"], pos, side="right") - 1
            assert grp == e - r * el
        roff = p["p_recv_pair_off"]
        for prow, (s_, t) in xpair[r].items():
            row = int(p["p_ret_off"][s_]) + prow - int(roff[s_])
            assert row not in ret[s_]
            ret[s_][row] = (r, t)
    for s_ in live:
        assert sorted(ret[s_]) == list(range(int(res[s_]["p_pairs_out"])))
        for row, (r, t) in ret[s_].items():
            assert int(res[s_]["p_send_pair_off"][r]) + res[s_]["_pl"][r, t] == row
