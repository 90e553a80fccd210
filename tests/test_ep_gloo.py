"""The expert-parallel host plumbing on CPU ranks (gloo, world size 2 and 4).

Each rank gates its own token slice (oracle), all-gathers its per-(slot,
expert) primary counts, plans its global rank offsets with the library's
``aem_ep_plan_bases``, routes its units locally, all-gathers its expert
starts and plans the exchange with ``aem_ep_plan_exchange``.  Rank 0 checks
that the distributed decision equals the capacity rule on the whole batch
(bit-exact) and that every rank's receive segments are exactly the peers'
send segments.  No GPU involved: the same host functions the NCCL layer uses.
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
    from aethermoe_b200.moe import ep_plan_bases, ep_plan_exchange
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
    np.savez(os.path.join(outdir, f"r{rank}.npz"), eff=eff, starts=starts,
             so=plan[0], sc=plan[1], ro=plan[2], rc=plan[3], groups=plan[4])
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
