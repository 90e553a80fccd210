"""Tolerant expert-parallel steps on 2 GPUs against the oracle.

The contract is Router::route_batch_tolerant (src/orchestration/router.hpp:
127-234, exercised by tests/test_chaos.cpp:238-292): every (token, slot) unit
resolves to exactly one outcome -- its expert output, or ``failed`` -- never a
raised error and never a silently missing result; a rank that failed once is
remembered as unhealthy and later steps route around it.

Failures are made on the host, never on the GPU:
* ``marked``: after a healthy step, rank 1 stops taking part (it keeps its
  process until rank 0 is done) and rank 0's host marks it unhealthy before
  its next step;
* ``silent``: rank 1 skips a step while alive, so rank 0's bounded device
  waits (1 s) run out: that step fails on rank 0 with every unit flagged and
  a zero output, ``health()`` reports rank 1, and the next step routes around
  it without another wait.
After the failure rank 0 runs alone: its batch is its own tokens, the
capacity rule runs over them only, and the units whose expert lives on rank
1 fail.  Host rendezvous is a TCPStore, so no collective is left in flight.
Skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

import aem_oracle as O
import native

pytestmark = pytest.mark.gpu

CFG = dict(T=1024, d=256, f=384, E=8, k=2)


def _data():
    rng = np.random.default_rng(11)
    T, d, f, E = CFG["T"], CFG["d"], CFG["f"], CFG["E"]
    qu = rng.integers(-127, 128, size=(E, d, f), dtype=np.int8)
    su = (rng.random(size=(E, 1, f)) * 1e-4 + 2e-4).astype(np.float32)
    qd = rng.integers(-127, 128, size=(E, f, d), dtype=np.int8)
    sd = (rng.random(size=(E, 1, d)) * 1e-4 + 2e-4).astype(np.float32)
    gw = (rng.normal(size=(d, E)) / np.sqrt(d)).astype(np.float32)
    gb = O.zipf_bias(E)
    x = O.bf16_round(rng.normal(size=(T, d)).astype(np.float32))
    return gw, gb, qu, su, qd, sd, x


def _worker(rank, world, port, outdir, scenario):
    import torch
    from torch.distributed import TCPStore
    from aethermoe_b200 import _lib
    from aethermoe_b200.moe import EPLayer, ep_unique_id
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    store = TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    if rank == 0:
        store.set("uid", bytes(ep_unique_id()))
    uid = store.get("uid")
    T, E, k = CFG["T"], CFG["E"], CFG["k"]
    gw, gb, qu, su, qd, sd, x = _data()
    el, tl = E // world, T // world
    lo, hi = rank * el, (rank + 1) * el
    layer = EPLayer(uid, rank, world, gw, gb, qu[lo:hi], su[lo:hi], qd[lo:hi], sd[lo:hi], k,
                    capacity=O.default_capacity(T, k, E), device=rank, max_tokens=tl)
    layer.set_timeout(1.0)
    bits = (x[rank * tl:(rank + 1) * tl].view(np.uint32) >> 16).astype(np.uint16)
    xt = torch.from_numpy(bits.view(np.int16)).to(dev).view(torch.bfloat16)
    saved = {}
    out, failed = layer.forward_tolerant(xt, out_dtype=torch.float32)  # healthy step
    _, _, eff = layer.last_routing(tl)
    torch.cuda.synchronize()
    saved.update(out1=out.cpu().numpy(), failed1=failed.cpu().numpy(), eff1=eff.cpu().numpy())
    store.set(f"step1_{rank}", "1")
    store.wait([f"step1_{r}" for r in range(world)])
    if rank == 1:
        if scenario == "marked":
            store.set("r1_left", "1")
        store.wait(["r0_done"])  # alive but idle: takes no part in rank 0's steps
        layer.mark_unhealthy(0)  # the host learned rank 0 went on without it
        saved["health"] = np.array(sorted(layer.health()))
        layer.close()
        np.savez(os.path.join(outdir, f"{scenario}_r{rank}.npz"), **saved)
        return
    if scenario == "marked":
        store.wait(["r1_left"])
        layer.mark_unhealthy(1)
        with pytest.raises(_lib.AemError):  # the strict step refuses a known-dead peer
            layer.forward(xt, out_dtype=torch.float32)
    else:
        out, failed = layer.forward_tolerant(xt, out_dtype=torch.float32)  # rank 1 is silent
        saved.update(out_silent=out.cpu().numpy(), failed_silent=failed.cpu().numpy())
        _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")  # not an error
    saved["health"] = np.array(sorted(layer.health()))
    out, failed = layer.forward_tolerant(xt, out_dtype=torch.float32)  # rank 0 alone
    _, _, eff = layer.last_routing(tl)
    torch.cuda.synchronize()
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    saved.update(out2=out.cpu().numpy(), failed2=failed.cpu().numpy(), eff2=eff.cpu().numpy())
    np.savez(os.path.join(outdir, f"{scenario}_r{rank}.npz"), **saved)
    store.set("r0_done", "1")
    layer.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_ref(x, idx, val, eff, failed, qu, su, qd, sd):
    """Oracle output with failed units contributing nothing."""
    k = CFG["k"]
    t = x.shape[0]
    keep = 1.0 - failed.reshape(k, t).T.astype(np.float64)
    return O.moe_layer_rows(np.arange(t), x, idx, val * keep, eff, k, qu, su, qd, sd)


@pytest.mark.parametrize("scenario", ["marked", "silent"])
def test_tolerant_step_routes_around_a_failed_rank(cuda, scenario):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    T, E, k = CFG["T"], CFG["E"], CFG["k"]
    with tempfile.TemporaryDirectory() as outdir:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        mp.start_processes(_worker, args=(world, _free_port(), outdir, scenario), nprocs=world,
                           join=True, start_method="spawn")
        res = [dict(np.load(os.path.join(outdir, f"{scenario}_r{r}.npz"))) for r in range(world)]
    gw, gb, qu, su, qd, sd, x = _data()
    tl, el = T // world, E // world
    cap = O.default_capacity(T, k, E)
    oidx, oval = O.fused_gating(x, gw, gb, k, extra=1)
    tol = lambda got, ref: np.all(np.abs(got - ref) <= 1e-3 + 1e-3 * np.abs(ref))
    # healthy step: the global rule, nothing failed
    oeff = native.moe_route(oidx, k, E, cap)
    eff1 = np.concatenate([r["eff1"].reshape(k, tl) for r in res], axis=1).reshape(-1)
    np.testing.assert_array_equal(eff1, oeff)
    assert not any(r["failed1"].any() for r in res)
    ref1 = O.moe_layer_rows(np.arange(T), x, oidx, oval, oeff, k, qu, su, qd, sd)
    assert tol(np.concatenate([r["out1"] for r in res]), ref1)
    r0 = res[0]
    if scenario == "silent":  # the step the silent rank skipped: every unit failed, out zero
        assert r0["failed_silent"].all()
        assert not r0["out_silent"].any()
    assert list(r0["health"]) == [1]
    assert list(res[1]["health"]) == [0]
    # rank 0 alone: its own tokens are the batch; units for rank 1's experts fail
    eff0 = native.moe_route(oidx[:tl], k, E, cap)
    np.testing.assert_array_equal(r0["eff2"], eff0)
    want_failed = (eff0 // el) == 1
    assert want_failed.any() and not want_failed.all()
    np.testing.assert_array_equal(r0["failed2"].astype(bool), want_failed)
    ref2 = _layer_ref(x[:tl], oidx[:tl], oval[:tl], eff0, want_failed, qu, su, qd, sd)
    assert tol(r0["out2"], ref2)
