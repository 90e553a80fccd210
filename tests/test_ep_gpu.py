"""Expert-parallel MoE layer over NCCL on 2+ GPUs vs the single-process oracle.

One process per GPU (spawned here), experts placed in contiguous blocks or
round-robin (expert e on rank e % R), tokens split contiguously; the step's
two-half pipeline automatic, forced on and forced off.  The routing of every (token, slot) unit must equal the
capacity rule applied to the GLOBAL batch (bit-exact, the contract of
Router::assign_effective_experts in src/orchestration/router.hpp:249-266),
and every output row must match the float64 layer oracle within the layer
tolerance ``1e-3 + 1e-3 * |ref|``.  Skipped on hosts with fewer than 2 GPUs.
"""
import os
import socket
import tempfile

import numpy as np
import pytest

import aem_oracle as O
import native

pytestmark = pytest.mark.gpu

CFG = dict(T=2048, d=256, f=384, E=16, k=4)


def _weights(seed, e, d, f):
    rng = np.random.default_rng(seed)
    qu = rng.integers(-127, 128, size=(e, d, f), dtype=np.int8)
    su = (rng.random(size=(e, 1, f)) * 1e-4 + 2e-4).astype(np.float32)
    qd = rng.integers(-127, 128, size=(e, f, d), dtype=np.int8)
    sd = (rng.random(size=(e, 1, d)) * 1e-4 + 2e-4).astype(np.float32)
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    gb = O.zipf_bias(e)
    x = O.bf16_round(rng.normal(size=(CFG["T"], d)).astype(np.float32))
    return gw, gb, qu, su, qd, sd, x


def _local_experts(rank, world, E, placement):
    if placement == "strided":
        return np.arange(rank, E, world), np.arange(E) % world
    el = E // world
    return np.arange(rank * el, (rank + 1) * el), None


def _worker(rank, world, port, outdir, placement, pipeline=-1):
    import datetime
    import torch
    import torch.distributed as dist
    from aethermoe_b200.moe import EPLayer, ep_unique_id
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    T, d, f, E, k = CFG["T"], CFG["d"], CFG["f"], CFG["E"], CFG["k"]
    cap = O.default_capacity(T, k, E)
    gw, gb, qu, su, qd, sd, x = _weights(7, E, d, f)
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    mine, place = _local_experts(rank, world, E, placement)
    tl = T // world
    layer = EPLayer(bytes(uid.cpu().numpy()), rank, world, gw, gb, qu[mine], su[mine],
                    qd[mine], sd[mine], k, capacity=cap, device=rank, max_tokens=tl,
                    expert_to_rank=place)
    layer.set_pipeline(pipeline)
    bits = (x[rank * tl:(rank + 1) * tl].view(np.uint32) >> 16).astype(np.uint16)
    xt = torch.from_numpy(bits.view(np.int16)).to(dev).view(torch.bfloat16)
    outs = []
    for _ in range(2):  # two steps through the same exchange buffers
        outs.append(layer.forward(xt, out_dtype=torch.float32))
    idx, val, eff = layer.last_routing(tl)
    ob = layer.forward(xt, out_dtype=torch.bfloat16)  # bf16 output of the same step
    torch.cuda.synchronize()
    from aethermoe_b200 import _lib
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    # the same step three times through the asynchronous host API
    import ctypes
    ctx = _lib.context(rank)
    xh = xt.cpu().pin_memory()
    oh = [torch.empty((tl, d), dtype=torch.float32).pin_memory() for _ in range(3)]
    tickets = []
    for o in oh:
        t = ctypes.c_uint64()
        _lib.check(_lib.lib().aem_ep_submit_host(ctx, layer.handle, xh.data_ptr(), _lib.BF16, tl,
                                                 o.data_ptr(), _lib.F32, ctypes.byref(t)))
        tickets.append(t.value)
    for t in tickets:
        _lib.check(_lib.lib().aem_context_wait(ctx, t))
    for o in oh:
        np.testing.assert_allclose(o.numpy(), outs[-1].cpu().numpy(), rtol=0, atol=1e-5)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=outs[-1].cpu().numpy(),
             out0=outs[0].cpu().numpy(), idx=idx.cpu().numpy(), val=val.cpu().numpy(),
             eff=eff.cpu().numpy(), outb=ob.float().cpu().numpy())
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("placement,pipeline", [("contiguous", -1), ("strided", 1),
                                                ("strided", 0)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_matches_global_oracle(cuda, world, placement, pipeline):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    T, d, f, E, k = CFG["T"], CFG["d"], CFG["f"], CFG["E"], CFG["k"]
    with tempfile.TemporaryDirectory() as outdir:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        mp.start_processes(_worker, args=(world, _free_port(), outdir, placement, pipeline),
                           nprocs=world,
                           join=True, start_method="spawn")
        res = [np.load(os.path.join(outdir, f"rank{r}.npz")) for r in range(world)]
    tl = T // world
    gw, gb, qu, su, qd, sd, x = _weights(7, E, d, f)
    cap = O.default_capacity(T, k, E)
    oidx, oval = O.fused_gating(x, gw, gb, k, extra=1)
    idx = np.concatenate([r["idx"] for r in res])
    np.testing.assert_array_equal(idx, oidx)
    # local slot-major units -> global slot-major order u = j*T + r*tl + t
    eff = np.concatenate([r["eff"].reshape(k, tl) for r in res], axis=1).reshape(-1)
    oeff = native.moe_route(oidx, k, E, cap)
    np.testing.assert_array_equal(eff, oeff)
    assert (oeff != O.moe_units(oidx, k, E)[0]).any()  # capacity reroutes happened
    out = np.concatenate([r["out"] for r in res])
    ref = O.moe_layer_rows(np.arange(T), x, oidx, oval, oeff, k, qu, su, qd, sd)
    err = np.abs(out.astype(np.float64) - ref)
    assert np.all(err <= 1e-3 + 1e-3 * np.abs(ref)), err.max()
    np.testing.assert_allclose(np.concatenate([r["out0"] for r in res]), out, rtol=0, atol=1e-5)
    outb = np.concatenate([r["outb"] for r in res])  # bf16 rounding of the same sums
    assert np.all(np.abs(outb - out) <= 2.0 ** -8 * np.abs(out) + 1e-6)


FULL = dict(T=16384, d=2048, f=1408, E=64, k=6)


def _full_expert(e):
    """Expert e's int8 weights of the full-size config (seeded by e alone)."""
    rng = np.random.default_rng(1000 + e)
    qu = rng.integers(-127, 128, size=(FULL["d"], FULL["f"]), dtype=np.int8)
    qd = rng.integers(-127, 128, size=(FULL["f"], FULL["d"]), dtype=np.int8)
    su = (rng.random(size=(1, FULL["f"])) * 1e-4 + 2e-4).astype(np.float32)
    sd = (rng.random(size=(1, FULL["d"])) * 1e-4 + 2e-4).astype(np.float32)
    return qu, su, qd, sd


def _full_inputs():
    rng = np.random.default_rng(99)
    d, E = FULL["d"], FULL["E"]
    gw = (rng.normal(size=(d, E)) / np.sqrt(d)).astype(np.float32)
    x = O.bf16_round(rng.normal(size=(FULL["T"], d)).astype(np.float32))
    return gw, O.zipf_bias(E), x


def _full_worker(rank, world, port, outdir):
    import datetime
    import torch
    import torch.distributed as dist
    from aethermoe_b200.moe import EPLayer, ep_unique_id
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    T, E, k = FULL["T"], FULL["E"], FULL["k"]
    cap = O.default_capacity(T, k, E)
    gw, gb, x = _full_inputs()
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(ep_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    mine = np.arange(rank, E, world)  # round-robin placement, as the benchmark
    w = [_full_expert(e) for e in mine]
    tl = T // world
    layer = EPLayer(bytes(uid.cpu().numpy()), rank, world, gw, gb,
                    np.stack([a[0] for a in w]), np.stack([a[1] for a in w]),
                    np.stack([a[2] for a in w]), np.stack([a[3] for a in w]), k, capacity=cap,
                    device=rank, max_tokens=tl, expert_to_rank=np.arange(E) % world)
    bits = (x[rank * tl:(rank + 1) * tl].view(np.uint32) >> 16).astype(np.uint16)
    xt = torch.from_numpy(bits.view(np.int16)).to(dev).view(torch.bfloat16)
    out = layer.forward(xt, out_dtype=torch.float32)
    out = layer.forward(xt, out_dtype=torch.float32)
    idx, _, eff = layer.last_routing(tl)
    torch.cuda.synchronize()
    from aethermoe_b200 import _lib
    _lib.check(_lib.lib().aem_device_status(None), "aem_device_status")
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=out.cpu().numpy(),
             idx=idx.cpu().numpy(), eff=eff.cpu().numpy())
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_full_config(cuda, world):
    """The expert-parallel benchmark configuration (E=64, top-6, d=2048,
    ffn=1408, T=16384 global tokens, capacity 1920, Zipf(1.1) gate bias,
    round-robin placement) on `world` GPUs: every one of the 98304 units'
    effective experts bit-exact with the capacity rule over the global batch,
    about 48 sampled output rows within the layer tolerance of the oracle."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    T, E, k = FULL["T"], FULL["E"], FULL["k"]
    with tempfile.TemporaryDirectory() as outdir:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        mp.start_processes(_full_worker, args=(world, _free_port(), outdir), nprocs=world,
                           join=True, start_method="spawn")
        res = [np.load(os.path.join(outdir, f"rank{r}.npz")) for r in range(world)]
    tl = T // world
    gw, gb, x = _full_inputs()
    cap = O.default_capacity(T, k, E)
    oidx, oval = O.fused_gating(x, gw, gb, k, extra=1)
    np.testing.assert_array_equal(np.concatenate([r["idx"] for r in res]), oidx)
    eff = np.concatenate([r["eff"].reshape(k, tl) for r in res], axis=1).reshape(-1)
    oeff = native.moe_route(oidx, k, E, cap)
    np.testing.assert_array_equal(eff, oeff)
    assert (oeff != O.moe_units(oidx, k, E)[0]).sum() > 1000  # heavy capacity rerouting
    rows = np.unique(np.r_[0, T - 1, tl - 1, tl, np.random.default_rng(5).integers(0, T, 44)])
    w = [_full_expert(e) for e in range(E)]
    ref = O.moe_layer_rows(rows, x, oidx, oval, oeff, k, [a[0] for a in w], [a[1] for a in w],
                           [a[2] for a in w], [a[3] for a in w])
    out = np.concatenate([r["out"] for r in res])[rows]
    err = np.abs(out.astype(np.float64) - ref)
    assert np.all(err <= 1e-3 + 1e-3 * np.abs(ref)), err.max()
