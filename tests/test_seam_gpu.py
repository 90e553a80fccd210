"""Scheduler -> MoE-layer seam on the GPU: one continuous-batching
iteration's slices (decode steps of 1 token, prefill chunks up to the
reference's max_prefill_chunk=512, SchedulerConfig, src/core/scheduler.hpp:
50-53) through ``aem_moe_forward_slices`` equal the same tokens run as one
concatenated batch: routing bit-exact (batch_position = iteration order) and
outputs within the layer tolerance of the float64 oracle."""
import numpy as np
import pytest

import aem_oracle as O

pytestmark = pytest.mark.gpu


def _iteration(rng, d, dtype):
    """Decode steps first, then prefill chunks -- the order step() emits.
    float32 slices hold raw float32 values; bf16 slices bf16 values."""
    sizes = [1] * 37 + [int(v) for v in rng.integers(2, 513, size=5)] + [0, 3]
    rnd = (lambda a: a) if dtype == "f32" else O.bf16_round
    return [(100 + i, rnd(rng.normal(size=(n, d)).astype(np.float32)))
            for i, n in enumerate(sizes)]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_iteration_slices_equal_concatenated_batch(cuda, dtype):
    import torch
    from aethermoe_b200 import _lib
    from aethermoe_b200.moe import MoELayer
    rng = np.random.default_rng(17)
    d, f, e, k = 256, 384, 8, 2
    qu = rng.integers(-127, 128, size=(e, d, f), dtype=np.int8)
    qd = rng.integers(-127, 128, size=(e, f, d), dtype=np.int8)
    su = (rng.random(size=(e, 1, f)) * 1e-4 + 2e-4).astype(np.float32)
    sd = (rng.random(size=(e, 1, d)) * 1e-4 + 2e-4).astype(np.float32)
    gw = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    gb = O.zipf_bias(e)
    its = _iteration(rng, d, dtype)
    T = sum(x.shape[0] for _, x in its)
    cap = O.default_capacity(T, k, e)
    layer = MoELayer(gw, gb, qu, su, qd, sd, k, capacity=cap)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    xs = [(sid, torch.from_numpy(x).to(cuda).to(tdt)) for sid, x in its]
    outs = layer.forward_slices(xs, out_dtype=torch.float32)
    idx_s, val_s, eff_s = [t.cpu().numpy() for t in layer.last_routing(T)]
    cat = torch.cat([x for _, x in xs])
    ref_out = layer.forward(cat, out_dtype=torch.float32)
    idx_c, val_c, eff_c = [t.cpu().numpy() for t in layer.last_routing(T)]
    torch.cuda.synchronize()
    _lib.check(_lib.lib().aem_device_status(None))
    np.testing.assert_array_equal(idx_s, idx_c)
    np.testing.assert_array_equal(eff_s, eff_c)
    got = torch.cat(outs).cpu().numpy()
    assert [o.shape[0] for o in outs] == [x.shape[0] for _, x in its]
    np.testing.assert_allclose(got, ref_out.cpu().numpy(), rtol=0, atol=1e-5)
    xh = cat.float().cpu().numpy()
    oidx, oval = O.fused_gating(xh, gw, gb, k, extra=1)
    oeff = O.moe_route(oidx, k, e, cap)
    np.testing.assert_array_equal(eff_s, oeff)
    # float32 slices: the float32 layer (x and hidden activation unrounded)
    ref = O.moe_layer_rows(np.arange(T), xh, oidx, oval, oeff, k, qu, su, qd, sd,
                           hidden="f32" if dtype == "f32" else "bf16")
    assert np.all(np.abs(got - ref) <= 1e-3 + 1e-3 * np.abs(ref))
    layer.close()
