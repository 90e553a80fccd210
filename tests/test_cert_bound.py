"""The CERTIFIED gating mode's error bound, checked on the CPU: fast logits
(float32 fused multiply-add chains over parts of d, the kernels' order) stay
within their bound of the sequential float32 logits of the reference
specification (prototype/math_proto.py:33-34) on every entry, over the
shapes and distributions the gating tests use, and the bound is tight enough
to order ordinary rows."""
import numpy as np
import pytest

import aem_oracle as O


@pytest.mark.parametrize("n,d,e,parts,seed", [
    (6, 4096, 8, 32, 1),     # d-split small kernel, 8 experts
    (4, 2048, 64, 4, 2),     # the bench gate's shape
    (3, 1000, 17, 8, 3),     # d not a multiple of the block
    (8, 512, 64, 1, 4),      # one part (the large kernel's chunk chain)
])
def test_bound_covers_fast_minus_exact(n, d, e, parts, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(n, d)).astype(np.float32)
    x[0] *= 1e3   # large activations
    x[1] *= 1e-3  # small ones
    w = (rng.normal(size=(d, e)) / np.sqrt(d)).astype(np.float32)
    b = O.zipf_bias(e)
    exact = O.gating_logits_seq(x, w, b)
    f, bound = O.certified_fast_logits(x, w, b, parts=parts)
    diff = np.abs(f.astype(np.float64) - exact.astype(np.float64))
    assert np.all(diff <= bound), float((diff - bound).max())
    # the bound certifies typical gaps: well under the logits' spread
    assert np.median(bound) < 0.01 * np.median(np.abs(exact))


def test_bound_is_not_vacuous_on_near_ties():
    """Two experts with logits one float32 ulp apart: the bound must not
    claim to order them (it exceeds half their gap)."""
    rng = np.random.default_rng(7)
    d = 256
    x = rng.normal(size=(1, d)).astype(np.float32)
    w = (rng.normal(size=(d, 2)) / np.sqrt(d)).astype(np.float32)
    w[:, 1] = w[:, 0]
    b = np.zeros(2, np.float32)
    b[1] = np.spacing(np.float32(abs(O.gating_logits_seq(x, w[:, :1], b[:1])[0, 0]) + 1.0))
    f, bound = O.certified_fast_logits(x, w, b)
    exact = O.gating_logits_seq(x, w, b)
    gap = abs(float(exact[0, 1]) - float(exact[0, 0]))
    assert bound[0, 0] + bound[0, 1] >= gap
