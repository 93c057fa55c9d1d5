"""The segmented prefill (segments of a long sequence run side by side, their entry states
from a scan of the segments' affine state maps) against the plain one-pass prefill, on B200.

Both paths run the same kernels over the same chunks; they differ only in how the state
reaches each segment (the scan in float64 instead of the chunk recurrence in fp32), so they
agree far inside the parity bars that tie the plain path to the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import max_abs, max_rel, tensor_l2_rel
import gdn_b200
from gdn_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

O_MAX_ABS = 2e-2
Y_MAX_REL = 2e-2


def _dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(dtype)


def _run(fn, inp, gated, **kw):
    q, k, v, z, w = _dev(inp.q), _dev(inp.k), _dev(inp.v), _dev(inp.z), _dev(inp.w)
    g, b, s = _dev(inp.g, torch.float32), _dev(inp.beta, torch.float32), _dev(inp.s0, torch.float32)
    if fn == "plain":
        out = (gdn_b200.chunk_prefill_gated(q, k, v, g, b, z, w, s) if gated else gdn_b200.chunk_prefill(q, k, v, g, b, s))
    elif gated:
        out = gdn_b200.chunk_prefill_segmented(q, k, v, g, b, s, z=z, w=w, **kw)
    else:
        out = gdn_b200.chunk_prefill_segmented(q, k, v, g, b, s, **kw)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in out]


@pytest.mark.parametrize("B,T,HQK,HV,segments,gated", [(1, 4133, 2, 4, 5, False), (1, 4133, 2, 4, 5, True),
                                                        (2, 2000, 2, 4, 3, True), (1, 65, 2, 4, 8, False)])
def test_segmented_matches_plain(B, T, HQK, HV, segments, gated):
    inp = make_inputs(B, T, HQK, HV, seed=11)
    o_ref, sf_ref = _run("plain", inp, gated)
    o, sf = _run("segmented", inp, gated, segments=segments)
    assert o.shape == o_ref.shape and sf.shape == sf_ref.shape
    if gated:
        assert max_rel(o, o_ref) < Y_MAX_REL
    else:
        assert max_abs(o, o_ref) <= O_MAX_ABS / 4
    assert tensor_l2_rel(sf, sf_ref) < 1e-4


def test_segmented_slow_decay_against_oracle():
    """Slow-decay heads (g = -U(0, 0.002), beta = U(0, 0.3)) with random initial states: each
    segment's state map Phi is far from zero, so the entry states come from the scan rather than
    being forgotten. Five segments of a 4,133-token sequence against the serial oracle and the
    one-pass call (with fast decay Phi underflows and the scan is not exercised)."""
    import dataclasses

    from oracle import gdn_oracle as O
    base = make_inputs(1, 4133, 2, 4, seed=13, with_s0=True)
    rng = np.random.default_rng(13)
    inp = dataclasses.replace(base, g=-(rng.random(base.g.shape) * 0.002).astype(np.float32),
                              beta=(rng.random(base.beta.shape) * 0.3).astype(np.float32))
    o_ref, sf_ref = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0)
    o_one, sf_one = _run("plain", inp, False)
    o, sf = _run("segmented", inp, False, segments=5)
    print({"o_abs_oracle": max_abs(o, o_ref), "st_rel_oracle": tensor_l2_rel(sf, sf_ref),
           "o_abs_onepass": max_abs(o, o_one), "st_rel_onepass": tensor_l2_rel(sf, sf_one)})
    assert max_abs(o, o_ref) <= O_MAX_ABS and tensor_l2_rel(sf, sf_ref) <= 1e-2
    assert max_rel(sf, sf_ref) < 1e-2
    assert max_abs(o, o_one) <= O_MAX_ABS / 4 and tensor_l2_rel(sf, sf_one) < 1e-4


def test_one_segment_is_the_plain_call():
    inp = make_inputs(1, 700, 2, 4, seed=12)
    o_ref, sf_ref = _run("plain", inp, False)
    o, sf = _run("segmented", inp, False, segments=1)
    assert np.array_equal(o, o_ref) and np.array_equal(sf, sf_ref)
