"""Host logic of the segmented prefill (``gdn_b200.chunk_prefill_segmented``), on CPU.

The segmented path cuts each sequence at chunk boundaries, computes every segment's affine
state map (A from a zero entry state, Phi from the identity with v = 0), scans the entry
states and reruns the segments from them. Here the segment passes are the oracle's (test
infrastructure only) and the cut and the scan are the product's own helpers: together they
must reproduce the serial oracle's output and final state.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gdn_b200 import segment_bounds, segment_entry_states
from oracle import gdn_oracle as ora


def test_segment_bounds_cut_at_chunk_boundaries():
    assert segment_bounds(2, 200, 2) == ([0, 128, 200, 328, 400], 2)
    assert segment_bounds(1, 64, 5) == ([0, 64], 1)
    assert segment_bounds(1, 130, 8) == ([0, 64, 128, 130], 3)
    cu, per = segment_bounds(1, 65536, 9)
    assert per == 9 and cu[1] == 114 * 64 and cu[-1] == 65536
    for B, T, n in ((1, 1, 1), (3, 1000, 4), (2, 4096, 37)):
        cu, per = segment_bounds(B, T, n)
        assert len(cu) == B * per + 1 and cu[0] == 0 and cu[-1] == B * T
        for b in range(B):  # inner boundaries of each sequence are chunk multiples
            for t in cu[b * per + 1:(b + 1) * per]:
                assert (t - b * T) % 64 == 0
    with pytest.raises(ValueError):
        segment_bounds(1, 0, 2)


def _inputs(B, T, HQK, HV, D, with_s0, decay, seed=7):
    """'fast': g = -0.3 softplus(N(0,1)) (about -0.24 per token: a segment's map Phi decays to ~0);
    'slow': g = -U(0, 0.002) and beta = U(0, 0.3 * D / 128) (the head-dim-128 rate of erasure,
    scaled to D), so that over a few hundred tokens Phi stays far from zero and the scan carries
    the state from segment to segment."""
    rng = np.random.default_rng(seed)
    q = ora.l2norm(rng.standard_normal((B, T, HQK, D)).astype(np.float32))
    k = ora.l2norm(rng.standard_normal((B, T, HQK, D)).astype(np.float32))
    v = rng.standard_normal((B, T, HV, D)).astype(np.float32)
    if decay == "fast":
        g = -np.log1p(np.exp(rng.standard_normal((B, T, HV)))).astype(np.float32) * 0.3
        beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))).astype(np.float32)
    else:
        g = -(rng.random((B, T, HV)) * 0.002).astype(np.float32)
        beta = (rng.random((B, T, HV)) * 0.3 * D / 128).astype(np.float32)
    s0 = (rng.standard_normal((B, HV, D, D)) * 0.5).astype(np.float32) if with_s0 else None
    return q, k, v, g, beta, s0


def _segmented(q, k, v, g, beta, s0, nseg, phi_fn=None):
    """The segmented scheme with the oracle as the segment pass; ``phi_fn`` may alter the maps."""
    B, T, HV, D = v.shape
    cu, per = segment_bounds(B, T, nseg)
    pk = lambda x: x.reshape(1, B * T, *x.shape[2:])  # noqa: E731
    N = B * per
    _, A = ora.chunk_gated_delta_rule_varlen(pk(q), pk(k), pk(v), pk(g), pk(beta), cu, return_fp32=True)
    eye = np.broadcast_to(np.eye(D, dtype=np.float32), (N, HV, D, D)).copy()
    _, Phi = ora.chunk_gated_delta_rule_varlen(pk(q), pk(k), np.zeros_like(pk(v)), pk(g), pk(beta), cu,
                                               initial_state=eye, return_fp32=True)
    if phi_fn is not None:
        Phi = phi_fn(Phi)
    starts = segment_entry_states(torch.from_numpy(Phi).view(B, per, HV, D, D),
                                  torch.from_numpy(A).view(B, per, HV, D, D),
                                  None if s0 is None else torch.from_numpy(s0))
    o, sf = ora.chunk_gated_delta_rule_varlen(pk(q), pk(k), pk(v), pk(g), pk(beta), cu,
                                              initial_state=starts.reshape(N, HV, D, D).numpy(), return_fp32=True)
    return o.reshape(B, T, HV, D), sf.reshape(B, per, HV, D, D)[:, -1], Phi


@pytest.mark.parametrize("B,T,HQK,HV,nseg,with_s0,decay", [(1, 300, 1, 2, 3, True, "fast"),
                                                           (2, 200, 1, 1, 2, False, "fast"),
                                                           (1, 2048, 1, 2, 4, True, "slow"),
                                                           (2, 1500, 1, 1, 3, True, "slow")])
def test_affine_segment_scan_reproduces_serial(B, T, HQK, HV, nseg, with_s0, decay):
    D = 64
    q, k, v, g, beta, s0 = _inputs(B, T, HQK, HV, D, with_s0, decay)
    o_ref, sf_ref = ora.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    o, sf_last, Phi = _segmented(q, k, v, g, beta, s0, nseg)
    if decay == "slow":  # the maps are far from zero: the scan carries real state between segments
        assert np.abs(np.diagonal(Phi, axis1=-2, axis2=-1)).mean() > 0.1
    assert np.abs(o - o_ref).max() < 1e-4
    assert np.linalg.norm(sf_last - sf_ref) / np.linalg.norm(sf_ref) < 1e-5


@pytest.mark.parametrize("alter", ["transposed", "zeroed"])
def test_wrong_state_map_is_caught_with_slow_decay(alter):
    """With slow decay the segments' state maps matter: a transposed or a zeroed Phi (the
    mistakes planted here, in the oracle-driven scheme) must move the result far outside the
    tolerances the correct scheme meets."""
    D = 64
    q, k, v, g, beta, s0 = _inputs(1, 2048, 1, 2, D, True, "slow")
    o_ref, sf_ref = ora.chunk_gated_delta_rule(q, k, v, g, beta, 64, s0, True, True)
    fn = (lambda P: np.ascontiguousarray(np.swapaxes(P, -1, -2))) if alter == "transposed" else np.zeros_like
    o, sf_last, _ = _segmented(q, k, v, g, beta, s0, 4, phi_fn=fn)
    # (the correct scheme: o within 1e-4 and the state within 1e-5, measured ~4e-8 and ~1.5e-7 here;
    # transposed: ~5e-3 and ~8e-3; zeroed: ~8e-2 and ~0.13)
    assert np.abs(o - o_ref).max() > 1e-3
    assert np.linalg.norm(sf_last - sf_ref) / np.linalg.norm(sf_ref) > 1e-3
