"""The segmented prefill (deltanet_chunk_prefill_segmented: segments of a long sequence run
side by side, their entry states from a device scan of the segments' affine state maps)
against the plain one-pass prefill, on B200.

Both paths run the same kernels over the same chunks; they differ only in how the state
reaches each segment (the scan of the maps instead of the chunk recurrence), so they agree
far inside the parity bars that tie the plain path to the oracle.
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


@pytest.mark.parametrize("kernel", ["fused", "split"])
@pytest.mark.parametrize("B,T,HQK,HV,segments,gated", [(1, 4133, 2, 4, 5, False), (1, 4133, 2, 4, 5, True),
                                                        (2, 2000, 2, 4, 3, True), (1, 65, 2, 4, 8, False),
                                                        (1, 2000, 1, 2, 7, True)])
def test_segmented_matches_plain(B, T, HQK, HV, segments, gated, kernel, monkeypatch):
    """Both kernels of the segmented passes: one CTA per (segment, head) ("fused") and a 4-CTA
    cluster per (segment, head) ("split"), chosen through GDN_B200_KERNEL."""
    inp = make_inputs(B, T, HQK, HV, seed=11)
    o_ref, sf_ref = _run("plain", inp, gated)
    monkeypatch.setenv("GDN_B200_KERNEL", kernel)
    nseg, per, kern = gdn_b200.segmented_plan(B, T, HV, segments)
    nc = (T + 63) // 64
    assert nseg == (nc + per - 1) // per and per == (nc + min(segments, nc) - 1) // min(segments, nc)
    assert kern == ({"fused": 1, "split": 2}[kernel] if nseg > 1 else 0)
    o, sf = _run("segmented", inp, gated, segments=segments)
    assert o.shape == o_ref.shape and sf.shape == sf_ref.shape
    if gated:
        assert max_rel(o, o_ref) < Y_MAX_REL
    else:
        assert max_abs(o, o_ref) <= O_MAX_ABS / 4
    assert tensor_l2_rel(sf, sf_ref) < 1e-4


@pytest.mark.parametrize("kernel", ["fused", "split"])
def test_segmented_slow_decay_against_oracle(kernel, monkeypatch):
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
    monkeypatch.setenv("GDN_B200_KERNEL", kernel)
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


def _timed(fn, reps=5):
    import statistics
    for _ in range(2):
        fn()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def test_config3_shard_library_choice_against_one_pass():
    """One rank's shard of BASELINE config 3 (B=1, S=65536, 4 v-heads, 2 qk-heads, zero initial
    state, fused norm) with the library's segment choice against the one-pass call; both timed
    (CUDA events, median of 5 after 2 warm-ups, through the binding)."""
    import warnings
    inp = make_inputs(1, 65536, 2, 4, seed=3, with_s0=False)
    q, k, v, z, w = _dev(inp.q), _dev(inp.k), _dev(inp.v), _dev(inp.z), _dev(inp.w)
    g, b = _dev(inp.g, torch.float32), _dev(inp.beta, torch.float32)
    nseg, per, kern = gdn_b200.segmented_plan(1, 65536, 4)
    assert nseg > 1, "the library should cut a 4-head 65,536-token stream into segments"
    y1, sf1 = gdn_b200.chunk_prefill_gated(q, k, v, g, b, z, w)
    y, sf = gdn_b200.chunk_prefill_segmented(q, k, v, g, b, z=z, w=w)
    torch.cuda.synchronize()
    y1, sf1, yh, sfh = (t.float().cpu().numpy() for t in (y1, sf1, y, sf))
    assert max_rel(yh, y1) < Y_MAX_REL and tensor_l2_rel(sfh, sf1) < 1e-4
    t_one = _timed(lambda: gdn_b200.chunk_prefill_gated(q, k, v, g, b, z, w))
    t_seg = _timed(lambda: gdn_b200.chunk_prefill_segmented(q, k, v, g, b, z=z, w=w))
    warnings.warn(f"config-3 shard (S=65536, 4 v-heads): one pass {t_one:.3f} ms, segmented "
                  f"({nseg} segments of {per} chunks, kernel {kern}) {t_seg:.3f} ms")


def test_full_gpu_takes_one_pass():
    """With 32 heads the GPU is full: the library's choice is one pass, the plain call's result."""
    inp = make_inputs(1, 700, 16, 32, seed=14, with_s0=True)
    o_ref, sf_ref = _run("plain", inp, True)
    o, sf = _run("segmented", inp, True)
    assert np.array_equal(o, o_ref) and np.array_equal(sf, sf_ref)
