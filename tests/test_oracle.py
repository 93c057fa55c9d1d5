"""Pin the CPU oracle (oracle/gdn_oracle.py) against the reference's golden vectors.

The vectors in tests/golden/ were produced by the reference's own oracle
(transformers ``torch_chunk_gated_delta_rule`` + ``Qwen3_5RMSNormGated``, which
the reference's verbatim copy at kernels/harness/parity_test.py:35-96 matched
bit for bit when they were generated). Inputs are regenerated from the stored
seed and checked against the stored checksum first.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, golden_index, max_abs, tensor_l2_rel
from oracle import gdn_oracle as O
from gdn_b200.synthetic import make_inputs

CASES = golden_index()

# numpy (float32) vs torch (float32): same math, different summation order.
STATE_RTOL, STATE_ATOL = 2e-4, 2e-6
FP32_RTOL, FP32_ATOL = 2e-4, 2e-6


def _digest(inp):
    import hashlib
    h = hashlib.sha256()
    for a in (inp.q, inp.k, inp.v, inp.g, inp.beta, inp.z, inp.w, inp.s0):
        h.update(b"none" if a is None else np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def _bf16_close(a, b):
    """Both sides are fp32 results rounded to bf16: they may land one bf16 step
    apart (|d| <= 2^-7 |ref|: one step at a binade edge), or differ by fp32 summation noise near zero
    (|d| <= 1e-5 max|ref|). Returns (worst ratio to that bound, mismatch fraction)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if a.size == 0:
        return 0.0, 0.0
    bound = 2.0 ** -7 * np.abs(b) + 1e-5 * np.abs(b).max() + 1e-30
    d = np.abs(a - b)
    return float((d / bound).max()), float((d > 0).mean())


@pytest.mark.parametrize("name", [n for n in CASES if not n.startswith("recurrent")])
def test_oracle_matches_golden(name):
    meta = CASES[name]
    kw = meta["kwargs"]
    inp = make_inputs(**kw)
    assert _digest(inp) == meta["input_sha256"], "synthetic generator no longer reproduces the golden inputs"
    gold = np.load(GOLDEN / f"{name}.npz")
    cu = meta.get("cu_seqlens")
    if cu is None:
        o, sf = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0,
                                         return_fp32=(kw.get("dtype") == "fp32"))
    else:
        o, sf = O.chunk_gated_delta_rule_varlen(inp.q, inp.k, inp.v, inp.g, inp.beta, np.array(cu), 64, inp.s0)
    np.testing.assert_allclose(sf, gold["sf"], rtol=STATE_RTOL, atol=STATE_ATOL)
    if "o_bits" in gold:
        o_ref = O.bf16_from_bits(gold["o_bits"]).reshape(o.shape)
        y_ref = O.bf16_from_bits(gold["y_bits"]).reshape(o.shape)
        worst, frac = _bf16_close(o, o_ref)
        assert worst <= 1.0 and frac < 0.01, (worst, frac)
        y = O.gated_rmsnorm(o_ref, inp.z, inp.w, inp.eps)
        worst, frac = _bf16_close(y, y_ref)
        assert worst <= 1.0 and frac < 0.01, (worst, frac)
    else:
        np.testing.assert_allclose(o, gold["o"], rtol=FP32_RTOL, atol=FP32_ATOL)
        # fp32 I/O: the norm's "round to input dtype" is a no-op in the reference module
        var = (gold["o"].astype(np.float32) ** 2).mean(-1, keepdims=True)
        n = gold["o"] / np.sqrt(var + np.float32(inp.eps))
        y = (inp.w * n) * (inp.z / (1 + np.exp(-inp.z)))
        np.testing.assert_allclose(y, gold["y"], rtol=1e-4, atol=1e-5)


def test_recurrent_matches_golden():
    meta = CASES["recurrent_bf16_s3_hv2"]
    inp = make_inputs(**meta["kwargs"])
    gold = np.load(GOLDEN / "recurrent_bf16_s3_hv2.npz")
    o, sf = O.recurrent_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, inp.s0)
    np.testing.assert_allclose(sf, gold["sf"], rtol=STATE_RTOL, atol=STATE_ATOL)
    worst, _ = _bf16_close(o, O.bf16_from_bits(gold["o_bits"]).reshape(o.shape))
    assert worst <= 1.0


@pytest.mark.parametrize("T", [1, 63, 64, 65, 150])
def test_chunked_equals_recurrent(T):
    """The chunked (WY) form and the token recurrence are the same function."""
    inp = make_inputs(1, T, 1, 2, 128, seed=100 + T, dist="refgrid", with_s0=True)
    o1, s1 = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0, return_fp32=True)
    o2, s2 = O.recurrent_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, inp.s0)
    assert tensor_l2_rel(s1, s2) < 1e-5
    assert max_abs(O.bf16_round(o1), o2) <= 2.0 ** -6


def test_split_sequence_continuation():
    """Running S tokens in two pieces, handing the final state over, equals one pass
    (the only resume semantics of this path: initial_state -> final_state)."""
    inp = make_inputs(1, 200, 2, 4, 128, seed=7, dist="baseline", with_s0=True)
    o, s = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0, return_fp32=True)
    cut = 128  # chunk-aligned split keeps the chunk partition identical
    oa, sa = O.chunk_gated_delta_rule(inp.q[:, :cut], inp.k[:, :cut], inp.v[:, :cut], inp.g[:, :cut],
                                      inp.beta[:, :cut], 64, inp.s0, return_fp32=True)
    ob, sb = O.chunk_gated_delta_rule(inp.q[:, cut:], inp.k[:, cut:], inp.v[:, cut:], inp.g[:, cut:],
                                      inp.beta[:, cut:], 64, sa, return_fp32=True)
    assert tensor_l2_rel(np.concatenate([oa, ob], 1), o) < 1e-6
    assert tensor_l2_rel(sb, s) < 1e-6


def test_grouped_heads_equal_expanded():
    """HQK < HV (v-head h reads qk-head h // (HV/HQK)) equals pre-expanded heads."""
    inp = make_inputs(1, 70, 2, 4, 128, seed=8)
    o1, s1 = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0)
    qe, ke = np.repeat(inp.q, 2, axis=2), np.repeat(inp.k, 2, axis=2)
    o2, s2 = O.chunk_gated_delta_rule(qe, ke, inp.v, inp.g, inp.beta, 64, inp.s0)
    assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 3.0e38, 1e-40], np.float32)
    r = O.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.0 + 2 ** -6 and r[3] == -1.0
    import torch
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(r, t)


def test_gate_math():
    a = np.array([-30.0, -1.0, 0.0, 1.0, 25.0], np.float32)
    g, beta = O.gdn_gate(a, a, np.float32(0.5), np.float32(0.1))
    import torch
    ta = torch.from_numpy(a)
    g_ref = -(torch.tensor(0.5).exp()) * torch.nn.functional.softplus(ta + 0.1)
    np.testing.assert_allclose(g, g_ref.numpy(), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(beta, torch.sigmoid(ta).numpy(), rtol=1e-6)
