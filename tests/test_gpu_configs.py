"""GPU parity at the full BASELINE shapes that are too large for the CPU oracle to check
whole: config 4 (B=32, S=4096, HQK=16, HV=32, random initial states, fused gated RMSNorm)
and config 2 (8 packed sequences of 200-4096 tokens) with random initial states.

The kernels run the whole batch with the launcher's automatic kernel choice; a seeded
sample of (sequence, v-head) units is checked against the oracle (each unit is an
independent recurrence, so a sample checks the kernel's indexing of the whole batch as
well as its math). Bars are those of tests/test_gpu_parity.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import max_abs, max_rel, row_cos_min, tensor_l2_rel
from oracle import gdn_oracle as O
import gdn_b200
from gdn_b200.synthetic import make_cu_seqlens, make_inputs

pytestmark = pytest.mark.gpu

O_MAX_ABS = 2e-2
STATE_REL = 1e-2
COS_MIN = 0.999
MAX_REL = 1e-2
Y_MAX_REL = 2e-2
D = 128


def _check(o, o_ref, sf, sf_ref, y, y_ref, tag):
    m = dict(o_abs=max_abs(o, o_ref), o_cos=row_cos_min(o, o_ref), o_rel=max_rel(o, o_ref),
             st_rel=tensor_l2_rel(sf, sf_ref), st_cos=row_cos_min(sf, sf_ref), st_mrel=max_rel(sf, sf_ref),
             y_cos=row_cos_min(y, y_ref), y_rel=max_rel(y, y_ref))
    print(tag, {k: f"{v:.3e}" for k, v in m.items()})
    assert np.isfinite(o).all() and np.isfinite(sf).all() and np.isfinite(y).all()
    assert m["o_abs"] <= O_MAX_ABS and m["st_rel"] <= STATE_REL, m
    assert m["o_cos"] >= COS_MIN and m["o_rel"] < MAX_REL, m
    assert m["st_cos"] >= COS_MIN and m["st_mrel"] < MAX_REL, m
    assert m["y_cos"] >= COS_MIN and m["y_rel"] < Y_MAX_REL, m


def _device_inputs(B, T, HQK, HV, seed):
    """BASELINE distributions drawn on the device (a CPU draw of config 4 takes minutes):
    q, k ~ N(0,1) L2-normalised in fp32 then bf16; v, z ~ N(0,1) bf16; beta = sigmoid(N(0,1));
    g = -softplus(N(0,1)); w = 1 + 0.1 N(0,1) bf16; s0 ~ N(0, 0.02)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen)  # noqa: E731
    q = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    k = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    v, z = n(B, T, HV, D).bfloat16(), n(B, T, HV, D).bfloat16()
    beta = torch.sigmoid(n(B, T, HV))
    g = -torch.nn.functional.softplus(n(B, T, HV))
    w = (1 + 0.1 * n(D)).bfloat16()
    s0 = n(B, HV, D, D) * 0.02
    return q, k, v, g, beta, z, w, s0


def test_config4_full_shape_sampled_units():
    """BASELINE config 4 at full shape through the public API (automatic kernel choice: 1,024
    (sequence, v-head) units), eight units checked against the oracle: the first, the last,
    and six drawn with a fixed seed."""
    B, T, HQK, HV = 32, 4096, 16, 32
    q, k, v, g, beta, z, w, s0 = _device_inputs(B, T, HQK, HV, seed=4)
    o, sf = gdn_b200.chunk_prefill(q, k, v, g, beta, s0)
    y, sf2 = gdn_b200.chunk_prefill_gated(q, k, v, g, beta, z, w, s0, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(sf, sf2)
    rng = np.random.default_rng(404)
    units = [(0, 0), (B - 1, HV - 1)] + [(int(b), int(h)) for b, h in
                                         zip(rng.integers(0, B, 6), rng.integers(0, HV, 6))]
    wh = w.float().cpu().numpy()
    for b, h in units:
        hq = h // (HV // HQK)
        hx = lambda t, i: t[b:b + 1, :, i:i + 1].float().cpu().numpy()  # noqa: E731
        qi, ki, vi, zi = hx(q, hq), hx(k, hq), hx(v, h), hx(z, h)
        gi = g[b:b + 1, :, h:h + 1].cpu().numpy()
        bi = beta[b:b + 1, :, h:h + 1].cpu().numpy()
        si = s0[b:b + 1, h:h + 1].cpu().numpy()
        o_ref, sf_ref = O.chunk_gated_delta_rule(qi, ki, vi, gi, bi, 64, si)
        y_ref = O.gated_rmsnorm(o_ref, zi, wh, 1e-6)
        _check(hx(o, h), o_ref, sf[b:b + 1, h:h + 1].cpu().numpy(), sf_ref, hx(y, h), y_ref,
               f"config4 b={b} h={h}")


@pytest.mark.parametrize("gated", [False, True])
def test_config2_random_initial_states(gated):
    """BASELINE config 2's packed batch (8 sequences, lengths U[200, 4096], seeded; HQK=16, HV=32)
    with a random initial state per sequence; three sequences checked against the oracle."""
    cu = make_cu_seqlens(8, 200, 4096, seed=2)
    T = int(cu[-1])
    inp = make_inputs(1, T, 16, 32, D, seed=23, dist="baseline", with_s0=True, n_states=8)
    dev = lambda x, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dt)  # noqa: E731
    args = (dev(inp.q), dev(inp.k), dev(inp.v), dev(inp.g, torch.float32), dev(inp.beta, torch.float32),
            torch.from_numpy(cu).cuda(), dev(inp.s0, torch.float32))
    o, sf = gdn_b200.chunk_prefill_varlen(*args)
    y = gdn_b200.chunk_prefill_varlen(*args, z=dev(inp.z), w=dev(inp.w), eps=inp.eps)[0] if gated else o
    torch.cuda.synchronize()
    o, sf, y = o.float().cpu().numpy(), sf.cpu().numpy(), y.float().cpu().numpy()
    for i in (0, 3, 7):
        a, b = int(cu[i]), int(cu[i + 1])
        sl = lambda x: x[:, a:b]  # noqa: E731
        o_ref, s_ref = O.chunk_gated_delta_rule(sl(inp.q), sl(inp.k), sl(inp.v), sl(inp.g), sl(inp.beta), 64,
                                                inp.s0[i:i + 1])
        y_ref = O.gated_rmsnorm(o_ref, sl(inp.z), inp.w, inp.eps) if gated else o_ref
        _check(o[:, a:b], o_ref, sf[i:i + 1], s_ref, y[:, a:b], y_ref, f"cfg2 seq{i} len{b - a} gated={gated}")
