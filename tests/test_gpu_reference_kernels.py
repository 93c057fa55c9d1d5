"""Our prefill against the reference's own CUDA kernels on the same B200.

``oracle/Makefile`` compiles the reference's kernels unmodified for sm_100a
(kernels/chunk_delta_cuda.cu, the canonical fp32-FMA kernel, and
kernels/chunk_delta_cuda_tco.cu, the production bf16 o-pass) into
``oracle/_ref/libref_chunk_delta.so``. This is the reference harness's own gate
(kernels/harness/parity_cuda.py:75-98: row cosine >= 0.999 and floored max-rel < 1e-2 on
o and the state) applied between the reference's kernels and ours on identical inputs,
plus the north-star bars (o max-abs <= 2e-2, state relative L2 <= 1e-2). Both sides are
timed through their C ABI with buffers allocated beforehand, with CUDA events (median of
five calls after two warm-ups, ungated, as the reference's contract), and the timings are
reported as a pytest warning so that they appear in the run's summary.

Skipped when ``oracle/_ref`` holds no build (it needs the reference checkout at build time).
"""
from __future__ import annotations

import ctypes
import statistics
import warnings

import numpy as np
import pytest
import torch

from conftest import ROOT, max_abs, max_rel, row_cos_min, tensor_l2_rel
import gdn_b200
from gdn_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

REF_LIB = ROOT / "oracle" / "_ref" / "libref_chunk_delta.so"
D = 128


def _ref_lib():
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libref_chunk_delta.so not built (oracle/Makefile needs the reference checkout)")
    lib = ctypes.CDLL(str(REF_LIB))  # RTLD_LOCAL: its symbols do not interpose on ours
    vp, ci = ctypes.c_void_p, ctypes.c_int
    for pre in ("deltanet", "deltanet_tcop"):
        ws = getattr(lib, f"{pre}_prefill_workspace_size")
        ws.restype, ws.argtypes = ctypes.c_size_t, [ci] * 6
        fn = getattr(lib, f"{pre}_chunk_prefill")
        fn.restype = ci
        fn.argtypes = [vp] * 8 + [ci] * 7 + [vp, ctypes.c_size_t, vp, ci]
    return lib


def _time(fn, reps=5, warm=2):
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    return statistics.median(ts)


def _bars(o, o_ref, sf, sf_ref, tag):
    m = dict(o_abs=max_abs(o, o_ref), o_cos=row_cos_min(o, o_ref), o_rel=max_rel(o, o_ref),
             st_rel=tensor_l2_rel(sf, sf_ref), st_cos=row_cos_min(sf, sf_ref), st_mrel=max_rel(sf, sf_ref))
    print(tag, {k: f"{v:.3e}" for k, v in m.items()})
    assert np.isfinite(o).all() and np.isfinite(sf).all()
    assert m["o_abs"] <= 2e-2 and m["st_rel"] <= 1e-2, m
    assert m["o_cos"] >= 0.999 and m["o_rel"] < 1e-2 and m["st_cos"] >= 0.999 and m["st_mrel"] < 1e-2, m
    return m


@pytest.mark.parametrize("cfg", ["config1", "config4"])
def test_agrees_with_reference_cuda_kernels(cfg):
    """BASELINE config 1 (whole) or config 4 (whole batch, compared on the first four sequences):
    the reference's canonical and TCO kernels against ours (ungated, the reference's contract)."""
    lib = _ref_lib()
    B, T, HQK, HV = (1, 1141, 16, 32) if cfg == "config1" else (32, 4096, 16, 32)
    if cfg == "config1":
        inp = make_inputs(B, T, HQK, HV, D, seed=1, dist="baseline", with_s0=True)
        dev = lambda x, dt=torch.bfloat16: torch.from_numpy(x).cuda().to(dt)  # noqa: E731
        q, k, v = dev(inp.q), dev(inp.k), dev(inp.v)
        g, beta, s0 = dev(inp.g, torch.float32), dev(inp.beta, torch.float32), dev(inp.s0, torch.float32)
    else:
        gen = torch.Generator(device="cuda").manual_seed(44)
        n = lambda *s: torch.randn(*s, device="cuda", generator=gen)  # noqa: E731
        q = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
        k = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
        v = n(B, T, HV, D).bfloat16()
        beta, g = torch.sigmoid(n(B, T, HV)), -torch.nn.functional.softplus(n(B, T, HV))
        s0 = n(B, HV, D, D) * 0.02
    o, sf = gdn_b200.chunk_prefill(q, k, v, g, beta, s0)
    torch.cuda.synchronize()
    # ours timed the way theirs is: through the C ABI with the buffers allocated beforehand
    ours = gdn_b200.load_library()
    vp = ctypes.c_void_p
    stream = vp(torch.cuda.current_stream().cuda_stream)
    o_t, sf_t = torch.empty_like(v), torch.empty(B, HV, D, D, device="cuda")
    ws_t = torch.zeros(256, dtype=torch.uint8, device="cuda")
    ours_us = _time(lambda: ours.deltanet_chunk_prefill(  # noqa: E731
        vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(g.data_ptr()), vp(beta.data_ptr()),
        vp(o_t.data_ptr()), vp(s0.data_ptr()), vp(sf_t.data_ptr()), B, T, HV, HQK, D, D, 64, vp(ws_t.data_ptr()),
        256, stream, 0))
    nb = B if cfg == "config1" else 4  # sequences compared (config 4: the first four of 32)
    host = lambda t: t[:nb].float().cpu().numpy()  # noqa: E731
    o_h, sf_h = host(o), host(sf)
    lines = [f"{cfg}: ours {ours_us:.1f} us"]
    for pre, name in (("deltanet", "canonical"), ("deltanet_tcop", "tco")):
        nbytes = getattr(lib, f"{pre}_prefill_workspace_size")(B, T, HV, D, D, 64)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        o_r = torch.empty_like(v)
        sf_r = torch.empty(B, HV, D, D, device="cuda")
        fn = getattr(lib, f"{pre}_chunk_prefill")
        call = lambda: fn(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(g.data_ptr()),  # noqa: E731
                          vp(beta.data_ptr()), vp(o_r.data_ptr()), vp(s0.data_ptr()), vp(sf_r.data_ptr()),
                          B, T, HV, HQK, D, D, 64, vp(ws.data_ptr()), nbytes, stream, 0)
        assert call() == 0
        torch.cuda.synchronize()
        us = _time(call)
        m = _bars(o_h, host(o_r), sf_h, host(sf_r), f"{cfg} ours vs reference {name}")
        lines.append(f"reference {name} {us:.1f} us ({us / ours_us:.1f}x ours; o max-abs {m['o_abs']:.1e}, "
                     f"state rel {m['st_rel']:.1e})")
        del ws
    warnings.warn("reference-kernel comparison on this B200: " + "; ".join(lines))
