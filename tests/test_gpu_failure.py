"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait in the prefill kernels is bounded (about 1 s). The test hook
``deltanet_test_withheld_load`` runs the gated prefill with one v-tile TMA load never
issued: a producer that never arrives. The consumer's wait must run out, the kernel must
record bit 0 in the workspace status word, stop, wait (bounded) for the copies and MMAs it
has in flight, free its tensor memory and return, all without a trap or a device assert.
The context must stay usable: the next normal call returns results bit-identical to a
clean call's, with a clean status word. Both kernels are covered: the one-CTA-per-head
kernel and the cluster-split kernel (whose abort path also has to stop its CTAs from
shipping chunks into peers whose slots were not armed).
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

import gdn_b200
from gdn_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

KERNELS = {1: "fused", 2: "split"}


def _dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(dtype)


def _status(lib, ws, clear):
    out = ctypes.c_int(-1)
    rc = lib.deltanet_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(out), int(clear),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return out.value


@pytest.mark.parametrize("kernel", sorted(KERNELS))
def test_withheld_load_times_out_and_the_next_call_is_clean(kernel, monkeypatch):
    monkeypatch.setenv("GDN_B200_KERNEL", KERNELS[kernel])  # the clean calls use the same kernel
    lib = gdn_b200.load_library()
    B, T, HQK, HV = 1, 300, 2, 4  # five chunks; the load of chunk 1's v tile is withheld
    inp = make_inputs(B, T, HQK, HV, 128, seed=61, dist="baseline", with_s0=True)
    q, k, v, z, w = (_dev(a) for a in (inp.q, inp.k, inp.v, inp.z, inp.w))
    g, beta, s0 = (_dev(a, torch.float32) for a in (inp.g, inp.beta, inp.s0))
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    vp = ctypes.c_void_p
    stream = vp(torch.cuda.current_stream().cuda_stream)

    def clean():
        y = torch.full_like(v, float("nan"))
        sf = torch.full((B, HV, 128, 128), float("nan"), device="cuda")
        rc = lib.deltanet_chunk_prefill_gated(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(g.data_ptr()),
                                              vp(beta.data_ptr()), vp(z.data_ptr()), vp(w.data_ptr()), 1e-6,
                                              vp(y.data_ptr()), vp(s0.data_ptr()), vp(sf.data_ptr()), B, T, HV, HQK,
                                              128, 128, 64, vp(ws.data_ptr()), ws.numel(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        return y.float().cpu().numpy(), sf.cpu().numpy()

    y0, sf0 = clean()
    assert _status(lib, ws, clear=True) == 0
    assert np.isfinite(y0).all() and np.isfinite(sf0).all()

    y = torch.empty_like(v)
    sf = torch.empty(B, HV, 128, 128, device="cuda")
    t0 = time.perf_counter()
    rc = lib.deltanet_test_withheld_load(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(g.data_ptr()),
                                         vp(beta.data_ptr()), vp(z.data_ptr()), vp(w.data_ptr()), 1e-6,
                                         vp(y.data_ptr()), vp(s0.data_ptr()), vp(sf.data_ptr()), B, T, HV, HQK,
                                         128, 128, 64, vp(ws.data_ptr()), ws.numel(), stream, kernel, 1)
    assert rc == 0, f"launch returned cudaError {rc}"
    torch.cuda.synchronize()  # raises if the kernel faulted
    elapsed = time.perf_counter() - t0
    status = _status(lib, ws, clear=True)
    print(f"kernel={KERNELS[kernel]}: withheld load -> status {status:#x} after {elapsed:.2f} s")
    assert status & 1, "the bounded wait did not report its timeout"
    assert elapsed < 20.0
    assert _status(lib, ws, clear=False) == 0  # cleared

    y1, sf1 = clean()
    assert _status(lib, ws, clear=False) == 0
    assert np.array_equal(y1, y0) and np.array_equal(sf1, sf0)
