"""The no-allocation entry point, deltanet_chunk_prefill_gated_noalloc.

Some callers cannot allocate device memory when they call the prefill: an
inference engine's enqueue path that forbids cudaMalloc, or a latency-bound loop
where an allocation would synchronise the device. This entry point takes its
scratch (the bounded-wait status word) from a static device array inside the
library, so the caller passes only inputs and outputs. These tests call it
through the C ABI twice in a row and compare each result with the
workspace-taking entry point deltanet_chunk_prefill_gated on the same inputs,
within the parity tolerances the other GPU tests use.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import max_rel, row_cos_min, tensor_l2_rel
import gdn_b200
from gdn_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu

Y_MAX_REL = 2e-2      # as tests/test_gpu_parity.py
STATE_REL = 1e-2
COS_MIN = 0.999


def _dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(dtype)


@pytest.mark.parametrize("B,T,HQK,HV", [(2, 200, 2, 4), (1, 1141, 16, 32)])
def test_noalloc_matches_workspace_entry_twice(B, T, HQK, HV):
    lib = gdn_b200.load_library()
    inp = make_inputs(B, T, HQK, HV, 128, seed=77 + T, dist="baseline", with_s0=True)
    q, k, v, z, w = (_dev(a) for a in (inp.q, inp.k, inp.v, inp.z, inp.w))
    g, beta, s0 = (_dev(a, torch.float32) for a in (inp.g, inp.beta, inp.s0))
    vp = ctypes.c_void_p
    stream = vp(torch.cuda.current_stream().cuda_stream)

    y_ref = torch.empty_like(v)
    sf_ref = torch.empty(B, HV, 128, 128, device="cuda")
    ws = torch.zeros(lib.deltanet_prefill_workspace_size(B, T, HV, 128, 128, 64), dtype=torch.uint8, device="cuda")
    rc = lib.deltanet_chunk_prefill_gated(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(g.data_ptr()),
                                          vp(beta.data_ptr()), vp(z.data_ptr()), vp(w.data_ptr()), 1e-6,
                                          vp(y_ref.data_ptr()), vp(s0.data_ptr()), vp(sf_ref.data_ptr()),
                                          B, T, HV, HQK, 128, 128, 64, vp(ws.data_ptr()), ws.numel(), stream)
    assert rc == 0
    torch.cuda.synchronize()
    y_ref_h, sf_ref_h = y_ref.float().cpu().numpy(), sf_ref.cpu().numpy()

    for call in range(2):  # two calls in a row share the static scratch
        y = torch.full_like(v, float("nan"))
        sf = torch.full((B, HV, 128, 128), float("nan"), device="cuda")
        rc = lib.deltanet_chunk_prefill_gated_noalloc(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()),
                                                      vp(g.data_ptr()), vp(beta.data_ptr()), vp(z.data_ptr()),
                                                      vp(w.data_ptr()), 1e-6, vp(y.data_ptr()), vp(s0.data_ptr()),
                                                      vp(sf.data_ptr()), B, T, HV, HQK, 128, 128, 64, stream)
        assert rc == 0, f"call {call}: cudaError {rc}"
        torch.cuda.synchronize()
        yh, sfh = y.float().cpu().numpy(), sf.cpu().numpy()
        assert np.isfinite(yh).all() and np.isfinite(sfh).all()
        assert row_cos_min(yh, y_ref_h) >= COS_MIN and max_rel(yh, y_ref_h) < Y_MAX_REL
        assert tensor_l2_rel(sfh, sf_ref_h) <= STATE_REL
        print(f"call {call}: identical={np.array_equal(yh, y_ref_h) and np.array_equal(sfh, sf_ref_h)}")


def test_noalloc_status_word_is_readable():
    """A caller of the no-allocation entry has no workspace to hand to deltanet_read_status,
    so deltanet_noalloc_read_status reads the status word of the library's static scratch:
    clean (0) after a normal call, and still 0 after being read with clear set."""
    lib = gdn_b200.load_library()
    B, T, HQK, HV = 1, 300, 2, 4
    inp = make_inputs(B, T, HQK, HV, 128, seed=5, dist="baseline", with_s0=True)
    q, k, v, z, w = (_dev(a) for a in (inp.q, inp.k, inp.v, inp.z, inp.w))
    g, beta, s0 = (_dev(a, torch.float32) for a in (inp.g, inp.beta, inp.s0))
    y = torch.empty_like(v)
    sf = torch.empty(B, HV, 128, 128, device="cuda")
    vp = ctypes.c_void_p
    stream = vp(torch.cuda.current_stream().cuda_stream)
    rc = lib.deltanet_chunk_prefill_gated_noalloc(vp(q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()),
                                                  vp(g.data_ptr()), vp(beta.data_ptr()), vp(z.data_ptr()),
                                                  vp(w.data_ptr()), 1e-6, vp(y.data_ptr()), vp(s0.data_ptr()),
                                                  vp(sf.data_ptr()), B, T, HV, HQK, 128, 128, 64, stream)
    assert rc == 0
    st = ctypes.c_int(-1)
    assert lib.deltanet_noalloc_read_status(ctypes.byref(st), 1, stream) == 0
    assert st.value == 0
    st.value = -1
    assert lib.deltanet_noalloc_read_status(ctypes.byref(st), 0, stream) == 0
    assert st.value == 0
    assert lib.deltanet_noalloc_read_status(None, 0, stream) == 1  # cudaErrorInvalidValue


def test_noalloc_rejects_bad_arguments():
    lib = gdn_b200.load_library()
    p = ctypes.c_void_p(1 << 20)
    # unsupported head dim: rejected before anything is launched
    assert lib.deltanet_chunk_prefill_gated_noalloc(p, p, p, p, p, p, p, 1e-6, p, None, p,
                                                    1, 64, 2, 1, 64, 64, 64, None) == 1
