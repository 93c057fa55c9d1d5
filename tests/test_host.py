"""Host-side checks that need no GPU: the C-ABI library loads, exports every
symbol include/gdn_prefill.h declares, and rejects bad arguments with
cudaErrorInvalidValue before touching the device (the reference's error
convention, kernels/chunk_delta_cuda.cu:706-727)."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
import gdn_b200
from gdn_b200 import _lib

INVALID = 1  # cudaErrorInvalidValue


def header_functions():
    text = (ROOT / "include" / "gdn_prefill.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)) - {"defined"})


def test_header_declares_reference_entry_points():
    names = header_functions()
    # the reference's C ABI (kernels/chunk_delta_cuda.h:39-55, chunk_delta_cuda_tco.h:39-55)
    for n in ("deltanet_prefill_workspace_size", "deltanet_chunk_prefill",
              "deltanet_tcop_prefill_workspace_size", "deltanet_tcop_chunk_prefill"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = gdn_b200.load_library()
    raw = ctypes.CDLL(str(_lib.library_path()))
    for n in header_functions():
        assert hasattr(raw, n), f"libgdn_b200.so does not export {n}"
        assert n in _lib.SIGNATURES, f"no ctypes signature for {n}"
    assert b"sm_100a" in lib.gdn_b200_version()


def test_workspace_size_is_small_and_constant():
    lib = gdn_b200.load_library()
    a = lib.deltanet_prefill_workspace_size(1, 1141, 32, 128, 128, 64)
    b = lib.deltanet_prefill_workspace_size(32, 4096, 32, 128, 128, 64)
    assert a == b == 256
    assert lib.deltanet_tcop_prefill_workspace_size(1, 1141, 32, 128, 128, 64) == a
    dbg = lib.deltanet_prefill_debug_workspace_size(1, 1141, 32, 128, 128, 64)
    assert dbg == 256 + 1 * 32 * 18 * (64 + 4096 + 3 * 8192 + 16384) * 4


def _call(lib, **kw):
    args = dict(q=1 << 20, k=1 << 20, v=1 << 20, g=1 << 20, beta=1 << 20, o=1 << 20, s0=None, sf=1 << 20,
                B=1, T=64, HV=2, HQK=1, DK=128, DV=128, chunk=64, ws=1 << 20, ws_bytes=256, dbg=0)
    args.update(kw)
    vp = ctypes.c_void_p
    return lib.deltanet_chunk_prefill(vp(args["q"]), vp(args["k"]), vp(args["v"]), vp(args["g"]),
                                      vp(args["beta"]), vp(args["o"]), vp(args["s0"]), vp(args["sf"]),
                                      args["B"], args["T"], args["HV"], args["HQK"], args["DK"], args["DV"],
                                      args["chunk"], vp(args["ws"]), args["ws_bytes"], None, args["dbg"])


@pytest.mark.parametrize("bad", [dict(DK=64), dict(DV=256), dict(chunk=32), dict(HQK=3), dict(HQK=0),
                                 dict(ws=None), dict(ws_bytes=16), dict(q=None), dict(sf=None),
                                 dict(q=(1 << 20) + 2), dict(T=-1), dict(dbg=1)])
def test_invalid_arguments_rejected(bad):
    lib = gdn_b200.load_library()
    assert _call(lib, **bad) == INVALID


def test_varlen_and_gated_argument_checks():
    lib = gdn_b200.load_library()
    vp = ctypes.c_void_p
    p = vp(1 << 20)
    # gated: z without weight
    assert lib.deltanet_chunk_prefill_gated(p, p, p, p, p, p, None, 1e-6, p, None, p, 1, 64, 2, 1, 128, 128, 64,
                                            p, 256, None) == INVALID
    # varlen: null cu_seqlens / z without weight
    assert lib.deltanet_chunk_prefill_varlen(p, p, p, p, p, None, None, 1e-6, p, None, p, None, 2, 64, 2, 1,
                                             128, 128, 64, p, 256, None) == INVALID
    assert lib.deltanet_chunk_prefill_varlen(p, p, p, p, p, p, None, 1e-6, p, None, p, p, 2, 64, 2, 1,
                                             128, 128, 64, p, 256, None) == INVALID
    # standalone norm: bad dtype / dv
    assert lib.gated_rmsnorm_forward(p, p, p, p, 10, 128, 1e-6, 7, None) == INVALID
    assert lib.gated_rmsnorm_forward(p, p, p, p, 10, 0, 1e-6, 1, None) == INVALID
    assert lib.gated_rmsnorm_forward(p, p, p, p, 0, 128, 1e-6, 1, None) == 0  # empty is a no-op


def test_binding_rejects_cpu_and_wrong_dtypes():
    import torch
    q = torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16)
    v = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)
    g = torch.zeros(1, 8, 2)
    with pytest.raises(ValueError):
        gdn_b200.chunk_prefill(q, q, v, g, g)  # CPU tensors
    with pytest.raises(ValueError):
        gdn_b200.binding._check_inputs(q.float(), q, v, g, g)
    with pytest.raises(ValueError):
        gdn_b200.chunk_prefill_segmented(q, q, v, g, g, segments=2)  # CPU tensors, before any launch


def test_product_path_has_no_oracle_import():
    """The shipped package never imports the test oracle (no CPU fallback)."""
    pkg = ROOT / "qwen-drive-edge-orin_b200"
    for f in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")):
        text = f.read_text()
        assert "oracle" not in text.replace("oracle/", "").lower() or f.name == "build.py", f


def test_segmented_workspace_and_argument_checks():
    """deltanet_chunk_prefill_segmented: workspace = status header + one zero tile + the state
    pass's maps A and Phi of every segment but the last ([B (segments - 1), 2 HV, 128, 128] fp32)
    + the entry states ([B segments, HV, 128, 128] fp32) + (passes on the one-CTA kernel, the only
    kernel without a device) a record of T' and W^T tiles per chunk of every segment (48 KB each);
    one segment is the plain call's 256 bytes; bad arguments are rejected before any device work."""
    lib = gdn_b200.load_library()
    D2 = 128 * 128 * 4
    ws = lambda B, HV, s, per: 256 + 64 * 128 * 2 + B * (2 * (s - 1) + s) * HV * D2 + B * s * HV * per * 49152  # noqa: E731
    assert lib.deltanet_segmented_workspace_size(1, 65536, 4, 128, 128, 64, 1) == 256
    assert lib.deltanet_segmented_workspace_size(1, 65536, 4, 128, 128, 64, 9) == ws(1, 4, 9, 114)
    # 1024 chunks in at most 10 segments of 103 chunks: 10 segments
    assert lib.deltanet_segmented_workspace_size(2, 65536, 4, 128, 128, 64, 10) == ws(2, 4, 10, 103)
    # 300 tokens = 5 chunks: 4 requested -> 2 chunks per segment -> 3 segments
    assert lib.deltanet_segmented_workspace_size(1, 300, 2, 128, 128, 64, 4) == ws(1, 2, 3, 2)
    p = ctypes.c_void_p(1 << 20)
    args = [p, p, p, p, p, None, None, ctypes.c_float(1e-6), p, None, p]
    call = lambda *a: lib.deltanet_chunk_prefill_segmented(*args, *a)  # noqa: E731
    assert call(1, 64, 2, 1, 64, 64, 64, 2, p, 1 << 20, None) == INVALID          # DK = 64
    assert call(1, 64, 2, 1, 128, 128, 64, -1, p, 1 << 20, None) == INVALID       # segments < 0
    assert lib.deltanet_chunk_prefill_segmented(p, p, p, p, p, p, None, 1e-6, p, None, p, 1, 64, 2, 1, 128, 128,
                                                64, 2, p, 1 << 20, None) == INVALID  # z without norm_w
