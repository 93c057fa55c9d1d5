"""Torch-facing binding over the C ABI (include/gdn_prefill.h).

Mirrors the reference's pybind wrapper ``kernels/torch_binding.cpp``:
``chunk_prefill(q, k, v, g, beta, s0=None) -> [o, sf]`` with the same input
checks (:89-101: CUDA tensors, bf16 q/k/v, fp32 g/beta, ranks 4/4/3), the same
s0 handling (:45-48: converted to contiguous fp32) and an error raised on any
non-success return (:55). ``chunk_prefill_debug`` returns the reference debug
entry's list of per-chunk views (:57-84); ``chunk_prefill_debug_native`` this
kernel's own records. Calls go through ctypes to ``libgdn_b200.so`` on torch's current
CUDA stream; outputs and the workspace are allocated with torch.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from ._lib import cuda_error_string, load_library

__all__ = ["chunk_prefill", "chunk_prefill_debug", "chunk_prefill_debug_native", "chunk_prefill_gated", "chunk_prefill_varlen",
           "run_chunk_prefill", "recurrent_decode", "gated_rmsnorm", "chunk_gated_delta_rule_fast", "workspace_size", "GdnError", "read_status"]

CHUNK = 64
HEAD_DIM = 128
DBG_REC = 64 + 4096 + 3 * 8192 + 16384


class GdnError(RuntimeError):
    """A C-ABI call returned a CUDA error."""


def _check(code: int, what: str):
    if code != 0:
        raise GdnError(f"{what} failed: {cuda_error_string(code)} ({code})")


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _same_device(*ts):
    """Every given tensor on one CUDA device; returns that device."""
    ts = [t for t in ts if t is not None]
    dev = ts[0].device
    if any(t.device != dev for t in ts):
        raise ValueError("all tensors must be on the same CUDA device")
    return dev


_ws_lock = threading.Lock()
_ws_cache: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device workspace (status header), zeroed on first use and reused."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


def workspace_size(B: int, T: int, HV: int, debug: bool = False) -> int:
    lib = load_library()
    fn = lib.deltanet_prefill_debug_workspace_size if debug else lib.deltanet_prefill_workspace_size
    return int(fn(B, T, HV, HEAD_DIM, HEAD_DIM, CHUNK))


def read_status(device=None, clear: bool = True) -> int:
    """Device status word of the cached workspace (0 = clean; bit 0 = a bounded wait timed out)."""
    lib = load_library()
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    ws = _workspace(dev, 256)
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _check(lib.deltanet_read_status(_ptr(ws), ctypes.byref(out), int(clear), _stream()), "deltanet_read_status")
    return out.value


def _check_inputs(q, k, v, g, beta, varlen=False):
    if not all(t.is_cuda for t in (q, k, v, g, beta)):
        raise ValueError("all inputs must be CUDA tensors")
    _same_device(q, k, v, g, beta)
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise ValueError("q/k/v must be bf16")
    if g.dtype != torch.float32 or beta.dtype != torch.float32:
        raise ValueError("g/beta must be fp32")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4 or g.dim() != 3 or beta.dim() != 3:
        raise ValueError("bad ranks: q/k/v must be 4-D [B,T,H,D], g/beta 3-D [B,T,HV]")
    B, T, HQK, DK = q.shape
    HV, DV = v.shape[2], v.shape[3]
    if k.shape != q.shape or v.shape[:2] != (B, T) or g.shape != (B, T, HV) or beta.shape != (B, T, HV):
        raise ValueError("shape mismatch between q/k/v/g/beta")
    if HQK <= 0 or HV % HQK != 0:
        raise ValueError("HV must be a multiple of HQK")
    if DK != HEAD_DIM or DV != HEAD_DIM:
        raise ValueError("only DK = DV = 128 is supported")
    if varlen and B != 1:
        raise ValueError("varlen inputs are packed: B must be 1")
    return B, T, HQK, HV


def _state(s0, shape, device):
    if s0 is None:
        return None
    s0 = s0.to(device=device, dtype=torch.float32).contiguous()
    if tuple(s0.shape) != tuple(shape):
        raise ValueError(f"initial state must have shape {tuple(shape)}, got {tuple(s0.shape)}")
    return s0


def _run_prefill(q, k, v, g, beta, s0, debug: bool):
    B, T, HQK, HV = _check_inputs(q, k, v, g, beta)
    lib = load_library()
    q, k, v, g, beta = (t.contiguous() for t in (q, k, v, g, beta))
    dev = q.device
    o = torch.empty_like(v)
    sf = torch.empty(B, HV, HEAD_DIM, HEAD_DIM, device=dev, dtype=torch.float32)
    s0 = _state(s0, (B, HV, HEAD_DIM, HEAD_DIM), dev)
    if debug:
        nbytes = workspace_size(B, T, HV, debug=True)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    else:
        nbytes = workspace_size(B, T, HV)
        ws = _workspace(dev, nbytes)
    with torch.cuda.device(dev):
        code = lib.deltanet_chunk_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(o), _ptr(s0),
                                          _ptr(sf), B, T, HV, HQK, HEAD_DIM, HEAD_DIM, CHUNK, _ptr(ws),
                                          ws.numel(), _stream(), int(debug))
    _check(code, "deltanet_chunk_prefill")
    if not debug:
        return [o, sf]
    NC = (T + CHUNK - 1) // CHUNK
    rec = ws[256:256 + B * HV * NC * DBG_REC * 4].view(torch.float32).view(B, HV, NC, DBG_REC)
    off = 0
    views = []
    for n, shp in (("c", (CHUNK,)), ("T", (CHUNK, CHUNK)), ("W", (CHUNK, HEAD_DIM)),
                   ("v_new", (CHUNK, HEAD_DIM)), ("o", (CHUNK, HEAD_DIM)), ("S_entry", (HEAD_DIM, HEAD_DIM))):
        sz = 1
        for d in shp:
            sz *= d
        views.append(rec[..., off:off + sz].reshape(B, HV, NC, *shp))
        off += sz
    return [o, sf, *views]


def chunk_prefill(q, k, v, g, beta, s0=None):
    """Chunked gated delta rule prefill: returns [o (bf16 [B,T,HV,128]), final_state (fp32 [B,HV,128,128])].

    Same contract as the reference binding ``chunk_prefill`` (kernels/torch_binding.cpp:113-117):
    q/k bf16 [B,T,HQK,128] pre-L2-normalised, v bf16 [B,T,HV,128], g/beta fp32 [B,T,HV],
    optional s0 fp32 [B,HV,128,128]; the 1/sqrt(128) query scale is applied inside.
    """
    return _run_prefill(q, k, v, g, beta, s0, debug=False)


def chunk_prefill_debug_native(q, k, v, g, beta, s0=None):
    """[o, sf, c, T, W, v_new, o_fp32, S_entry]: this kernel's per-chunk intermediates, each [B, HV, NC, ...].

    The kernel keeps its intermediates on chip; with the debug flag it dumps them: in-chunk
    cumsum c, T = (I+L)^-1, W = T diag(beta e^c) K, v_new = U - W S, o before rounding, and the
    chunk-entry state.
    """
    return _run_prefill(q, k, v, g, beta, s0, debug=True)


def chunk_prefill_debug(q, k, v, g, beta, s0=None):
    """The reference's debug entry (kernels/torch_binding.cpp:119-124, views carved at :57-84):
    [o, sf, w, u, de, eg, ed, gl, Sc, M, T, A, T_post_leaf], per chunk and fp32:

    * w [B,HV,NC,64,DV] = T (v beta), u [B,HV,NC,64,DK] = T (k beta e^c) (chunk_delta_cuda.cu:268-282);
    * de [B,HV,NC,64,64] = e^{c_i - c_j} for i >= j else 0, eg = e^c, ed = e^{c_L - c} [B,HV,NC,64],
      gl = e^{c_L} [B,HV,NC] (:284-294);
    * Sc [B,HV,NC,DK,DV] the chunk-entry states; M = scale (q k^T) de (:480-509);
    * T = (I - A)^-1, A the assembled strict-lower -(beta k k^T) de (:158-175), and T_post_leaf:
      T after its 16 x 16 diagonal leaves are inverted, the other blocks still holding A (:176-214).

    o, sf, T, u (= this kernel's W), Sc and the cumsum c behind the decay terms are the kernel's
    own dumps (``chunk_prefill_debug_native``); w, A, M and the leaf stage, which this kernel does
    not form in that shape (its U enters C12 through T' = T diag(beta), its inverse is not a leaf
    doubling), are formed from those dumps and the inputs with fp32 tensor ops on the same device.
    """
    o, sf, c, T, W, _vnew, _of, sc = _run_prefill(q, k, v, g, beta, s0, debug=True)
    B, T_len, HQK, HV = q.shape[0], q.shape[1], q.shape[2], v.shape[2]
    NC = c.shape[2]
    pad = NC * CHUNK - T_len

    def chunked(x):  # [B, T, H, D] -> [B, HV, NC, 64, D] fp32, zero tail, heads expanded h // (HV / HQK)
        x = torch.nn.functional.pad(x.float().permute(0, 2, 1, 3), (0, 0, 0, pad))
        x = x.reshape(B, x.shape[1], NC, CHUNK, x.shape[-1])
        return x.repeat_interleave(HV // x.shape[1], dim=1) if x.shape[1] != HV else x

    kc, qc, vc = chunked(k), chunked(q), chunked(v)
    bc = torch.nn.functional.pad(beta.float().permute(0, 2, 1), (0, pad)).reshape(B, HV, NC, CHUNK)
    c = c.float()
    tri = torch.ones(CHUNK, CHUNK, dtype=torch.bool, device=c.device).tril()
    strict = tri.tril(-1)
    diff = c[..., :, None] - c[..., None, :]
    de = torch.where(tri, torch.exp(torch.where(tri, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
    eg = torch.exp(c)
    ed = torch.exp(c[..., -1:] - c)
    gl = torch.exp(c[..., -1]).contiguous()
    kk = kc @ kc.transpose(-1, -2)
    A = torch.where(strict, -(bc[..., None] * kk) * de, torch.zeros_like(kk))
    M = (qc @ kc.transpose(-1, -2)) * de * (1.0 / HEAD_DIM ** 0.5)
    w = T @ (vc * bc[..., None])
    post = A.clone()
    eye16 = torch.eye(16, dtype=torch.float32, device=c.device)
    for bl in range(CHUNK // 16):
        blk = slice(16 * bl, 16 * bl + 16)
        post[..., blk, blk] = torch.linalg.solve_triangular(eye16 - A[..., blk, blk], eye16.expand_as(A[..., blk, blk]),
                                                            upper=False, unitriangular=True)
    return [o, sf, w, W, de, eg, ed, gl, sc, M, T, A, post]


def chunk_prefill_gated(q, k, v, g, beta, z, w, s0=None, eps: float = 1e-6):
    """Prefill with the gated RMSNorm fused: returns [y (bf16 [B,T,HV,128]), final_state].

    y = bf16(w * bf16(o * rsqrt(mean(o^2) + eps)) * silu(z)) with o the bf16 GDN output,
    the semantics of the reference's gated_rmsnorm plugin (gatedRmsNormKernel.cu:21-54).
    """
    B, T, HQK, HV = _check_inputs(q, k, v, g, beta)
    if not (z.is_cuda and w.is_cuda) or z.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("z and w must be bf16 CUDA tensors")
    if tuple(z.shape) != tuple(v.shape) or tuple(w.shape) != (HEAD_DIM,):
        raise ValueError("z must match v's shape and w must be [128]")
    _same_device(q, z, w)
    lib = load_library()
    q, k, v, g, beta, z, w = (t.contiguous() for t in (q, k, v, g, beta, z, w))
    dev = q.device
    y = torch.empty_like(v)
    sf = torch.empty(B, HV, HEAD_DIM, HEAD_DIM, device=dev, dtype=torch.float32)
    s0 = _state(s0, (B, HV, HEAD_DIM, HEAD_DIM), dev)
    ws = _workspace(dev, workspace_size(B, T, HV))
    with torch.cuda.device(dev):
        code = lib.deltanet_chunk_prefill_gated(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(z), _ptr(w),
                                                float(eps), _ptr(y), _ptr(s0), _ptr(sf), B, T, HV, HQK, HEAD_DIM,
                                                HEAD_DIM, CHUNK, _ptr(ws), ws.numel(), _stream())
    _check(code, "deltanet_chunk_prefill_gated")
    return [y, sf]


def chunk_prefill_varlen(q, k, v, g, beta, cu_seqlens, s0=None, z=None, w=None, eps: float = 1e-6):
    """Packed variable-length prefill (B = 1): returns [o or y, final_states [N,HV,128,128]].

    ``cu_seqlens`` is int32 [N+1] (on the device); sequence i covers tokens
    [cu[i], cu[i+1]) and starts from s0[i] (or zeros). When z and w are given
    the gated RMSNorm is fused and the first output is y.
    """
    _, T, HQK, HV = _check_inputs(q, k, v, g, beta, varlen=True)
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or not cu_seqlens.is_cuda:
        raise ValueError("cu_seqlens must be a 1-D int32 CUDA tensor")
    N = cu_seqlens.numel() - 1
    _same_device(q, cu_seqlens, z, w)
    if (z is None) != (w is None):
        raise ValueError("pass both z and w (fused norm) or neither")
    lib = load_library()
    q, k, v, g, beta = (t.contiguous() for t in (q, k, v, g, beta))
    cu = cu_seqlens.contiguous()
    if z is not None:
        z, w = z.contiguous(), w.contiguous()
        if z.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or tuple(z.shape) != tuple(v.shape):
            raise ValueError("z must be bf16 with v's shape and w bf16 [128]")
    dev = q.device
    out = torch.empty_like(v)
    sf = torch.empty(N, HV, HEAD_DIM, HEAD_DIM, device=dev, dtype=torch.float32)
    s0 = _state(s0, (N, HV, HEAD_DIM, HEAD_DIM), dev)
    ws = _workspace(dev, workspace_size(1, T, HV))
    with torch.cuda.device(dev):
        code = lib.deltanet_chunk_prefill_varlen(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(z), _ptr(w),
                                                 float(eps), _ptr(out), _ptr(s0), _ptr(sf), _ptr(cu), N, T, HV, HQK,
                                                 HEAD_DIM, HEAD_DIM, CHUNK, _ptr(ws), ws.numel(), _stream())
    _check(code, "deltanet_chunk_prefill_varlen")
    return [out, sf]


def segment_bounds(B: int, T: int, segments: int):
    """Cut each of B sequences of T tokens into at most ``segments`` runs of whole chunks.

    Returns (cu_seqlens over the B*T packed tokens as a list of ints, segments per sequence).
    Every segment but the last of a sequence is a multiple of the chunk length, so the
    chunking inside a segment is the chunking of the whole sequence. This is the cut the
    segmented kernels make (segment j of a sequence covers tokens [j p 64, min((j+1) p 64, T))
    with p = ceil(chunks / segments) chunks per segment); the host-side form serves tests.
    """
    if B < 1 or T < 1 or segments < 1:
        raise ValueError("B, T and segments must be positive")
    nc = (T + CHUNK - 1) // CHUNK
    per = (nc + min(segments, nc) - 1) // min(segments, nc)  # chunks per segment
    starts = list(range(0, T, per * CHUNK))
    cu = []
    for b in range(B):
        cu.extend(b * T + t for t in starts)
    cu.append(B * T)
    return cu, len(starts)


def segment_entry_states(Phi, A, s0=None):
    """Entry states of consecutive segments: S_0 = s0 (zeros if None), S_{j+1} = Phi_j S_j + A_j.

    Phi, A: [B, nseg, HV, d, d] (segment maps of each sequence, in order); s0: [B, HV, d, d].
    Returns float32 [B, nseg, HV, d, d]. The host-side form of the scan the segmented call runs
    on the device (there in fp32, a block per 8 state columns); here in float64, for tests.
    """
    B, nseg, HV, d = A.shape[0], A.shape[1], A.shape[2], A.shape[3]
    Phi = Phi.double().transpose(0, 1).reshape(nseg, B * HV, d, d)
    A = A.double().transpose(0, 1).reshape(nseg, B * HV, d, d)
    S = (torch.zeros_like(A[0]) if s0 is None
         else s0.to(device=A.device, dtype=torch.float64).reshape(B * HV, d, d))
    states = [S]
    for j in range(nseg - 1):
        S = torch.baddbmm(A[j], Phi[j], S)
        states.append(S)
    return torch.stack(states, dim=1).view(B, HV, nseg, d, d).transpose(1, 2).float().contiguous()


def segmented_plan(B: int, T: int, HV: int, segments: int = 0):
    """The plan ``deltanet_chunk_prefill_segmented`` makes for these sizes on the current device:
    (segments per sequence, chunks per segment, kernel), kernel 0 = one pass (the plain call),
    1 = one CTA per (segment, head), 2 = a 4-CTA cluster per (segment, head)."""
    if B < 0 or T < 0 or HV <= 0 or segments < 0:
        raise ValueError("B, T >= 0, HV > 0 and segments >= 0 required")
    lib = load_library()
    nseg, per, kernel = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _check(lib.deltanet_segmented_plan(B, T, HV, segments, ctypes.byref(nseg), ctypes.byref(per), ctypes.byref(kernel)),
           "deltanet_segmented_plan")
    return nseg.value, per.value, kernel.value


def chunk_prefill_segmented(q, k, v, g, beta, s0=None, z=None, w=None, eps: float = 1e-6,
                            segments: int | None = None):
    """Prefill of long sequences cut into segments that run in parallel: [o or y, final_state].

    Same inputs and results as ``chunk_prefill`` (or ``chunk_prefill_gated`` when z and w are
    given), for a few long sequences: one 65,536-token stream over 4 v-heads is a 1,024-step
    chain on 4 clusters of the split kernel, with most of the GPU idle. The state update of a
    chunk, S <- (e^{cL} I - K^T diag(e^{cL-c}) W) S + K^T diag(e^{cL-c}) U, is affine in S, so a
    run of chunks maps its entry state as S_end = Phi S_start + A. ``deltanet_chunk_prefill_segmented``
    cuts each sequence at chunk boundaries into segments and runs, on the current stream:
      1. one grid with every segment from a zero state (A) and from the identity with v = 0 (Phi);
      2. a device scan S_{j+1} = Phi_j S_j + A_j of the entry states, from s0;
      3. every segment from its entry state, which produces the output and the final state.
    ``segments`` (per sequence) defaults to the library's choice for this device and shape, which
    is one pass when the heads alone fill the GPU.
    """
    B, T, HQK, HV = _check_inputs(q, k, v, g, beta)
    if (z is None) != (w is None):
        raise ValueError("pass both z and w (fused norm) or neither")
    if z is not None and (z.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or not z.is_cuda or not w.is_cuda
                          or tuple(z.shape) != tuple(v.shape) or tuple(w.shape) != (HEAD_DIM,)):
        raise ValueError("z must be a bf16 CUDA tensor of v's shape and w a bf16 CUDA tensor [128]")
    dev = _same_device(q, z, w)
    seg = 0 if segments is None else int(segments)
    if seg < 0:
        raise ValueError("segments must be >= 0 (0: the library's choice)")
    lib = load_library()
    q, k, v, g, beta = (t.contiguous() for t in (q, k, v, g, beta))
    if z is not None:
        z, w = z.contiguous(), w.contiguous()
    out = torch.empty_like(v)
    sf = torch.empty(B, HV, HEAD_DIM, HEAD_DIM, device=dev, dtype=torch.float32)
    s0 = _state(s0, (B, HV, HEAD_DIM, HEAD_DIM), dev)
    with torch.cuda.device(dev):
        ws = _workspace(dev, int(lib.deltanet_segmented_workspace_size(B, T, HV, HEAD_DIM, HEAD_DIM, CHUNK, seg)))
        code = lib.deltanet_chunk_prefill_segmented(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(z), _ptr(w),
                                                    float(eps), _ptr(out), _ptr(s0), _ptr(sf), B, T, HV, HQK,
                                                    HEAD_DIM, HEAD_DIM, CHUNK, seg, _ptr(ws), ws.numel(), _stream())
    _check(code, "deltanet_chunk_prefill_segmented")
    return [out, sf]


def gated_rmsnorm(o, z, w, eps: float = 1e-6):
    """Standalone gated RMSNorm over the last dim (fp16 or bf16 I/O): the reference's
    ``kernel::gatedRmsNormForward`` (gatedRmsNormKernel.h:16) / ``gated_rmsnorm`` plugin."""
    if o.dtype not in (torch.float16, torch.bfloat16) or z.dtype != o.dtype or w.dtype != o.dtype:
        raise ValueError("o, z, w must share dtype fp16 or bf16")
    if tuple(z.shape) != tuple(o.shape) or w.dim() != 1 or w.shape[0] != o.shape[-1]:
        raise ValueError("z must match o and w must be [dv]")
    if not (o.is_cuda and z.is_cuda and w.is_cuda):
        raise ValueError("all inputs must be CUDA tensors")
    dev = _same_device(o, z, w)
    lib = load_library()
    o, z, w = o.contiguous(), z.contiguous(), w.contiguous()
    y = torch.empty_like(o)
    dv = o.shape[-1]
    rows = o.numel() // dv if dv else 0
    with torch.cuda.device(dev):
        code = lib.gated_rmsnorm_forward(_ptr(o), _ptr(z), _ptr(w), _ptr(y), rows, dv, float(eps),
                                         0 if o.dtype == torch.float16 else 1, _stream())
    _check(code, "gated_rmsnorm_forward")
    return y


def run_chunk_prefill(q, k, v, a, b, A_log, dt_bias, h0, z=None, norm_w=None, eps: float = 1e-6):
    """The reference's TRT prefill adapter (runGdnChunkPrefillSm87, gdnChunkPrefillSm87.cu:186-320) as one
    fused launch: fp16 q/k [n,T,h,128] (not normalised), v [n,T,hv,128], a/b [n,T,hv], dt_bias [hv],
    fp32 A_log [hv]; h0 fp32 [n,hv,128,128] holds the initial state and receives the final state in place.
    Returns o (fp16 [n,T,hv,128]), or y when z and norm_w (fp16) are given."""
    for t in (q, k, v, a, b, dt_bias) + ((z, norm_w) if z is not None else ()):
        if t.dtype != torch.float16 or not t.is_cuda:
            raise ValueError("q, k, v, a, b, dt_bias (and z, norm_w) must be fp16 CUDA tensors")
    if A_log.dtype != torch.float32 or h0.dtype != torch.float32 or not h0.is_contiguous():
        raise ValueError("A_log must be fp32 and h0 a contiguous fp32 tensor")
    from ._lib import GdnPrefillParams
    _same_device(q, k, v, a, b, A_log, dt_bias, h0, z, norm_w)
    lib = load_library()
    n, T, h, kd = q.shape
    hv, vd = v.shape[2], v.shape[3]
    q, k, v, a, b, A_log, dt_bias = (t.contiguous() for t in (q, k, v, a, b, A_log, dt_bias))
    if z is not None:
        z, norm_w = z.contiguous(), norm_w.contiguous()
    o = torch.empty_like(v)
    ws = _workspace(q.device, workspace_size(n, T, hv))
    prm = GdnPrefillParams(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), a=a.data_ptr(), b=b.data_ptr(),
                           A_log=A_log.data_ptr(), dt_bias=dt_bias.data_ptr(), h0_source=h0.data_ptr(),
                           o=o.data_ptr(), z=None if z is None else z.data_ptr(),
                           norm_w=None if norm_w is None else norm_w.data_ptr(), eps=float(eps), n=n, seq_len=T, h=h,
                           hv=hv, k_dim=kd, v_dim=vd, workspace=ws.data_ptr(), workspace_bytes=ws.numel())
    with torch.cuda.device(q.device):
        rc = lib.gdn_run_chunk_prefill(ctypes.byref(prm), _stream())
    if rc != 0:
        raise GdnError("gdn_run_chunk_prefill failed (see stderr)")
    return o


def recurrent_decode(q, k, v, g, beta, state, z=None, w=None, eps: float = 1e-6):
    """Decode step(s): q/k bf16 [B,T,HQK,128], v bf16 [B,T,HV,128], g/beta fp32 [B,T,HV]; the fp32
    ``state`` [B,HV,128,128] (e.g. a prefill's final state) is updated in place. Returns o (or y with
    z, w bf16) [B,T,HV,128]; semantics of transformers ``torch_recurrent_gated_delta_rule``."""
    B, T, HQK, HV = _check_inputs(q, k, v, g, beta)
    if state.dtype != torch.float32 or not state.is_contiguous() or tuple(state.shape) != (B, HV, HEAD_DIM, HEAD_DIM):
        raise ValueError("state must be a contiguous fp32 [B, HV, 128, 128] tensor")
    if (z is None) != (w is None):
        raise ValueError("pass both z and w (fused norm) or neither")
    dev = _same_device(q, state, z, w)
    lib = load_library()
    q, k, v, g, beta = (t.contiguous() for t in (q, k, v, g, beta))
    if z is not None:
        z, w = z.contiguous(), w.contiguous()
    out = torch.empty_like(v)
    with torch.cuda.device(dev):
        code = lib.deltanet_recurrent_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(z), _ptr(w), float(eps),
                                             _ptr(out), _ptr(state), B, T, HV, HQK, HEAD_DIM, HEAD_DIM, _stream())
    _check(code, "deltanet_recurrent_decode")
    return out


def _l2norm_fp32(x):
    inv = torch.rsqrt((x.float() * x.float()).sum(-1, keepdim=True) + 1e-6)
    return (x.float() * inv).to(torch.bfloat16)


def chunk_gated_delta_rule_fast(query, key, value, g, beta, chunk_size=64, initial_state=None,
                                output_final_state=True, use_qk_l2norm_in_kernel=False):
    """transformers-compatible signature (the reference's twin,
    kernels/harness/chunk_delta.py:361-368): returns (o, final_state or None).

    q/k may carry HQK heads (grouped) or HV heads; with use_qk_l2norm_in_kernel
    they are L2-normalised in fp32 and rounded to bf16 first, as the
    reference's adapter does (gdnChunkPrefillSm87.cu:52-85).
    """
    if chunk_size != CHUNK:
        raise ValueError("only chunk_size=64 is supported")
    if use_qk_l2norm_in_kernel:
        query, key = _l2norm_fp32(query), _l2norm_fp32(key)
    o, sf = chunk_prefill(query.to(torch.bfloat16), key.to(torch.bfloat16), value.to(torch.bfloat16),
                          g.float(), beta.float(), initial_state)
    return o, (sf if output_final_state else None)
