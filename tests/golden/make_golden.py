"""Generate the golden vectors under tests/golden/ from the reference's own oracle.

The reference's parity harness takes its oracle from transformers
(``kernels/harness/parity_test.py:22-26``: ``torch_chunk_gated_delta_rule`` and
``l2norm`` from ``transformers.models.qwen3_5.modeling_qwen3_5``), with a
verbatim copy of the same function as its fallback (``parity_test.py:35-96``).
This script runs that oracle on seeded synthetic inputs and stores the
outputs; the inputs are regenerated from the seed by
``gdn_b200.synthetic.make_inputs`` and pinned by a checksum stored alongside.

When the reference checkout is present, the verbatim copy is also extracted
from ``kernels/harness/parity_test.py`` and must reproduce the transformers
outputs bit for bit (a check that the installed transformers 5.5.0 matches the
5.14.1 copy the reference pins).

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import ast
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "qwen-drive-edge-orin_b200"))
from gdn_b200.synthetic import make_inputs, make_cu_seqlens  # noqa: E402

from transformers.models.qwen3_5.modeling_qwen3_5 import (  # noqa: E402
    Qwen3_5RMSNormGated,
    torch_chunk_gated_delta_rule,
    torch_recurrent_gated_delta_rule,
)

# the reference checkout: $GDN_REFERENCE_ROOT, else a `reference` directory beside this repository
REF_ROOT = Path(os.environ.get("GDN_REFERENCE_ROOT") or Path(__file__).resolve().parents[3] / "reference")
REF_HARNESS = REF_ROOT / "kernels/harness/parity_test.py"


def verbatim_ref_chunk():
    """The reference's verbatim fallback copy (parity_test.py:35-96), or None."""
    if not REF_HARNESS.exists():
        return None
    tree = ast.parse(REF_HARNESS.read_text())
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == "_ref_chunk":
            ns = {"torch": torch, "F": F}
            l2 = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef) and n.name == "_ref_l2norm")
            exec(compile(ast.Module(body=[l2, node], type_ignores=[]), str(REF_HARNESS), "exec"), ns)
            return ns["_ref_chunk"]
    return None


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def to_t(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dtype)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def run_ref(inp, hv, dtype, cu=None):
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    q, k = to_t(inp.q, tdt), to_t(inp.k, tdt)
    rep = hv // q.shape[2]
    q, k = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
    v, z = to_t(inp.v, tdt), to_t(inp.z, tdt)
    g, beta = to_t(inp.g, torch.float32), to_t(inp.beta, torch.float32)
    s0 = None if inp.s0 is None else to_t(inp.s0, torch.float32)
    if cu is None:
        o, sf = torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=s0,
                                             output_final_state=True, use_qk_l2norm_in_kernel=False)
    else:
        outs, states = [], []
        for i in range(len(cu) - 1):
            a, b = int(cu[i]), int(cu[i + 1])
            s = None if s0 is None else s0[i:i + 1]
            oi, si = torch_chunk_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                                  chunk_size=64, initial_state=s, output_final_state=True,
                                                  use_qk_l2norm_in_kernel=False)
            outs.append(oi)
            states.append(si)
        o, sf = torch.cat(outs, dim=1), torch.cat(states, dim=0)
    norm = Qwen3_5RMSNormGated(o.shape[-1], eps=inp.eps)
    with torch.no_grad():
        norm.weight.copy_(to_t(inp.w, torch.float32))
        y = norm(o.reshape(-1, o.shape[-1]), z.reshape(-1, z.shape[-1])).reshape(o.shape)
    return o, sf, y, (q, k, v, g, beta, s0)


CASES = [
    # name, dict(make_inputs kwargs), dtype, varlen spec
    ("cfg0_fp32_h4_d64_s256", dict(B=1, T=256, HQK=4, HV=4, D=64, seed=0, dist="baseline", with_s0=False, dtype="fp32"), None),
    ("bf16_b1_s130_hqk1_hv2_s0", dict(B=1, T=130, HQK=1, HV=2, D=128, seed=1, dist="baseline", with_s0=True), None),
    ("bf16_b2_s64_hqk1_hv2_refgrid", dict(B=2, T=64, HQK=1, HV=2, D=128, seed=2, dist="refgrid", with_s0=False), None),
    ("bf16_b1_s1_hqk1_hv2_s0", dict(B=1, T=1, HQK=1, HV=2, D=128, seed=3, dist="refgrid", with_s0=True), None),
    ("bf16_b1_s200_hqk2_hv2_refgrid_s0", dict(B=1, T=200, HQK=2, HV=2, D=128, seed=4, dist="refgrid", with_s0=True), None),
    ("bf16_varlen_70_65_hqk1_hv2", dict(B=1, T=135, HQK=1, HV=2, D=128, seed=5, dist="baseline", with_s0=True, n_states=2),
     [0, 70, 135]),
]


def main():
    ref_copy = verbatim_ref_chunk()
    index = {}
    for name, kw, cu in CASES:
        inp = make_inputs(**kw)
        dtype = kw.get("dtype", "bf16")
        o, sf, y, tens = run_ref(inp, kw["HV"], dtype, cu)
        entry = {"kwargs": kw, "cu_seqlens": cu, "input_sha256": digest(inp.q, inp.k, inp.v, inp.g, inp.beta,
                                                                         inp.z, inp.w, inp.s0)}
        if ref_copy is not None and cu is None:
            q, k, v, g, beta, s0 = tens
            o2, sf2 = ref_copy(q, k, v, g=g, beta=beta, chunk_size=64, initial_state=s0,
                               output_final_state=True, use_qk_l2norm_in_kernel=False)
            same = torch.equal(o2, o) and torch.equal(sf2, sf)
            entry["verbatim_copy_bit_identical"] = bool(same)
            assert same, f"{name}: verbatim reference copy differs from transformers"
        arrays = {"sf": sf.numpy().astype(np.float32)}
        if dtype == "bf16":
            arrays["o_bits"] = bits(o)
            arrays["y_bits"] = bits(y)
        else:
            arrays["o"] = o.numpy().astype(np.float32)
            arrays["y"] = y.numpy().astype(np.float32)
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        index[name] = entry
        print(f"{name}: o{tuple(o.shape)} sf{tuple(sf.shape)} verbatim={entry.get('verbatim_copy_bit_identical')}")

    # decode-step (single-token recurrence) vectors: transformers torch_recurrent_gated_delta_rule
    inp = make_inputs(B=1, T=3, HQK=1, HV=2, D=128, seed=6, dist="baseline", with_s0=True)
    q, k = to_t(inp.q, torch.bfloat16).repeat_interleave(2, 2), to_t(inp.k, torch.bfloat16).repeat_interleave(2, 2)
    o, sf = torch_recurrent_gated_delta_rule(q, k, to_t(inp.v, torch.bfloat16), to_t(inp.g, torch.float32),
                                             to_t(inp.beta, torch.float32), initial_state=to_t(inp.s0, torch.float32),
                                             output_final_state=True, use_qk_l2norm_in_kernel=False)
    np.savez_compressed(HERE / "recurrent_bf16_s3_hv2.npz", o_bits=bits(o), sf=sf.numpy().astype(np.float32))
    index["recurrent_bf16_s3_hv2"] = {"kwargs": dict(B=1, T=3, HQK=1, HV=2, D=128, seed=6, dist="baseline",
                                                     with_s0=True),
                                      "input_sha256": digest(inp.q, inp.k, inp.v, inp.g, inp.beta, inp.z, inp.w,
                                                             inp.s0)}
    meta = {"generator": "transformers.models.qwen3_5.modeling_qwen3_5 (torch CPU, fp32 math)",
            "transformers": __import__("transformers").__version__, "torch": torch.__version__,
            "numpy": np.__version__, "cases": index}
    (HERE / "index.json").write_text(json.dumps(meta, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
