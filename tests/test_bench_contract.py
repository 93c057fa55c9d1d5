"""CPU checks of bench.py's roofline arithmetic and its committed inputs.

The bench line's ``roofline.achieved`` is algorithmic bytes per launch divided by the
kernel's event-timed duration, so the byte and FLOP counts must equal the per-unit figures
the design states: 33,024 B per token (HQK=16, HV=32, d=128, bf16 q/k/v/z/y, fp32 g/beta)
plus 2·HV·d²·4 B per sequence for s0 and sf, and 2·(5·C·d + 3·d² + C²/3) FLOP per token
per v-head (182,954.7 at C=64, d=128).
"""
from __future__ import annotations

import json

import pytest

from conftest import ROOT

bench = pytest.importorskip("bench")


def test_bytes_per_token_and_per_sequence():
    per_tok = bench.alg_bytes(1, 1, 16, 32, with_s0=False) - 32 * 128 * 128 * 4
    assert per_tok == 33_024
    assert bench.alg_bytes(1, 0, 16, 32) == 2 * 32 * 128 * 128 * 4


def test_config1_and_config4_totals():
    # config 1: 41.87 MB per call; config 4: 4.463 GB per call (one GPU)
    assert bench.alg_bytes(1, 1141, 16, 32) == 41_874_688
    assert abs(bench.alg_bytes(32, 4096, 16, 32) / 1e9 - 4.463) < 5e-4
    assert abs(bench.alg_flops(1, 1141, 32) / 1e9 - 6.680) < 5e-4


def test_flops_per_token_per_head():
    assert abs(bench.alg_flops(1, 1, 1) - 182_954.67) < 0.01


def test_configs_match_baseline_shapes():
    c1, c4 = bench.CONFIGS[1], bench.CONFIGS[4]
    assert (c1["B"], c1["T"], c1["HQK"], c1["HV"]) == (1, 1141, 16, 32)
    assert (c4["B"], c4["T"], c4["HQK"], c4["HV"]) == (32, 4096, 16, 32)


def test_committed_traffic_and_peaks_are_readable():
    traffic, kernel = bench.load_traffic(1)
    assert traffic is not None and kernel == "gdn::split::gdn_prefill_split_kernel<false>"
    # reads: every input once (q, k, v, z, g, beta, s0); writes: y and sf once. The recorded
    # traffic (DRAM reads + SM writes into L2) is within 10% of the algorithmic bytes.
    d = json.loads((ROOT / "profiles" / "traffic.json").read_text())["config1"]
    must_read = bench.alg_bytes(1, 1141, 16, 32) - 1141 * 32 * 128 * 2 - 32 * 128 * 128 * 4
    assert 0.95 * must_read <= d["dram_bytes_read"] <= 1.05 * must_read
    assert traffic == d["dram_bytes_read"] + d["l2_write_bytes_from_sm"]
    assert 0.95 * bench.alg_bytes(1, 1141, 16, 32) <= traffic <= 1.1 * bench.alg_bytes(1, 1141, 16, 32)
    hbm, tf_burst, tf_sust, kind = bench.load_peaks()
    if (ROOT / "MEASURED_PEAKS.json").exists():
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        assert kind == "measured" and hbm == float(d["hbm_gbs"])
    assert hbm > 1000 and tf_burst > 100


def test_reference_arm_prints_one_json_line():
    """``bench.py --impl reference`` (the driver's reference arm) runs the reference's CPU
    implementation on this host and prints one JSON line with the contract's keys."""
    import subprocess
    import sys
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0 and d["higher_is_better"]
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == bench.CONFIGS[1]["desc"] and d["config"]["seq_len"] == 1141
