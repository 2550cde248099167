"""bench.py's host-side pieces (no GPU): the reference arm times the unmodified reference for the
steps it reports, and the roofline denominators come from the committed machine-readable
records."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_reports_what_it_timed():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1", "--cpu-sample-params", "3000000"], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1
    assert line["unit"] == "Gparams/s" and line["higher_is_better"] is True
    assert line["e2e"] == {"value": line["value"], "unit": "Gparams/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    cfg1 = line["config1"]
    assert cfg1["params"] == 8_912_896 and cfg1["steps"] == 9 and cfg1["warmup"] == 1
    assert 2.9 < cfg1["last_norm"] < 3.1  # every step of configuration 1 clips


def test_link_peak_and_traffic_records():
    peak, src = bench.measured_link_peak(8)
    assert src.startswith("measured") and 500 < peak < 900
    peak2, _ = bench.measured_link_peak(2)
    assert peak2 >= 700
    for mode in ("full", "changed groups"):
        tpp, path = bench.profiled_traffic_per_param(mode)
        assert path is not None and 25.0 < tpp < 29.0


def test_sampled_positions_cover_every_tensor_edge():
    import torch
    numels = [5, 1, 70000, 3]
    sp = bench.SampledParity(numels, per_rank=50, world=2, seed=3, dev=torch.device("cpu"))
    starts = {0, 5, 6, 70006}
    got = set()
    for i, idx in sp.groups:
        base = [0, 5, 6, 70006][i]
        got.update(base + int(x) for x in idx)
    assert starts <= got and {4, 5, 70005, 70008} <= got
    assert sp.k == len(got)


def test_phase_roofline_names_the_binding_resource():
    # the W=8 push of the Qwen3-8B set: 14.33 GB over NVLink, 32.8 GB in HBM, 20.53 ms
    push = bench.phase_roofline("push", 20.53, 4 * 8_190_735_360, 2 * 7_166_893_440, 6554.9, 705.7)
    assert push["bound"] == "nvlink" and abs(push["link_gbs_achieved"] - 698.2) < 1.0
    assert abs(push["frac"] - push["frac_of_link_peak"]) < 1e-3
    # its update: 26.6 GB in HBM, 83 MB of changed sectors to the peers, 5.0 ms
    upd = bench.phase_roofline("adamw", 5.006, 26.6e9, 82.5e6, 6554.9, 705.7)
    assert upd["bound"] == "hbm" and abs(upd["frac"] - 26.6e9 / 6554.9e9 / 5.006e-3) < 1e-3
