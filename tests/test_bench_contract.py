"""CPU checks of bench.py's contract: the reference arm's JSON line (it runs
the oracle on the host cores) and the helpers that build the GPU line."""
import json
import os
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--cpu-tokens", "64"], capture_output=True, text=True, cwd=ROOT,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "dtype", "data",
              "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["config"]["workload"] == bench.workload_config(bench.T_PER_GPU, 1, bench.T_PER_GPU)["workload"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] in ("port", "reference")
    cb = d["cpu_baseline"]
    assert cb["cores"] >= 1 and cb["torch_threads"] >= 1 and cb["value"] == d["value"]


def test_roofline_of_the_slower_fused_gemm():
    pk = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "source": "measured"}
    kernels = {"sffn_ffn_up": {"mean_ms": 1.40}, "sffn_ffn_dgrad": {"mean_ms": 1.50},
               "sffn_gemm_bf16": {"mean_ms": 1.20}}
    r = bench.roofline(kernels, 16384, pk, 0.9)
    flops = 2.0 * 16384 * bench.D_MODEL * bench.D_FF
    assert r["kernel"] == "sffn_ffn_dgrad" and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    # the activation gradient is only needed at the live 10% of the entries
    assert abs(r["achieved"] - 0.1 * flops / 1.5e-3 / 1e12) < 0.1
    assert abs(r["frac"] - r["achieved"] / 1400.0) < 1e-3
    assert abs(r["executed_achieved"] - flops / 1.5e-3 / 1e12) < 0.1
    # the up-projection is dense: algorithmic and executed agree
    r = bench.roofline({"sffn_ffn_up": {"mean_ms": 1.6}, "sffn_ffn_dgrad": {"mean_ms": 1.5}}, 16384, pk, 0.9)
    assert r["kernel"] == "sffn_ffn_up" and r["achieved"] == r["executed_achieved"]
    assert bench.roofline({}, 16384, pk) is None


def test_peaks_come_from_the_measured_file_when_present():
    pk = bench.peaks()
    assert pk["source"] in ("measured", "fallback") and pk["hbm_gbs"] > 0 and pk["bf16_tflops_sustained"] > 0
