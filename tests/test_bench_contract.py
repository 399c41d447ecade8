"""bench.py's reference arm (the reference's CPU decode kernel on the host
cores) keeps the JSON contract the driver reads: one line with the same
metric, unit and direction as the GPU arm, impl "reference", a cpu_baseline
describing the run and an e2e with no host-device bytes. Runs on CPU in a
few seconds."""
import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_json_line():
    # one layer of the 8B shape keeps the GGUF small; the line is the same
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1",
                          "--ref-layers", "1"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "decode tokens/s, Llama-3-8B Q4_K shape" and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and abs(d["ms_per_step"] - 1000.0 / d["value"]) <= 0.01 * d["ms_per_step"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    if cb["kind"] == "reference":   # the reference's vbs_cpu path after a short prompt, one thread
        assert cb["cores"] == 1 and d["config"]["ctx"] > 0 and "vbs_cpu_step_ex" in d["config"]["workload"]
        assert d["config"]["tiny_e2e"]["tokens_match_golden"] is True
    else:
        assert d["config"]["ctx"] == 4096
