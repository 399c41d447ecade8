"""The step kernel's plan (`step_plan` in csrc/step.cu), on the host.

Which models the persistent step kernel takes, how it cuts each op's
matrix into ring stages, and where its shared-memory regions lie. The plan
is compiled from the library's own source into a small harness
(tests/step_plan_harness.cu, PTX only: no GPU, no ptxas). The reference has
no such kernel; its decode step is forward_token, one backend call per op
(src/vbs_specializer.c:270-349).
"""
import json
import shutil
import subprocess
from pathlib import Path

import pytest

import models

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "verum-bespoke-singularity_b200"
N_SM = 148
SMEM = 227 * 1024                 # dynamic shared memory of the kernel
HDR = 3072 + 2 * 8 * 8 * 16 * 4   # barriers, flags, parameters, row-sum batches
Q4_K, Q6_K, Q8_0, F16 = 12, 14, 8, 1
QKV, O, GU, DOWN, OUT = range(5)

W6144 = dict(n_layers=2, dim=6144, n_heads=48, n_kv_heads=8, ffn=16384, vocab=4096)
ALL_Q4 = {k: Q4_K for k in models.L8B_TYPES}


@pytest.fixture(scope="module")
def plan(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc is not available")
    exe = tmp_path_factory.mktemp("plan") / "step_plan"
    subprocess.run([nvcc, "-std=c++17", "-O0", "-gencode", "arch=compute_100a,code=compute_100a",
                    "--expt-relaxed-constexpr", "-I", str(PKG / "csrc"), "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "step_plan_harness.cu"), str(PKG / "csrc" / "step.cu"), "-o", str(exe)],
                   check=True, capture_output=True, timeout=900)

    def run(*shapes):
        text = "".join(" ".join(str(int(v)) for v in s) + "\n" for s in shapes)
        out = subprocess.run([str(exe)], input=text, capture_output=True, text=True, check=True, timeout=60).stdout
        return [json.loads(line) for line in out.splitlines()]
    return run


def shape(cfg, types, tp=0, hd=None):
    hd = hd or cfg["dim"] // cfg["n_heads"]
    return (cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], hd, cfg["ffn"], cfg["vocab"],
            types["token_embd"], types["attn_q"], types["attn_output"], types["ffn_gate"], types["ffn_down"],
            types["output"], tp, N_SM)


def check_layout(cfg, p):
    """Every region in its place, every stage fits the ring, every op's
    chunks cover its columns."""
    dim, ffn = cfg["dim"], cfg["ffn"]
    hd = dim // cfg["n_heads"]
    qd, G = cfg["n_heads"] * hd, cfg["n_heads"] // cfg["n_kv_heads"]
    geo = p["geo"]
    nb = max(dim, qd, min(ffn, 2 * geo[DOWN][0])) // 32          # x blocks quantized at once
    assert p["x_off"] >= HDR and p["x_off"] + 4 * dim <= p["xq_off"]
    assert p["xq_off"] % 1024 == 0 and p["ring_off"] % 1024 == 0
    assert p["xf_off"] == p["xq_off"] + nb * 80
    attn = 8 * G * (4 + hd) * 4 + 16 * (2 * hd + 16) + 4 * hd    # attention states alias the x buffers
    assert p["xq_off"] + max(nb * 96, attn) <= p["ring_off"]
    assert p["ring_off"] + p["ring_bytes"] <= SMEM
    assert p["ring_bytes"] >= 2 * p["stage_max"] >= 2 * 4 * dim  # the norm weight is a stage too
    cols = [dim, qd, dim, ffn, dim]
    for k, (ck, rs, nch, ntiles) in enumerate(geo):
        assert 0 < ck <= 4096 and ck % 32 == 0
        assert nch == -(-cols[k] // ck), k
        assert rs % 16 == 0 and 16 * rs <= p["stage_max"]
    rows = [qd + 2 * cfg["n_kv_heads"] * hd, dim, ffn, dim, cfg["vocab"]]
    assert geo[GU][3] == -(-ffn // 8)                            # 8 gate + 8 up rows per tile
    for k in (QKV, O, DOWN, OUT):
        assert geo[k][3] == -(-rows[k] // 16)
    # down units are chunk-major; every CTA's share lies within two chunks
    assert -(-geo[DOWN][3] * geo[DOWN][2] // N_SM) <= geo[DOWN][3]
    assert p["attn_splits"] * cfg["n_kv_heads"] <= N_SM
    assert p["acc_layer"] == rows[QKV] + dim + ffn + geo[DOWN][2] * dim


def test_8b_mix_has_whole_rows(plan):
    """The benchmarked shape: every op but the down projection in one stage
    per row tile (the kernel instance without the wide code)."""
    cfg = dict(models.L8B)
    (p,) = plan(shape(cfg, models.L8B_TYPES))
    assert p["ok"] == 1, p["why"]
    assert [g[2] for g in p["geo"]] == [1, 1, 1, 4, 1]
    assert p["attn_splits"] == 18
    check_layout(cfg, p)


@pytest.mark.parametrize("name", ["70b", "w6144"])
def test_wide_models_stream_row_chunks(plan, name):
    """Above 4096 columns: two row chunks per tile for Q/K/V, O, gate/up and
    the output (the wide instances accumulate them), the down projection in
    4096-column planes (7 for the 70B shape's 28672)."""
    cfg = dict(models.L70B) if name == "70b" else dict(W6144)
    (p,) = plan(shape(cfg, ALL_Q4))
    assert p["ok"] == 1, p["why"]
    down = 7 if name == "70b" else 4
    assert [g[2] for g in p["geo"]] == [2, 2, 2, down, 2]
    assert all(g[0] == 4096 for g in p["geo"])
    check_layout(cfg, p)


def test_tensor_parallel_keeps_whole_rows(plan):
    """Under tensor parallelism the exchange addresses one plane per rank:
    the 8B shard is taken, a 70B shard (8192 columns) is declined and runs
    the per-op kernels."""
    p8, p70 = plan(shape(dict(models.L8B, n_heads=16, n_kv_heads=4, ffn=7168), models.L8B_TYPES, tp=1, hd=128),
                   shape(dict(models.L70B, n_heads=32, n_kv_heads=4, ffn=14336), ALL_Q4, tp=1, hd=128))
    assert p8["ok"] == 1, p8["why"]
    assert p70["ok"] == 0 and "4096" in p70["why"]


@pytest.mark.parametrize("change, why", [
    (dict(dim=20480, n_heads=160, n_kv_heads=20), "16384"),
    (dict(n_kv_heads=2), "query heads per KV head"),
    (dict(dim=3072, n_heads=32), "head_dim"),
])
def test_declined_shapes(plan, change, why):
    cfg = dict(models.L8B, **change)
    (p,) = plan(shape(cfg, ALL_Q4))
    assert p["ok"] == 0 and why in p["why"], p["why"]


def test_declined_weight_type(plan):
    (p,) = plan(shape(dict(models.L8B), dict(ALL_Q4, ffn_down=F16)))
    assert p["ok"] == 0 and "Q4_K, Q6_K or Q8_0" in p["why"]


def test_q8_0_and_head_dim_64(plan):
    cfg = dict(n_layers=2, dim=1024, n_heads=16, n_kv_heads=4, ffn=2816, vocab=2048)
    (p,) = plan(shape(cfg, {k: Q8_0 for k in models.L8B_TYPES}))
    assert p["ok"] == 1, p["why"]
    check_layout(cfg, p)
