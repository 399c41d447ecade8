"""Generate the golden fixtures under tests/golden/ from the REFERENCE itself.

Run here, where the reference sources exist, after `make -C oracle all`
has compiled them (unmodified) into oracle/_ref/. The GPU box has no
reference tree: the tests read only the committed outputs of this script.

  golden.npz        inputs and the reference's outputs:
                    * vbs_dequant_block on seeded random blocks of every
                      supported type (src/vbs_dequant.c:339-356)
                    * vbs_host_* ops (src/vbs_host_math.h): rms_norm, rope,
                      silu_mul, cache_store, attention, linear_tile
                    * the hot-kernel table's matvec_q8_0 / matvec_f32
                      (src/hotkernels/vbs_hot_ref_impl.h:49-118)
                    * sha256 of vbs_f16_to_f32 over all 65536 halves and of
                      vbs_f32_to_f16 over edge-case floats
  tiny_greedy.json  the tiny model's sha256, prompt, the 64 greedy tokens
                    and final logits of `vbs-cpu` (src/vbs_cpu_main.c)

Inputs come from numpy's PCG64 with fixed seeds and are stored in the
fixture, so the tests never depend on a random stream.
"""
from __future__ import annotations

import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import models  # noqa: E402
import oracle as orc  # noqa: E402

C = __import__("ctypes")


def finite_blocks(t: int, nb: int, rng) -> np.ndarray:
    """nb random blocks of type t whose fp16 scale fields are finite (the
    exponent's top bit cleared keeps |scale| <= 2)."""
    e, b = orc.BLOCK[t]
    raw = rng.integers(0, 256, size=nb * b, dtype=np.uint8).reshape(nb, b)
    fields = {orc.Q4_0: [0], orc.Q4_1: [0, 2], orc.Q8_0: [0], orc.Q4_K: [0, 2], orc.Q6_K: [208],
              orc.F16: list(range(0, b, 2))}[t]
    for off in fields:
        raw[:, off + 1] &= 0xBF
    return raw.reshape(-1)


def main() -> None:
    R = orc.ref()
    if R is None:
        sys.exit("oracle/_ref/libvbsref.so is missing: run `make -C oracle all` where the reference exists")
    rng = np.random.default_rng(20261201)
    g: dict[str, np.ndarray] = {}

    # ---- dequant ----
    for t in (orc.Q4_0, orc.Q4_1, orc.Q8_0, orc.Q4_K, orc.Q6_K, orc.F16):
        e, b = orc.BLOCK[t]
        nb = 96 if e > 1 else 4096
        blob = finite_blocks(t, nb, rng)
        out = np.empty(nb * e, dtype=np.float32)
        if t == orc.F16:
            for i in range(nb):
                out[i] = R.ref_f16_to_f32(int(blob[2 * i]) | (int(blob[2 * i + 1]) << 8))
        else:
            for i in range(nb):
                n = R.ref_dequant_block(t, orc.ptr(blob[i * b:(i + 1) * b]), orc.ptr(out[i * e:(i + 1) * e]))
                assert n == e
        g[f"dq_in_{t}"] = blob
        g[f"dq_out_{t}"] = out

    # ---- half conversions ----
    allh = np.array([R.ref_f16_to_f32(h) for h in range(65536)], dtype=np.float32)
    g["f16_to_f32_sha"] = np.frombuffer(hashlib.sha256(allh.view(np.uint32).tobytes()).digest(), dtype=np.uint8)
    edge = np.concatenate([
        rng.standard_normal(2048).astype(np.float32),
        (rng.standard_normal(1024) * 1e-5).astype(np.float32),      # subnormal halves
        (rng.standard_normal(512) * 7e4).astype(np.float32),        # overflow
        np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65520.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                  2.9802326e-08], dtype=np.float32)])
    g["f32_to_f16_in"] = edge
    g["f32_to_f16_out"] = np.array([R.ref_f32_to_f16(float(v)) for v in edge], dtype=np.uint16)

    # ---- host_math ops ----
    x = (rng.standard_normal(384) * 2).astype(np.float32)
    w = rng.standard_normal(384).astype(np.float32)
    y = np.empty(384, np.float32)
    R.ref_rms_norm(orc.ptr(x), orc.ptr(w), orc.ptr(y), 384, C.c_float(1e-5))
    g["rms_x"], g["rms_w"], g["rms_y"] = x, w, y
    for th in (10000.0, 500000.0):
        v = rng.standard_normal(4 * 64).astype(np.float32)
        o = v.copy()
        R.ref_rope(orc.ptr(o), 7, 64, 4, C.c_float(th))
        g[f"rope_in_{int(th)}"], g[f"rope_out_{int(th)}"] = v, o
    gg = (rng.standard_normal(777) * 3).astype(np.float32)
    uu = rng.standard_normal(777).astype(np.float32)
    so = np.empty(777, np.float32)
    R.ref_silu_mul(orc.ptr(gg), orc.ptr(uu), orc.ptr(so), 777)
    g["silu_g"], g["silu_u"], g["silu_out"] = gg, uu, so
    # attention: the reference self-test case and a Llama-3 head layout
    for tag, (nqh, nkh, hd, seq, layer, mc) in {"small": (4, 2, 32, 6, 1, 16), "l3": (32, 8, 128, 24, 0, 24)}.items():
        kc = np.zeros((layer + 1) * mc * nkh * hd, np.uint16)
        vc = np.zeros_like(kc)
        for p in range(seq):
            k = rng.standard_normal(nkh * hd).astype(np.float32)
            v = rng.standard_normal(nkh * hd).astype(np.float32)
            R.ref_cache_store(orc.ptr(k), orc.ptr(v), orc.ptr(kc), orc.ptr(vc), p, layer, mc, nkh * hd)
        q = rng.standard_normal(nqh * hd).astype(np.float32)
        out = np.empty(nqh * hd, np.float32)
        R.ref_attention(orc.ptr(q), orc.ptr(kc), orc.ptr(vc), orc.ptr(out), seq, layer, mc, nqh, nkh, hd,
                        C.c_float(1.0 / np.sqrt(np.float32(hd))))
        g[f"attn_{tag}_q"], g[f"attn_{tag}_kc"], g[f"attn_{tag}_vc"], g[f"attn_{tag}_out"] = q, kc, vc, out
        g[f"attn_{tag}_dims"] = np.array([nqh, nkh, hd, seq, layer, mc], np.int64)
    # linear tiles: synthesized weights of every type
    sc = orc.synth_scale(0.02)
    for t in (orc.F32, orc.F16, orc.Q4_0, orc.Q4_1, orc.Q8_0, orc.Q4_K, orc.Q6_K):
        rows, cols = 24, 512
        if t in (orc.Q4_0, orc.Q4_1):
            wb = finite_blocks(t, rows * cols // 32, rng)
        else:
            wb = orc.synth_tensor(t, 99 + t, rows, cols, sc)
        xx = rng.standard_normal(cols).astype(np.float32)
        yy = np.empty(rows, np.float32)
        assert R.ref_linear_tile(orc.ptr(wb), t, orc.ptr(xx), orc.ptr(yy), cols, rows, 0, 0, 0) == 0
        g[f"lin_w_{t}"], g[f"lin_x_{t}"], g[f"lin_y_{t}"] = wb, xx, yy
    # hot-kernel table
    rows, cols = 20, 256
    wq8 = orc.synth_tensor(orc.Q8_0, 5, rows, cols, sc)
    xq = rng.integers(-127, 128, size=cols, dtype=np.int8)
    qd = (rng.random(cols // 32) * 0.05).astype(np.float32)
    yq = np.empty(rows, np.float32)
    R.ref_hot_matvec_q8_0(orc.ptr(wq8), rows, cols, orc.ptr(xq), orc.ptr(qd), orc.ptr(yq))
    g["hot_w"], g["hot_xq"], g["hot_qd"], g["hot_y"] = wq8, xq, qd, yq
    wf = rng.standard_normal(rows * 688).astype(np.float32)
    xf = rng.standard_normal(688).astype(np.float32)
    yf = np.empty(rows, np.float32)
    R.ref_hot_matvec_f32(orc.ptr(wf), rows, 688, orc.ptr(xf), orc.ptr(yf))
    g["hotf_w"], g["hotf_x"], g["hotf_y"] = wf, xf, yf
    np.savez_compressed(HERE / "golden.npz", **g)

    # ---- tiny model greedy tokens from the reference CPU CLI ----
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "tiny.gguf"
        models.make_tiny_gguf(path)
        sha = hashlib.sha256(path.read_bytes()).hexdigest()
        prompt = models.tiny_prompt()
        r = subprocess.run([str(orc.REF_CPU), "--model", str(path), "--context", "128", "--max-new", str(models.N_NEW),
                            "--dump-logits"], input=" ".join(map(str, prompt)) + "\n", capture_output=True, text=True,
                           check=True)
        res = json.loads(r.stdout)
    # The final logits are those after the last step vbs-cpu ran (the 63rd
    # generated token fed back; the 64th is not fed).
    (HERE / "tiny_greedy.json").write_text(json.dumps(
        {"gguf_sha256": sha, "prompt": prompt, "generated": res["generated"], "final_logits": res["logits"],
         "command": "vbs-cpu --model tiny.gguf --context 128 --max-new 64 --dump-logits (prompt ids on stdin)"},
        indent=None) + "\n")
    print("wrote", HERE / "golden.npz", HERE / "tiny_greedy.json")


if __name__ == "__main__":
    main()
