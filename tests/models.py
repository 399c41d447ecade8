"""Model definitions shared by the fixture generator, the tests and bench.py.

TINY is BASELINE config 0: a llama-style GGUF runnable on the reference's
CPU path (4 layers, dim 256, 8/2 heads, FFN 688, vocab 512, eps 1e-5,
RoPE theta 1e4). Weights are N(0, 0.02) from the seeded synthesizer,
quantized to Q8_0, except ffn_down, which is stored F32: 688 columns are
not whole 32-element blocks and the reference loader rejects such a Q8_0
tensor (src/vbs_gguf.c:189-195). Norm weights are 1.0, as in the
reference's own tiny-model tool (tools/make_tiny_gguf.py:101-103).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import vbs_b200 as vbs  # noqa: E402
import oracle as orc  # noqa: E402

TINY = dict(n_layers=4, dim=256, n_heads=8, n_kv_heads=2, ffn=688, vocab=512, eps=1e-5, theta=10000.0)
TINY_TYPES = dict(token_embd=orc.Q8_0, output=orc.Q8_0, attn_q=orc.Q8_0, attn_k=orc.Q8_0, attn_v=orc.Q8_0,
                  attn_output=orc.Q8_0, ffn_gate=orc.Q8_0, ffn_up=orc.Q8_0, ffn_down=orc.F32)
TINY_SEED = 1234
PROMPT_SEED = 7
N_PROMPT, N_NEW = 16, 64

# Llama-3-8B shape and its quantization mix.
L8B = dict(n_layers=32, dim=4096, n_heads=32, n_kv_heads=8, ffn=14336, vocab=128256, eps=1e-5, theta=500000.0)
L8B_TYPES = dict(token_embd=orc.Q6_K, output=orc.Q6_K, attn_q=orc.Q4_K, attn_k=orc.Q4_K, attn_v=orc.Q4_K,
                 attn_output=orc.Q4_K, ffn_gate=orc.Q4_K, ffn_up=orc.Q4_K, ffn_down=orc.Q6_K)
# Llama-3-70B shape, all Q4_K.
L70B = dict(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, ffn=28672, vocab=128256, eps=1e-5, theta=500000.0)
L70B_TYPES = {k: orc.Q4_K for k in L8B_TYPES}


def splitmix_ints(seed: int, n: int, modulo: int) -> list[int]:
    """n integers in [0, modulo) from splitmix64 (prompt token ids)."""
    out, z = [], seed & 0xFFFFFFFFFFFFFFFF
    for _ in range(n):
        z = (z + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        x = z
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 31
        out.append(x % modulo)
    return out


def tiny_prompt() -> list[int]:
    return splitmix_ints(PROMPT_SEED, N_PROMPT, TINY["vocab"])


def shape_of(cfg: dict) -> "vbs.LlamaShape":
    return vbs.LlamaShape(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["ffn"], cfg["vocab"],
                          cfg["eps"], cfg["theta"])


def host_tensors(cfg: dict, types: dict, seed: int, std: float = 0.02) -> dict:
    """All tensors of a seeded model, synthesized by the host oracle:
    {name: (type, rows, cols, array)} with the same bytes the device
    synthesizer produces for the same seed."""
    shape = shape_of(cfg)
    scale = orc.synth_scale(std)
    t = {}

    def add(name, base):
        rows, cols, _, _, _ = vbs.shard_spec(name, shape, 0, 1)
        ty = types[base]
        t[name] = (ty, rows, cols, orc.synth_tensor(ty, vbs.tensor_seed(seed, name), rows, cols, scale))

    add("token_embd", "token_embd")
    add("output", "output")
    t["output_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
    for l in range(cfg["n_layers"]):
        for base in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            add(f"blk.{l}.{base}", base)
        t[f"blk.{l}.attn_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
        t[f"blk.{l}.ffn_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
    return t


def host_tensors_parallel(cfg: dict, types: dict, seed: int, std: float = 0.02, threads: int = 0) -> dict:
    """host_tensors() with the tensors synthesized on a thread pool (the C
    synthesizer releases the GIL), for full-size models."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    shape = shape_of(cfg)
    scale = orc.synth_scale(std)
    jobs = [("token_embd", "token_embd"), ("output", "output")]
    for l in range(cfg["n_layers"]):
        jobs += [(f"blk.{l}.{b}", b) for b in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up",
                                               "ffn_down")]

    def one(job):
        name, base = job
        rows, cols, _, _, _ = vbs.shard_spec(name, shape, 0, 1)
        ty = types[base]
        return name, (ty, rows, cols, orc.synth_tensor(ty, vbs.tensor_seed(seed, name), rows, cols, scale))

    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as ex:
        t = dict(ex.map(one, jobs))
    t["output_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
    for l in range(cfg["n_layers"]):
        t[f"blk.{l}.attn_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
        t[f"blk.{l}.ffn_norm"] = (orc.F32, 1, cfg["dim"], np.ones(cfg["dim"], dtype=np.float32))
    return t


def write_model_gguf(path, cfg: dict, tensors: dict, context_length: int = 2048) -> None:
    meta = {"general.architecture": "llama", "general.alignment": 32, "llama.block_count": cfg["n_layers"],
            "llama.context_length": context_length, "llama.embedding_length": cfg["dim"],
            "llama.feed_forward_length": cfg["ffn"], "llama.attention.head_count": cfg["n_heads"],
            "llama.attention.head_count_kv": cfg["n_kv_heads"], "llama.rope.freq_base": float(cfg["theta"]),
            "llama.attention.layer_norm_rms_epsilon": float(cfg["eps"]), "llama.vocab_size": cfg["vocab"]}
    order = ["token_embd", "output_norm", "output"]
    for l in range(cfg["n_layers"]):
        order += [f"blk.{l}.{b}" for b in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm",
                                            "ffn_gate", "ffn_up", "ffn_down")]
    tl = []
    for name in order:
        ty, rows, cols, arr = tensors[name]
        dims = [cols] if name.endswith("norm") else [cols, rows]
        tl.append((name + ".weight", ty, dims, np.ascontiguousarray(arr).view(np.uint8)))
    vbs.write_gguf(path, meta, tl)


def make_tiny_gguf(path) -> None:
    write_model_gguf(path, TINY, host_tensors(TINY, TINY_TYPES, TINY_SEED))


def host_model_from_device(cfg: dict, dm) -> "orc.HostModel":
    """The oracle's host copy of a device model (vbs.DeviceModel): every
    tensor copied back, matrices cut to their packed size."""
    host = {}
    for name, t in dm.tensors.items():
        arr = t.cpu().numpy()
        if name.endswith("norm"):
            host[name] = (orc.F32, 1, cfg["dim"], arr)
        else:
            base = name.split(".")[-1]
            rows, cols, *_ = vbs.shard_spec(name, dm.shape, 0, 1)
            host[name] = (dm.types[base], rows, cols, arr[:rows * orc.row_bytes(dm.types[base], cols)])
    return orc.HostModel(cfg, host)

