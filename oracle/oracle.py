"""ctypes binding of the CPU checker (TEST INFRASTRUCTURE ONLY).

Loads liboracle.so (this project's C restatement of the reference
arithmetic, oracle/vbs_oracle.c) and, when it was built here from the
reference sources, _ref/libvbsref.so (the reference's own dequant, host
math, hot-kernel table and vbs_cpu, exported by ref_shim.c). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
module; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "liboracle.so"
REF_LIB = ORACLE_DIR / "_ref" / "libvbsref.so"
REF_CPU = ORACLE_DIR / "_ref" / "vbs-cpu"

F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K, LNS8 = 0, 1, 2, 3, 8, 12, 14, 40
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210),
         LNS8: (32, 36)}

_P = C.c_void_p
_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)


def ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def row_bytes(t, cols):
    e, b = BLOCK[t]
    return cols // e * b


_lib = None
_ref = None


def reference_dir() -> Path:
    """The reference checkout: $VBS_REFDIR when set, else a `reference`
    folder beside this repository (absent on machines that only run the
    prebuilt checker)."""
    env = os.environ.get("VBS_REFDIR")
    return Path(env) if env else ORACLE_DIR.parent.parent / "reference"


def build(ref: bool = True) -> None:
    subprocess.run(["make", "-C", str(ORACLE_DIR), "oracle"], check=True, capture_output=True)
    refdir = reference_dir()
    if ref and (refdir / "src").is_dir():
        subprocess.run(["make", "-C", str(ORACLE_DIR), "ref", f"REFDIR={refdir}"], check=True, capture_output=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build(ref=False)
        L = C.CDLL(str(LIB))
        u32, u64, i32, f32, sz = C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_size_t
        sig = {
            "orc_f16_to_f32": (f32, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [f32]),
            "orc_f32_to_f16_rne": (C.c_uint16, [f32]),
            "orc_dequant": (sz, [i32, _P, sz, _P]),
            "orc_rms_norm": (None, [_P, _P, _P, u32, f32]),
            "orc_rope": (None, [_P, u32, u32, u32, f32]),
            "orc_silu_mul": (None, [_P, _P, _P, u32]),
            "orc_add": (None, [_P, _P, _P, u32]),
            "orc_embed_row": (i32, [_P, i32, u32, _P, u32]),
            "orc_cache_store": (None, [_P, _P, _P, _P, u32, u32, u32, u32]),
            "orc_attention": (None, [_P, _P, _P, _P, u32, u32, u32, u32, u32, u32, f32]),
            "orc_linear_tile": (i32, [_P, i32, _P, _P, u32, u32, u32, u32, i32]),
            "orc_cpu_quantize_q8": (None, [_P, sz, _P, _P, _P]),
            "orc_cpu_matvec_q8_0": (None, [_P, sz, sz, _P, _P, _P]),
            "orc_cpu_matvec_f32": (None, [_P, sz, sz, _P, _P]),
            "orc_state_create": (_P, [_P, u32, i32]),
            "orc_state_destroy": (None, [_P]),
            "orc_step": (i32, [_P, u32, _P]),
            "orc_argmax": (u32, [_P, sz]),
            "orc_synth_scale": (f32, [f32]),
            "orc_synth_f32": (None, [u64, u64, u64, u64, u64, u64, f32, _P]),
            "orc_quantize_q8_0": (None, [_P, sz, _P]),
            "orc_quantize_q4_k": (None, [_P, sz, _P]),
            "orc_quantize_q6_k": (None, [_P, sz, _P]),
            "orc_synth_tensor": (i32, [i32, u64, u64, u64, u64, u64, u64, f32, _P]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(L, n)
            fn.restype, fn.argtypes = r, a
        _lib = L
    return _lib


def ref() -> C.CDLL | None:
    """The reference compiled from its own sources, or None when absent."""
    global _ref
    if _ref is None and REF_LIB.exists():
        L = C.CDLL(str(REF_LIB))
        u32, i32, f32, sz = C.c_uint32, C.c_int, C.c_float, C.c_size_t
        sig = {
            "ref_dequant_block": (i32, [i32, _P, _P]),
            "ref_f16_to_f32": (f32, [C.c_uint16]),
            "ref_f32_to_f16": (C.c_uint16, [f32]),
            "ref_rms_norm": (None, [_P, _P, _P, u32, f32]),
            "ref_rope": (None, [_P, u32, u32, u32, f32]),
            "ref_silu_mul": (None, [_P, _P, _P, u32]),
            "ref_add": (None, [_P, _P, _P, u32]),
            "ref_embed_row": (i32, [_P, i32, u32, _P, u32]),
            "ref_cache_store": (None, [_P, _P, _P, _P, u32, u32, u32, u32]),
            "ref_attention": (None, [_P, _P, _P, _P, u32, u32, u32, u32, u32, u32, f32]),
            "ref_linear_tile": (i32, [_P, i32, _P, _P, u32, u32, u32, u32, i32]),
            "ref_hot_matvec_q8_0": (None, [_P, sz, sz, _P, _P, _P]),
            "ref_hot_matvec_f32": (None, [_P, sz, sz, _P, _P]),
            # the reference CPU inference path itself (include/vbs_cpu.h:13-24)
            "vbs_cpu_open": (_P, [C.c_char_p, sz, C.c_char_p, sz]),
            "vbs_cpu_close": (None, [_P]),
            "vbs_cpu_reset": (None, [_P]),
            "vbs_cpu_step_ex": (C.c_bool, [_P, u32, C.c_bool, C.c_char_p, sz]),
            "vbs_cpu_logits": (_P, [_P]),
            "vbs_cpu_vocab_size": (sz, [_P]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(L, n)
            fn.restype, fn.argtypes = r, a
        _ref = L
    return _ref


# ---------------------------------------------------------------------------
# numpy-friendly wrappers
# ---------------------------------------------------------------------------
def dequant(t: int, blob: np.ndarray) -> np.ndarray:
    e, b = BLOCK[t]
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    nb = blob.size // b
    out = np.empty(nb * e, dtype=np.float32)
    lib().orc_dequant(t, ptr(blob), nb, ptr(out))
    return out


def linear_tile(w: np.ndarray, t: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    y = np.zeros(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rc = lib().orc_linear_tile(ptr(np.ascontiguousarray(w, dtype=np.uint8)), t, ptr(x), ptr(y), cols, rows, 0, 0, 0)
    assert rc == 0
    return y


def attention(q, kc, vc, seq_len, layer, max_ctx, nqh, nkh, hd, scale) -> np.ndarray:
    out = np.zeros(nqh * hd, dtype=np.float32)
    lib().orc_attention(ptr(np.ascontiguousarray(q, np.float32)), ptr(np.ascontiguousarray(kc, np.uint16)),
                        ptr(np.ascontiguousarray(vc, np.uint16)), ptr(out), seq_len, layer, max_ctx, nqh, nkh, hd,
                        scale)
    return out


def synth_scale(std: float) -> float:
    return float(lib().orc_synth_scale(std))


def synth_tensor(t: int, seed: int, rows: int, cols: int, scale: float, row0=0, col0=0, full_cols=None) -> np.ndarray:
    out = np.empty(rows * row_bytes(t, cols), dtype=np.uint8)
    rc = lib().orc_synth_tensor(t, seed, rows, cols, row0, col0, full_cols or cols, scale, ptr(out))
    assert rc == 0
    return out


def synth_f32(seed: int, rows: int, cols: int, scale: float, row0=0, col0=0, full_cols=None) -> np.ndarray:
    out = np.empty(rows * cols, dtype=np.float32)
    lib().orc_synth_f32(seed, rows, cols, row0, col0, full_cols or cols, scale, ptr(out))
    return out


class RefCpu:
    """The reference's own CPU inference (vbs_cpu_open / vbs_cpu_step_ex,
    src/vbs_cpu.c:572-639), loaded from a GGUF file: K-quant weights are
    requantized to Q8_0 at load (src/vbs_cpu.c:312-346), one host thread.
    Needs oracle/_ref/libvbsref.so (the reference compiled from its
    sources)."""

    def __init__(self, path, context: int):
        R = ref()
        if R is None:
            raise FileNotFoundError(f"{REF_LIB} is not built")
        self.R = R
        err = C.create_string_buffer(512)
        self.h = R.vbs_cpu_open(str(path).encode(), context, err, 512)
        if not self.h:
            raise RuntimeError(f"vbs_cpu_open: {err.value.decode()}")
        self.vocab = int(R.vbs_cpu_vocab_size(self.h))
        self._err = err

    def step(self, token: int, logits: bool = True) -> None:
        if not self.R.vbs_cpu_step_ex(self.h, token, logits, self._err, 512):
            raise RuntimeError(f"vbs_cpu_step_ex: {self._err.value.decode()}")

    def logits(self) -> np.ndarray:
        p = self.R.vbs_cpu_logits(self.h)
        return np.ctypeslib.as_array(C.cast(p, _f32p), shape=(self.vocab,)).copy()

    def argmax(self) -> int:
        """First maximum, as src/vbs_cpu_main.c:78-80."""
        return int(np.argmax(self.logits()))

    def close(self) -> None:
        if self.h:
            self.R.vbs_cpu_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# whole-model oracle
# ---------------------------------------------------------------------------
class OrcModel(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("dim", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("vocab", C.c_uint32), ("eps", C.c_float),
        ("theta", C.c_float), ("embd_type", C.c_int), ("out_type", C.c_int), ("embd", _P), ("out", _P),
        ("out_norm", _P), ("attn_norm", C.POINTER(_P)), ("ffn_norm", C.POINTER(_P)), ("wq", C.POINTER(_P)),
        ("wk", C.POINTER(_P)), ("wv", C.POINTER(_P)), ("wo", C.POINTER(_P)), ("wgate", C.POINTER(_P)),
        ("wup", C.POINTER(_P)), ("wdown", C.POINTER(_P)), ("tq", C.POINTER(C.c_int)), ("tk", C.POINTER(C.c_int)),
        ("tv", C.POINTER(C.c_int)), ("to", C.POINTER(C.c_int)), ("tgate", C.POINTER(C.c_int)),
        ("tup", C.POINTER(C.c_int)), ("tdown", C.POINTER(C.c_int)),
    ]


class HostModel:
    """A llama model in host memory: tensors {name: (type, rows, cols, np.uint8 / np.float32 array)}."""

    def __init__(self, cfg: dict, tensors: dict):
        self.cfg = cfg
        self.t = tensors
        n = cfg["n_layers"]
        P, I = _P * n, C.c_int * n
        g = lambda key: P(*[self.t[f"blk.{l}.{key}"][3].ctypes.data for l in range(n)])
        ty = lambda key: I(*[self.t[f"blk.{l}.{key}"][0] for l in range(n)])
        self._arrs = dict(attn_norm=g("attn_norm"), ffn_norm=g("ffn_norm"), wq=g("attn_q"), wk=g("attn_k"),
                          wv=g("attn_v"), wo=g("attn_output"), wgate=g("ffn_gate"), wup=g("ffn_up"),
                          wdown=g("ffn_down"), tq=ty("attn_q"), tk=ty("attn_k"), tv=ty("attn_v"),
                          to=ty("attn_output"), tgate=ty("ffn_gate"), tup=ty("ffn_up"), tdown=ty("ffn_down"))
        m = OrcModel()
        m.n_layers, m.dim, m.n_heads, m.n_kv_heads = n, cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"]
        m.head_dim, m.ffn, m.vocab = cfg["dim"] // cfg["n_heads"], cfg["ffn"], cfg["vocab"]
        m.eps, m.theta = cfg["eps"], cfg["theta"]
        m.embd_type, m.out_type = self.t["token_embd"][0], self.t["output"][0]
        m.embd, m.out = self.t["token_embd"][3].ctypes.data, self.t["output"][3].ctypes.data
        m.out_norm = self.t["output_norm"][3].ctypes.data
        for k, v in self._arrs.items():
            setattr(m, k, C.cast(v, C.POINTER(_P) if not k.startswith("t") else C.POINTER(C.c_int)))
        self.m = m


class OrcState:
    """orc_state_t: mode 0 = vbs_cpu arithmetic, mode 1 = engine / host_math."""

    def __init__(self, model: HostModel, context: int, mode: int):
        self.model = model
        self.vocab = model.cfg["vocab"]
        self.h = lib().orc_state_create(C.byref(model.m), context, mode)
        if not self.h:
            raise MemoryError("orc_state_create failed")

    def step(self, token: int, logits: bool = True):
        out = np.empty(self.vocab, dtype=np.float32) if logits else None
        rc = lib().orc_step(self.h, token, ptr(out) if logits else None)
        if rc:
            raise RuntimeError("orc_step failed")
        return out

    def generate(self, prompt, n_new):
        """Greedy like vbs-cpu (src/vbs_cpu_main.c:70-86): logits of the last
        prompt token, then n_new tokens, the last one not fed back."""
        for i, t in enumerate(prompt):
            lg = self.step(t, logits=(i + 1 == len(prompt)))
        out = []
        for i in range(n_new):
            best = int(lib().orc_argmax(ptr(lg), self.vocab))
            out.append(best)
            if i + 1 < n_new:
                lg = self.step(best)
        return out

    def __del__(self):
        try:
            lib().orc_state_destroy(self.h)
        except Exception:
            pass


def load_gguf_host(path) -> HostModel:
    """Read a llama GGUF into host arrays (norms as float32)."""
    import struct
    data = Path(path).read_bytes()
    o = 0

    def rd(fmt):
        nonlocal o
        v = struct.unpack_from(fmt, data, o)
        o += struct.calcsize(fmt)
        return v

    def rs():
        (n,) = rd("<Q")
        nonlocal o
        v = data[o:o + n].decode()
        o += n
        return v

    _, _, nt, nkv = rd("<4sIQQ")
    meta = {}
    scal = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
    for _ in range(nkv):
        k = rs()
        (ty,) = rd("<I")
        meta[k] = rs() if ty == 8 else rd(scal[ty])[0]
    infos = []
    for _ in range(nt):
        name = rs()
        (nd,) = rd("<I")
        dims = rd("<" + "Q" * nd)
        ty, rel = rd("<IQ")
        infos.append((name, ty, dims, rel))
    align = int(meta.get("general.alignment", 32))
    start = (o + align - 1) // align * align
    t = {}
    for name, ty, dims, rel in infos:
        cols = dims[0]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        nbytes = row_bytes(ty, cols) * rows
        raw = np.frombuffer(data, dtype=np.uint8, count=nbytes, offset=start + rel).copy()
        key = name[:-len(".weight")] if name.endswith(".weight") else name
        arr = raw.view(np.float32).copy() if key.endswith("norm") else raw
        t[key] = (ty, rows, cols, arr)
    if "output" not in t:
        t["output"] = t["token_embd"]
    a = "llama."
    cfg = dict(n_layers=int(meta[a + "block_count"]), dim=int(meta[a + "embedding_length"]),
               n_heads=int(meta[a + "attention.head_count"]),
               n_kv_heads=int(meta.get(a + "attention.head_count_kv", meta[a + "attention.head_count"])),
               ffn=int(meta[a + "feed_forward_length"]), vocab=int(t["token_embd"][1]),
               eps=float(meta.get(a + "attention.layer_norm_rms_epsilon", 1e-5)),
               theta=float(meta.get(a + "rope.freq_base", 10000.0)))
    return HostModel(cfg, t)
