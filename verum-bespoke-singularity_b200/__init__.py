"""Python host binding of libvbs_b200.so (the sm_100a decode backend).

The C ABI is include/vbs_b200.h. This module mirrors it with ctypes so the
tests and the benchmark drive the library exactly as the reference engine
would: through the `g_vbs_cuda_backend` ops table (the reference's
vbs_backend_ops_t, include/vbs_backend.h:64-99 of the reference) and through
the vbs_cu_* extension entry points. PyTorch is used only to own device
memory and streams; no tensor math runs in PyTorch.

There is no CPU fallback: `lib()` raises when the shared library is missing
or cannot be loaded, and every entry point that fails raises VbsError with
the backend's latched message.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libvbs_b200.so"

# GGML type ids (include/vbs_gguf.h:13-48 of the reference)
F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K, Q8_K, LNS8 = 0, 1, 2, 3, 8, 12, 14, 15, 40
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K",
              LNS8: "LNS8"}
# LNS8: the reference's log-scaled type, 32 x u8 log2 values + an f32 scale (value = 2^q * scale)
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210),
         LNS8: (32, 36)}

# op kinds (include/vbs_graph.h:12-24 of the reference)
(OP_EMBEDDING, OP_LINEAR, OP_NORMALIZE, OP_ATTENTION, OP_ROTARY, OP_ACTIVATION, OP_ELEMENTWISE,
 OP_STATE_SPACE, OP_CONVOLUTION, OP_CACHE, OP_PROJECTION) = range(11)
ARG_BUFFER, ARG_SCALAR = 0, 1

MV_ACCUMULATE, MV_PORTABLE = 1, 2
DEC_STRICT, DEC_NO_GRAPH, DEC_NO_PDL, DEC_NO_PERSIST = 1, 2, 4, 8
DEC_TP_NCCL = 16   # tensor parallelism: NCCL all-reduce for the per-layer sums (the reference collective)
DEC_WORDS = 32     # one GPU: the step kernel's tensor-parallel instance over a local word area (for testing it)
DEC_STREAM = 64    # slice streaming: per-layer matrices in pinned host memory, copied in per layer (two device slots)


class VbsError(RuntimeError):
    """A backend call failed; the message is the backend's latched error."""


def row_bytes(type_id: int, cols: int) -> int:
    e, b = BLOCK[type_id]
    if cols % e:
        raise ValueError(f"{cols} columns are not whole {e}-element blocks")
    return cols // e * b


# ---------------------------------------------------------------------------
# ctypes mirror of the reference ops-table types
# ---------------------------------------------------------------------------
class Device(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("type", C.c_int), ("max_working_set_bytes", C.c_uint64),
                ("max_buffer_bytes", C.c_uint64), ("internal_handle", C.c_void_p)]


class Buffer(C.Structure):
    _fields_ = [("internal_handle", C.c_void_p), ("host_ptr", C.c_void_p), ("size", C.c_size_t),
                ("device", C.POINTER(Device))]


class Arg(C.Structure):
    _fields_ = [("tag", C.c_int), ("value", C.c_void_p), ("size", C.c_size_t)]


class PrimPipeline(C.Structure):
    _fields_ = [("native", C.c_void_p), ("kind", C.c_int)]


_P_DEV = C.POINTER(Device)
_P_BUF = C.POINTER(Buffer)


class OpsTable(C.Structure):
    _fields_ = [
        ("init", C.CFUNCTYPE(C.c_bool)),
        ("get_device_count", C.CFUNCTYPE(C.c_size_t)),
        ("get_device", C.CFUNCTYPE(_P_DEV, C.c_size_t)),
        ("alloc_buffer", C.CFUNCTYPE(_P_BUF, _P_DEV, C.c_size_t, C.c_bool)),
        ("free_buffer", C.CFUNCTYPE(None, _P_BUF)),
        ("copy_to_device", C.CFUNCTYPE(C.c_bool, _P_BUF, C.c_void_p, C.c_size_t)),
        ("copy_to_host", C.CFUNCTYPE(C.c_bool, C.c_void_p, _P_BUF, C.c_size_t)),
        ("compile_linear_pipeline", C.CFUNCTYPE(C.c_void_p, _P_DEV, C.c_int, C.c_char_p, C.c_size_t)),
        ("compile_embed_pipeline", C.CFUNCTYPE(C.c_void_p, _P_DEV, C.c_int, C.c_char_p, C.c_size_t)),
        ("compile_primitive_pipeline", C.CFUNCTYPE(C.c_void_p, _P_DEV, C.c_int, C.c_char_p, C.c_size_t)),
        ("dispatch_linear_tile", C.CFUNCTYPE(C.c_bool, _P_DEV, C.c_void_p, _P_BUF, _P_BUF, C.c_size_t, _P_BUF, _P_BUF,
                                             C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_bool)),
        ("dispatch_primitive", C.CFUNCTYPE(C.c_bool, _P_DEV, C.c_void_p, C.POINTER(Arg), C.c_size_t, C.c_size_t,
                                           C.c_size_t)),
        ("synchronize_device", C.CFUNCTYPE(None, _P_DEV)),
        ("launch_persistent_kernel", C.CFUNCTYPE(C.c_bool, _P_DEV, C.c_void_p, _P_BUF)),
    ]


# PGAE states and the control block (include/vbs_engine.h:22-40 of the reference)
PGAE_IDLE, PGAE_PREFILL, PGAE_GENERATE, PGAE_EXIT = 0, 1, 2, 3
PGAE_EOS_NONE = 0xFFFFFFFF


class GpuControl(C.Structure):
    """vbs_gpu_control_t: the device-resident state of a generation run."""
    _fields_ = [("state", C.c_uint32), ("current_token", C.c_uint32), ("position", C.c_uint32),
                ("max_tokens", C.c_uint32), ("vocab_size", C.c_uint32), ("eos_token_id", C.c_uint32),
                ("generated_tokens_dev", C.c_uint64), ("logits_dev", C.c_uint64)]


class ModelDesc(C.Structure):
    """vbs_cu_model_t (include/vbs_b200.h)."""
    _fields_ = [
        ("n_layers", C.c_uint32), ("dim", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("vocab", C.c_uint32),
        ("eps", C.c_float), ("theta", C.c_float),
        ("embd_type", C.c_int), ("out_type", C.c_int),
        ("embd", C.c_void_p), ("out", C.c_void_p), ("out_norm", C.c_void_p),
        ("attn_norm", C.POINTER(C.c_void_p)), ("ffn_norm", C.POINTER(C.c_void_p)),
        ("wq", C.POINTER(C.c_void_p)), ("wk", C.POINTER(C.c_void_p)), ("wv", C.POINTER(C.c_void_p)),
        ("wo", C.POINTER(C.c_void_p)), ("wgate", C.POINTER(C.c_void_p)), ("wup", C.POINTER(C.c_void_p)),
        ("wdown", C.POINTER(C.c_void_p)),
        ("tq", C.POINTER(C.c_int)), ("tk", C.POINTER(C.c_int)), ("tv", C.POINTER(C.c_int)),
        ("to", C.POINTER(C.c_int)), ("tgate", C.POINTER(C.c_int)), ("tup", C.POINTER(C.c_int)),
        ("tdown", C.POINTER(C.c_int)),
        ("vocab_full", C.c_uint32), ("vocab_offset", C.c_uint32),
    ]


_LIB = None


def build(force: bool = False) -> Path:
    """Compile libvbs_b200.so in place (nvcc, sm_100a). Returns its path."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-C", str(PKG_DIR), "-j8"], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    """The loaded library; raises when it is missing (no fallback exists)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise VbsError(f"{LIB_PATH} is not built; run build() (make -C {PKG_DIR})")
    # torch first: the library's libnccl.so.2 then resolves to the NCCL that
    # torch already loaded. Loaded the other way round, the older system NCCL
    # takes the soname and torch's CUDA library fails to import.
    import torch  # noqa: F401
    L = C.CDLL(str(LIB_PATH))
    vp, u32, u64, i32, f32, sz = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_size_t
    sig = {
        "vbs_cuda_last_error": (C.c_char_p, []),
        "vbs_cu_status": (i32, []),
        "vbs_cu_clear_error": (None, []),
        "vbs_cu_version": (C.c_char_p, []),
        "vbs_cu_kernel_launches": (u64, []),
        "vbs_cu_dequant": (i32, [i32, vp, vp, u64, vp]),
        "vbs_cu_matvec": (i32, [i32, vp, vp, vp, u32, u32, u32, u32, vp]),
        "vbs_cu_ffn_gate_up": (i32, [i32, vp, vp, vp, vp, f32, vp, u32, u32, vp]),
        "vbs_cu_attention": (i32, [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, f32, u32, u64, vp]),
        "vbs_cu_attention_static": (i32, [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, f32, u32, u64, vp]),
        "vbs_cu_synth": (i32, [i32, vp, u64, u64, u64, u64, u64, u64, f32, vp]),
        "vbs_cu_upload_file": (i32, [C.c_char_p, sz, vp, vp, vp, u32, u64]),
        "vbs_cu_decoder_create": (vp, [C.POINTER(ModelDesc), u32, u32, C.c_char_p, sz]),
        "vbs_cu_decoder_destroy": (None, [vp]),
        "vbs_cu_decoder_forward": (i32, [vp, C.POINTER(u32), sz, C.POINTER(f32)]),
        "vbs_cu_decoder_prefill": (i32, [vp, C.POINTER(u32), sz]),
        "vbs_cu_decoder_reset": (None, [vp]),
        "vbs_cu_decoder_generate": (i32, [vp, C.POINTER(u32), sz, u32, C.POINTER(u32)]),
        "vbs_cu_decoder_enqueue_steps": (i32, [vp, u32]),
        "vbs_cu_decoder_run_control": (i32, [vp, vp]),
        "vbs_cu_decoder_set_wait_test": (i32, [vp, u64, u32]),
        "vbs_cu_decoder_set_position": (i32, [vp, u32, u32]),
        "vbs_cu_decoder_position": (u32, [vp]),
        "vbs_cu_decoder_stream": (vp, [vp]),
        "vbs_cu_batch_decoder_create": (vp, [C.POINTER(ModelDesc), u32, u32, C.c_char_p, sz]),
        "vbs_cu_batch_decoder_destroy": (None, [vp]),
        "vbs_cu_batch_decoder_step": (i32, [vp, C.POINTER(u32), C.POINTER(f32), C.POINTER(u32)]),
        "vbs_cu_batch_decoder_enqueue_steps": (i32, [vp, u32]),
        "vbs_cu_batch_decoder_set_position": (i32, [vp, u32, C.POINTER(u32)]),
        "vbs_cu_batch_decoder_position": (u32, [vp]),
        "vbs_cu_batch_decoder_reset": (None, [vp]),
        "vbs_cu_batch_decoder_stream": (vp, [vp]),
        "vbs_cu_decoder_logits_device": (vp, [vp]),
        "vbs_cu_decoder_kernels_per_step": (u32, [vp]),
        "vbs_cu_decoder_tp_mode": (u32, [vp]),
        "vbs_cu_tp_unique_id": (i32, [vp]),
        "vbs_cu_tp_init": (i32, [i32, i32, vp]),
        "vbs_cu_tp_finalize": (i32, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = L
    return L


def last_error() -> str:
    return lib().vbs_cuda_last_error().decode()


def clear_error() -> None:
    lib().vbs_cu_clear_error()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise VbsError(f"{what}: {last_error()}")


def ops() -> OpsTable:
    """The drop-in ops table g_vbs_cuda_backend."""
    return OpsTable.in_dll(lib(), "g_vbs_cuda_backend")


def kernel_launches() -> int:
    return int(lib().vbs_cu_kernel_launches())


# ---------------------------------------------------------------------------
# thin wrappers over the extension entry points (device pointers as ints)
# ---------------------------------------------------------------------------
def dequant(type_id: int, w_ptr: int, out_ptr: int, n_elems: int, stream: int = 0) -> None:
    check(lib().vbs_cu_dequant(type_id, w_ptr, out_ptr, n_elems, stream or None), "vbs_cu_dequant")


def matvec(type_id, w_ptr, x_ptr, y_ptr, rows, cols, batch=1, flags=0, stream=0) -> None:
    check(lib().vbs_cu_matvec(type_id, w_ptr, x_ptr, y_ptr, rows, cols, batch, flags, stream or None), "vbs_cu_matvec")


def ffn_gate_up(type_id, wg_ptr, wu_ptr, x_ptr, norm_ptr, eps, h_ptr, rows, cols, stream=0) -> None:
    check(lib().vbs_cu_ffn_gate_up(type_id, wg_ptr, wu_ptr, x_ptr, norm_ptr or None, eps, h_ptr, rows, cols,
                                   stream or None), "vbs_cu_ffn_gate_up")


def attention(q, kc, vc, out, seq_len, layer, max_ctx, nqh, nkh, hd, scale, batch=1, kv_batch_stride=0, stream=0):
    check(lib().vbs_cu_attention(q, kc, vc, out, seq_len, layer, max_ctx, nqh, nkh, hd, scale, batch,
                                 kv_batch_stride, stream or None), "vbs_cu_attention")


def attention_static(q, kc, vc, out, seq_len, layer, max_ctx, nqh, nkh, hd, scale, batch=1, kv_batch_stride=0,
                     stream=0):
    """vbs_cu_attention_static: the same op with a fixed per-device scratch
    and no device allocation (see include/vbs_b200.h for its limit)."""
    check(lib().vbs_cu_attention_static(q, kc, vc, out, seq_len, layer, max_ctx, nqh, nkh, hd, scale, batch,
                                        kv_batch_stride, stream or None), "vbs_cu_attention_static")


def synth(type_id, dst_ptr, rows, cols, seed, scale, row0=0, col0=0, full_cols=None, stream=0) -> None:
    check(lib().vbs_cu_synth(type_id, dst_ptr, rows, cols, row0, col0, full_cols or cols, seed, scale,
                             stream or None), "vbs_cu_synth")


def synth_scale(std: float) -> float:
    """Float scale that gives the Irwin-Hall(4) synthesizer a standard deviation `std`."""
    return float(struct.unpack("<f", struct.pack("<f", std / ((65536.0 * 65536.0 - 1.0) / 3.0) ** 0.5))[0])


# ---------------------------------------------------------------------------
# models resident on the device
# ---------------------------------------------------------------------------
@dataclass
class LlamaShape:
    n_layers: int
    dim: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    eps: float = 1e-5
    theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads


@dataclass
class DeviceModel:
    """Weights on the device (torch uint8/float32 tensors own the memory)
    plus the vbs_cu_model_t that points at them."""
    shape: LlamaShape
    types: dict
    tensors: dict = field(default_factory=dict)
    desc: ModelDesc | None = None
    _keep: list = field(default_factory=list)
    tp_rank: int = 0
    tp_world: int = 1

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors.values())

    def make_desc(self) -> ModelDesc:
        s, T = self.shape, self.tensors
        n = s.n_layers
        P = C.c_void_p * n
        I = C.c_int * n
        lw = lambda key: P(*[T[f"blk.{l}.{key}"].data_ptr() for l in range(n)])
        lt = lambda key: I(*[self.types[key]] * n)
        arrs = dict(attn_norm=lw("attn_norm"), ffn_norm=lw("ffn_norm"), wq=lw("attn_q"), wk=lw("attn_k"),
                    wv=lw("attn_v"), wo=lw("attn_output"), wgate=lw("ffn_gate"), wup=lw("ffn_up"),
                    wdown=lw("ffn_down"), tq=lt("attn_q"), tk=lt("attn_k"), tv=lt("attn_v"),
                    to=lt("attn_output"), tgate=lt("ffn_gate"), tup=lt("ffn_up"), tdown=lt("ffn_down"))
        self._keep = list(arrs.values())
        d = ModelDesc()
        d.n_layers, d.dim, d.n_heads, d.n_kv_heads = n, s.dim, s.n_heads // self.tp_world, s.n_kv_heads // self.tp_world
        d.head_dim, d.ffn, d.vocab = s.head_dim, s.ffn // self.tp_world, s.vocab // self.tp_world
        d.eps, d.theta = s.eps, s.theta
        d.embd_type, d.out_type = self.types["token_embd"], self.types["output"]
        d.embd, d.out, d.out_norm = T["token_embd"].data_ptr(), T["output"].data_ptr(), T["output_norm"].data_ptr()
        for k, v in arrs.items():
            setattr(d, k, C.cast(v, C.POINTER(C.c_void_p) if k.startswith(("w", "attn", "ffn")) else C.POINTER(C.c_int)))
        d.vocab_full = s.vocab
        d.vocab_offset = self.tp_rank * (s.vocab // self.tp_world)
        self.desc = d
        return d


def streamed_model(model: "DeviceModel") -> "DeviceModel":
    """The same model with its per-layer matrices moved to pinned host
    memory, for a VBS_CU_DEC_STREAM decoder (slice streaming); the
    embedding, output matrix and norm weights stay on the device."""
    import torch
    m = DeviceModel(shape=model.shape, types=dict(model.types), tp_rank=model.tp_rank, tp_world=model.tp_world)
    for name, t in model.tensors.items():
        if name.startswith("blk.") and not name.endswith("norm"):
            h = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            h.copy_(t)
            m.tensors[name] = h
        else:
            m.tensors[name] = t
    m.make_desc()
    return m


# Per-tensor seeds of synthetic models: a fixed function of the model seed
# and the tensor's name, so every rank of a TP group (and the host oracle)
# draws the same full tensors and takes its own slice.
def tensor_seed(model_seed: int, name: str) -> int:
    h = 1469598103934665603
    for ch in name.encode():
        h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return (h ^ (model_seed * 0x9E3779B97F4A7C15)) & 0xFFFFFFFFFFFFFFFF


def shard_spec(name: str, shape: LlamaShape, rank: int, world: int):
    """(rows, cols, row0, col0, full_cols) of this rank's slice of `name`.
    Megatron-style: q/k/v/gate/up/output by rows, o/down by columns."""
    hd, D, F = shape.head_dim, shape.dim, shape.ffn
    base = name.split(".")[-1] if name.startswith("blk.") else name
    full = {"attn_q": (shape.n_heads * hd, D), "attn_k": (shape.n_kv_heads * hd, D),
            "attn_v": (shape.n_kv_heads * hd, D), "attn_output": (D, shape.n_heads * hd), "ffn_gate": (F, D),
            "ffn_up": (F, D), "ffn_down": (D, F), "output": (shape.vocab, D), "token_embd": (shape.vocab, D)}[base]
    rows, cols = full
    if world == 1 or base == "token_embd":
        return rows, cols, 0, 0, cols
    if base in ("attn_output", "ffn_down"):
        if cols % world:
            raise ValueError(f"{name}: {cols} columns do not split over {world} ranks")
        c = cols // world
        return rows, c, 0, rank * c, cols
    if rows % world:
        raise ValueError(f"{name}: {rows} rows do not split over {world} ranks")
    r = rows // world
    return r, cols, rank * r, 0, cols


def synth_llama(shape: LlamaShape, types: dict, seed: int = 1234, std: float = 0.02, device="cuda",
                tp_rank: int = 0, tp_world: int = 1, stream: int = 0) -> DeviceModel:
    """A seeded random llama-shaped model generated and quantized on the
    device (norm weights 1.0). `types` maps token_embd, output, attn_q,
    attn_k, attn_v, attn_output, ffn_gate, ffn_up, ffn_down to type ids."""
    import torch
    m = DeviceModel(shape=shape, types=dict(types), tp_rank=tp_rank, tp_world=tp_world)
    sc = synth_scale(std)

    def add(name, base):
        rows, cols, r0, c0, fc = shard_spec(name, shape, tp_rank, tp_world)
        t = torch.empty(rows * row_bytes(types[base], cols) + 256, dtype=torch.uint8, device=device)
        synth(types[base], t.data_ptr(), rows, cols, tensor_seed(seed, name), sc, r0, c0, fc, stream)
        m.tensors[name] = t

    add("token_embd", "token_embd")
    add("output", "output")
    m.tensors["output_norm"] = torch.ones(shape.dim, dtype=torch.float32, device=device)
    for l in range(shape.n_layers):
        for base in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            add(f"blk.{l}.{base}", base)
        m.tensors[f"blk.{l}.attn_norm"] = torch.ones(shape.dim, dtype=torch.float32, device=device)
        m.tensors[f"blk.{l}.ffn_norm"] = torch.ones(shape.dim, dtype=torch.float32, device=device)
    m.make_desc()
    torch.cuda.synchronize(device)   # the weights are complete when this returns
    return m


class Decoder:
    """vbs_cu_decoder_t: the decode step as one replayable device program."""

    def __init__(self, model: DeviceModel, max_ctx: int, flags: int = 0):
        self.model = model
        desc = model.desc or model.make_desc()
        err = C.create_string_buffer(512)
        self.h = lib().vbs_cu_decoder_create(C.byref(desc), max_ctx, flags, err, 512)
        if not self.h:
            raise VbsError(f"vbs_cu_decoder_create: {err.value.decode()}")
        self.max_ctx = max_ctx
        self.vocab = model.shape.vocab

    def forward(self, tokens, logits: bool = True):
        import numpy as np
        arr = (C.c_uint32 * len(tokens))(*[int(t) for t in tokens])
        out = np.empty(self.vocab, dtype=np.float32) if logits else None
        ptr = out.ctypes.data_as(C.POINTER(C.c_float)) if logits else None
        check(lib().vbs_cu_decoder_forward(self.h, arr, len(tokens), ptr), "vbs_cu_decoder_forward")
        return out

    def prefill(self, tokens) -> None:
        """The tokens as context (KV rows only, chunks of up to 512 through
        the tcgen05 GEMM); the next forward continues after them."""
        arr = (C.c_uint32 * max(len(tokens), 1))(*tokens)
        check(lib().vbs_cu_decoder_prefill(self.h, arr, len(tokens)), "vbs_cu_decoder_prefill")

    def forward_prompt(self, tokens):
        """Logits after the whole prompt: prefill all but the last token,
        then one step for the last."""
        if len(tokens) > 1:
            self.prefill(tokens[:-1])
        return self.forward(tokens[-1:])

    def forward_into(self, tok_arr, n: int, logits_ptr) -> None:
        check(lib().vbs_cu_decoder_forward(self.h, tok_arr, n, logits_ptr), "vbs_cu_decoder_forward")

    def generate(self, prompt, n_new: int):
        arr = (C.c_uint32 * len(prompt))(*[int(t) for t in prompt])
        out = (C.c_uint32 * max(1, n_new))()
        check(lib().vbs_cu_decoder_generate(self.h, arr, len(prompt), n_new, out), "vbs_cu_decoder_generate")
        return list(out)[:n_new]

    def reset(self) -> None:
        lib().vbs_cu_decoder_reset(self.h)

    def set_position(self, pos: int, token: int) -> None:
        check(lib().vbs_cu_decoder_set_position(self.h, pos, token), "vbs_cu_decoder_set_position")

    @property
    def position(self) -> int:
        return int(lib().vbs_cu_decoder_position(self.h))

    def set_wait_test(self, wait_ns: int, drop_op: int = 0xFFFFFFFF) -> None:
        """Bounded-wait test control: the step kernel's wait limit and an op
        before whose grid barrier CTA 0 withholds its arrival."""
        check(lib().vbs_cu_decoder_set_wait_test(self.h, wait_ns, drop_op), "vbs_cu_decoder_set_wait_test")

    def enqueue_steps(self, n: int) -> None:
        check(lib().vbs_cu_decoder_enqueue_steps(self.h, n), "vbs_cu_decoder_enqueue_steps")

    @property
    def stream(self) -> int:
        return int(lib().vbs_cu_decoder_stream(self.h) or 0)

    @property
    def kernels_per_step(self) -> int:
        return int(lib().vbs_cu_decoder_kernels_per_step(self.h))

    @property
    def tp_mode(self) -> str:
        """"single", "nccl" or "peer-memory": how the per-layer TP sums run."""
        return ("single", "nccl", "peer-memory")[int(lib().vbs_cu_decoder_tp_mode(self.h))]

    def close(self) -> None:
        if self.h:
            lib().vbs_cu_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchDecoder:
    """vbs_cu_batch_decoder_t: `batch` sequences decoded in lockstep, one
    token each per step at the same position."""

    def __init__(self, model: DeviceModel, max_ctx: int, batch: int):
        self.model = model
        desc = model.desc or model.make_desc()
        err = C.create_string_buffer(512)
        self.h = lib().vbs_cu_batch_decoder_create(C.byref(desc), max_ctx, batch, err, 512)
        if not self.h:
            raise VbsError(f"vbs_cu_batch_decoder_create: {err.value.decode()}")
        self.batch, self.max_ctx, self.vocab = batch, max_ctx, model.shape.vocab

    def step(self, tokens=None, logits: bool = True):
        """One step; tokens: one id per sequence (None: the previous argmaxes).
        Returns (logits [batch][vocab] or None, next tokens)."""
        import numpy as np
        arr = (C.c_uint32 * self.batch)(*[int(t) for t in tokens]) if tokens is not None else None
        out = np.empty((self.batch, self.vocab), dtype=np.float32) if logits else None
        nxt = (C.c_uint32 * self.batch)()
        check(lib().vbs_cu_batch_decoder_step(self.h, arr, out.ctypes.data_as(C.POINTER(C.c_float)) if logits else None,
                                               nxt), "vbs_cu_batch_decoder_step")
        return out, list(nxt)

    def enqueue_steps(self, n: int) -> None:
        check(lib().vbs_cu_batch_decoder_enqueue_steps(self.h, n), "vbs_cu_batch_decoder_enqueue_steps")

    def set_position(self, pos: int, tokens=None) -> None:
        arr = (C.c_uint32 * self.batch)(*[int(t) for t in tokens]) if tokens is not None else None
        check(lib().vbs_cu_batch_decoder_set_position(self.h, pos, arr), "vbs_cu_batch_decoder_set_position")

    @property
    def position(self) -> int:
        return int(lib().vbs_cu_batch_decoder_position(self.h))

    def reset(self) -> None:
        lib().vbs_cu_batch_decoder_reset(self.h)

    @property
    def stream(self) -> int:
        return int(lib().vbs_cu_batch_decoder_stream(self.h) or 0)

    def close(self) -> None:
        if self.h:
            lib().vbs_cu_batch_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# GGUF v3 (the container the reference loads, src/vbs_gguf.c)
# ---------------------------------------------------------------------------
_GG_U32, _GG_F32, _GG_STR, _GG_ARR = 4, 6, 8, 9


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32) -> None:
    """tensors: [(name, type_id, dims (ne0 = columns first), data)], data
    any bytes-like buffer (written as is, not copied). metadata values: int
    -> u32, float -> f32, str -> string, and a list of one of those -> array
    (the tokenizer tables of real model files)."""
    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    def typed(v) -> tuple[int, bytes]:
        if isinstance(v, str):
            return _GG_STR, s(v)
        if isinstance(v, float):
            return _GG_F32, struct.pack("<f", v)
        return _GG_U32, struct.pack("<I", int(v))

    kv = b""
    for k, v in metadata.items():
        if isinstance(v, (list, tuple)):
            et = typed(v[0])[0] if v else _GG_U32
            kv += s(k) + struct.pack("<IIQ", _GG_ARR, et, len(v)) + b"".join(typed(e)[1] for e in v)
        else:
            t, b = typed(v)
            kv += s(k) + struct.pack("<I", t) + b
    info, blobs, off = b"", [], 0
    for name, typ, dims, data in tensors:
        if off % alignment:
            pad = alignment - off % alignment
            blobs.append(b"\0" * pad)
            off += pad
        info += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        info += struct.pack("<IQ", typ, off)
        mv = memoryview(data).cast("B")
        blobs.append(mv)
        off += mv.nbytes
    head = struct.pack("<4sIQQ", b"GGUF", 3, len(tensors), len(metadata)) + kv + info
    start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (start - len(head)))
        for b in blobs:
            f.write(b)


_GG_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


@dataclass
class GgufTensor:
    type: int
    dims: tuple            # ne0 (columns) first
    offset: int            # absolute file offset of the data
    nbytes: int | None     # None for a type this library has no block size for


def gguf_layout(path) -> tuple[dict, dict]:
    """GGUF v3 header (src/vbs_gguf.c): (metadata, {name: GgufTensor}),
    reading only the header, never the tensor data. Metadata arrays (the
    tokenizer's, in real model files) are read into lists."""
    with open(path, "rb") as f:
        def rd(fmt):
            n = struct.calcsize(fmt)
            b = f.read(n)
            if len(b) != n:
                raise ValueError(f"{path}: GGUF header ends early")
            return struct.unpack(fmt, b)

        def rs():
            (n,) = rd("<Q")
            b = f.read(n)
            if len(b) != n:
                raise ValueError(f"{path}: GGUF header ends early")
            return b.decode("utf-8", errors="replace")

        def value(t):
            if t == _GG_STR:
                return rs()
            if t in _GG_SCALAR:
                return rd(_GG_SCALAR[t])[0]
            if t == _GG_ARR:
                et, n = rd("<IQ")
                if et in _GG_SCALAR:   # one read for a scalar array
                    fmt = _GG_SCALAR[et]
                    return list(rd("<" + fmt[1:] * n)) if n else []
                return [value(et) for _ in range(n)]
            raise ValueError(f"unsupported GGUF metadata type {t}")

        magic, ver, nt, nkv = rd("<4sIQQ")
        if magic != b"GGUF" or ver != 3:
            raise ValueError("not a GGUF v3 file")
        meta = {}
        for _ in range(nkv):
            k = rs()
            (t,) = rd("<I")
            meta[k] = value(t)
        infos = []
        for _ in range(nt):
            name = rs()
            (nd,) = rd("<I")
            dims = rd("<" + "Q" * nd)
            typ, rel = rd("<IQ")
            infos.append((name, typ, dims, rel))
        o = f.tell()
    align = int(meta.get("general.alignment", 32))
    start = (o + align - 1) // align * align
    tens = {}
    for name, typ, dims, rel in infos:
        rows = 1
        for d in dims[1:]:
            rows *= d
        nbytes = row_bytes(typ, dims[0]) * rows if typ in BLOCK else None
        tens[name] = GgufTensor(typ, tuple(dims), start + rel, nbytes)
    return meta, tens


def read_gguf(path) -> tuple[dict, dict]:
    """Minimal GGUF v3 reader: (metadata, {name: (type, dims, bytes)})."""
    meta, lay = gguf_layout(path)
    tens = {}
    with open(path, "rb") as f:
        for name, t in lay.items():
            if t.nbytes is None:
                raise ValueError(f"{name}: tensor type {t.type} is not supported")
            f.seek(t.offset)
            b = f.read(t.nbytes)
            if len(b) != t.nbytes:
                raise ValueError(f"{name}: file ends inside the tensor")
            tens[name] = (t.type, t.dims, b)
    return meta, tens


def upload_file(path, ranges, n_threads: int = 0, chunk_bytes: int = 0) -> None:
    """ranges: [(file offset, bytes, device pointer)]; one native call
    (vbs_cu_upload_file: reader threads, pinned staging, async copies)."""
    n = len(ranges)
    offs = (C.c_uint64 * max(n, 1))(*[r[0] for r in ranges])
    sizes = (C.c_uint64 * max(n, 1))(*[r[1] for r in ranges])
    dsts = (C.c_void_p * max(n, 1))(*[r[2] for r in ranges])
    check(lib().vbs_cu_upload_file(str(path).encode(), n, offs, sizes, dsts, n_threads, chunk_bytes),
          "vbs_cu_upload_file")


def upload_gguf(path, device="cuda", n_threads: int = 0) -> DeviceModel:
    """Load a llama GGUF onto the device straight from the file: the header
    gives every tensor's offset, device buffers are allocated (matrices with
    256 zero bytes of tail padding), then one vbs_cu_upload_file call moves
    all tensors through pinned staging buffers. Replaces the reference's
    host mirror plus one synchronous copy_to_device per tensor
    (src/vbs_fabric.c:81-94)."""
    import torch
    meta, tens = gguf_layout(path)
    a = "llama."
    nl = int(meta[a + "block_count"])
    dim = int(meta[a + "embedding_length"])
    nh = int(meta[a + "attention.head_count"])
    nkv = int(meta.get(a + "attention.head_count_kv", nh))
    ffn = int(meta[a + "feed_forward_length"])
    vocab = tens["token_embd.weight"].dims[1]
    shape = LlamaShape(nl, dim, nh, nkv, ffn, vocab, float(meta.get(a + "attention.layer_norm_rms_epsilon", 1e-5)),
                       float(meta.get(a + "rope.freq_base", 10000.0)))
    types = {"token_embd": tens["token_embd.weight"].type,
             "output": tens.get("output.weight", tens["token_embd.weight"]).type}
    for base in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
        types[base] = tens[f"blk.0.{base}.weight"].type
    m = DeviceModel(shape=shape, types=types)
    ranges = []

    def put(key, name, as_float=False):
        t = tens[name]
        if t.nbytes is None:
            raise ValueError(f"{name}: tensor type {t.type} is not supported")
        if as_float:
            if t.type != F32:
                raise ValueError(f"{name}: norm weights must be F32")
            buf = torch.empty(t.nbytes // 4, dtype=torch.float32, device=device)
        else:
            buf = torch.zeros(t.nbytes + 256, dtype=torch.uint8, device=device)
        m.tensors[key] = buf
        ranges.append((t.offset, t.nbytes, buf.data_ptr()))

    put("token_embd", "token_embd.weight")
    put("output", "output.weight" if "output.weight" in tens else "token_embd.weight")
    put("output_norm", "output_norm.weight", as_float=True)
    for l in range(nl):
        for base in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
            put(f"blk.{l}.{base}", f"blk.{l}.{base}.weight")
        put(f"blk.{l}.attn_norm", f"blk.{l}.attn_norm.weight", as_float=True)
        put(f"blk.{l}.ffn_norm", f"blk.{l}.ffn_norm.weight", as_float=True)
    torch.cuda.synchronize()   # the buffers' clears come before the copies
    upload_file(path, ranges, n_threads)
    m.make_desc()
    return m
