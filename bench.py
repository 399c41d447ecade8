"""Decode benchmark: Llama-3-8B-shaped Q4_K model, tokens/s.

A "step" is one decode token of the full model: embedding, 32 layers of
norm + Q/K/V + RoPE + KV store + split-KV attention + o_proj + norm +
gate/up + SiLU + down, final norm, the 128256-row output projection and
the greedy argmax, replayed as one CUDA graph through the C ABI
(libvbs_b200.so, vbs_cu_decoder_*). Weights are seeded N(0, 0.02) synthesized
and quantized on the device (Q4_K attention and gate/up, Q6_K down, output
and embedding; no network, no checkpoint); the KV cache is filled by a real
prefill of `--ctx` seeded prompt tokens (untimed), then K timed steps decode
at context ctx..ctx+K. 4.84 GB of weights per token are far larger than the
126 MB L2, so nothing is flushed between steps.

Prints one JSON line (rank 0). N > 1 runs under torchrun as tensor
parallelism over NVLink (NCCL all-reduce after o_proj and down_proj).
`--impl reference` times the reference's CPU decode kernel instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "tests"):
    sys.path.insert(0, str(p))

# Algorithmic bytes (weights excluding the embedding table, which decode
# reads one row of) per token for the 8B shape, and KV bytes per position.
L8B_WEIGHT_BYTES = 4_841_250_816
KV_BYTES_PER_POS = 32 * 8 * 128 * 2 * 2     # layers x kv heads x head_dim x (K,V) x fp16
FFN_GATE_UP_BYTES = 2 * 14336 * 4096 // 256 * 144   # the dominant kernel: two Q4_K [14336 x 4096]
# weights (elements) one decode step multiplies: 32 x 218,103,808 + 128256 x 4096
L8B_WEIGHTS = 32 * (2 * 4096 * 4096 + 2 * 1024 * 4096 + 3 * 14336 * 4096) + 128256 * 4096


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-layers", type=int, default=32,
                    help="--impl reference: layers of the 8B shape (fewer only to check the JSON contract quickly)")
    ap.add_argument("--profile", default=None,
                    choices=["ffn_gate_up", "down", "output", "qkv_like", "attention", "decode", "sweep", "prefill",
                             "upload", "stream", "timeline"],
                    help="run only this kernel on its 8B shape, --steps launches over rotating weight sets "
                         "(a small case for ncu); prints per-launch times")
    ap.add_argument("--layers", type=int, default=32, help="--profile decode/timeline: layers of the model")
    ap.add_argument("--vocab", type=int, default=128256, help="--profile decode: vocabulary rows")
    ap.add_argument("--shape", default="8b", choices=["8b", "70b"],
                    help="--profile decode/timeline: the Llama-3-8B mix (BASELINE config 3) or the 70B shape, all Q4_K "
                         "(config 4)")
    ap.add_argument("--batch", type=int, default=1,
                    help="--profile decode: sequences decoded in lockstep (the batch decoder when above 1)")
    ap.add_argument("--per-op", action="store_true",
                    help="--profile decode: the per-op kernels (one launch per op) instead of the one-launch step")
    return ap.parse_args()


TIMELINE_LIB = ROOT / "verum-bespoke-singularity_b200" / "libvbs_b200_trace.so"


def profile_timeline(args):
    """Where a step kernel's time goes, op by op: the profiling build of the
    library (`make -C verum-bespoke-singularity_b200 trace`) stamps
    %globaltimer per CTA at each op's start (after its grid barrier), at the
    end of its prologue and at its end, and the producer warp's first and
    last stage issue. One step at position --ctx - 1, three times; the last
    one's per-op figures, medians over CTAs, averaged over the middle layers
    (1 .. L-2) per op kind, in microseconds:
      span      last CTA's end of the previous op -> last CTA's end of this op
      barrier   last CTA's end of the previous op -> first CTA's start
      prologue  start -> prologue done (norm, x quantization)
      body      prologue done (ATTN: start) -> end
      prod_lead consumer start - producer's last issue for the op (> 0: the
                op's weights were all in flight before its consumers began)
    and the phases inside (medians over CTAs of thread 0's stamps): the
    prologue's first instruction after the barrier (pro_entry), the norm
    prologue's loads and sum of squares, its wait for the norm weight stage
    and its quantization; attention's q/KV setup, first and last stage
    arrival, stage loop, partial store, wait for the head's other splits and
    merge; l2_probe, one dependent L2 load of the op's input timed right
    after the prologue (attention: after the merge); and stamp, two stamps
    back to back (what one stamp costs)."""
    import ctypes as C
    import numpy as np
    import torch
    import vbs_b200 as vbs
    import models
    if not TIMELINE_LIB.exists():
        raise SystemExit(f"{TIMELINE_LIB} is not built: make -C {TIMELINE_LIB.parent} trace")
    vbs.LIB_PATH = TIMELINE_LIB
    L = vbs.lib()
    L.vbs_cu_decoder_trace.restype = C.c_void_p
    L.vbs_cu_decoder_trace.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
    torch.cuda.set_device(0)
    if not vbs.ops().init():
        raise SystemExit(vbs.last_error())
    nl = args.layers
    base, types = (models.L70B, models.L70B_TYPES) if args.shape == "70b" else (models.L8B, models.L8B_TYPES)
    cfg = dict(base, n_layers=nl, vocab=args.vocab)
    model = vbs.synth_llama(models.shape_of(cfg), types, seed=2024)
    dec = vbs.Decoder(model, args.ctx + 64)
    dec.forward([1], logits=False)
    dec.set_position(args.ctx - 1, 1)
    dec.enqueue_steps(4)
    torch.cuda.synchronize()
    kinds = ["QKV", "ATTN", "O", "GU", "DOWN"]
    ops_t = vbs.ops()
    s = torch.cuda.ExternalStream(dec.stream)
    for rep in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        dec.enqueue_steps(1)
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        nc, no, ns = C.c_uint32(), C.c_uint32(), C.c_uint32()
        ptr = L.vbs_cu_decoder_trace(dec.h, C.byref(nc), C.byref(no), C.byref(ns))
        n = nc.value * no.value * ns.value
        host = np.zeros(n, np.uint64)
        buf = vbs.Buffer()
        buf.internal_handle, buf.size = ptr, n * 8
        assert ops_t.copy_to_host(host.ctypes.data, C.byref(buf), n * 8), vbs.last_error()
    raw = host.reshape(nc.value, no.value, ns.value)
    T = raw.astype(np.int64)
    T -= T[:, 0, 0].min()

    def phase(i, a, b):   # median over the CTAs that stamped both
        ok = (raw[:, i, a] > 0) & (raw[:, i, b] > 0)
        return float(np.median(T[ok, i, b] - T[ok, i, a])) / 1e3 if ok.any() else 0.0

    per_op, prev_end = [], 0
    for i in range(no.value):
        st, pro, en, pf, pl = (T[:, i, k] for k in range(5))
        k = kinds[i % 5] if i < 5 * nl else ("OUT", "ARGMAX")[i - 5 * nl]
        normed = k not in ("ATTN", "ARGMAX")
        r = {"op": k, "i": i, "span": (en.max() - prev_end) / 1e3, "barrier": (st.min() - prev_end) / 1e3 if i else 0.0,
             "prologue": float(np.median(pro - st)) / 1e3 if normed else 0.0,
             "body": float(np.median(en - (pro if normed else st))) / 1e3,
             "prod_lead": float(np.median(st - pl)) / 1e3 if k != "ARGMAX" else 0.0}
        if k in ("QKV", "GU", "OUT"):
            r.update(pro_entry=phase(i, 0, 8), pro_sums=phase(i, 8, 5), pro_weight=phase(i, 5, 6),
                     pro_quant=phase(i, 6, 7), l2_probe=phase(i, 9, 10))
        if k in ("O", "DOWN"):
            r.update(pro_entry=phase(i, 0, 8), l2_probe=phase(i, 9, 10))
        r.update(stamp=phase(i, 0, 11))
        if k not in ("ATTN", "ARGMAX"):
            r.update(param=phase(i, 11, 12), layer_ptr=phase(i, 11, 13))
        if k == "ATTN":
            r.update(setup=phase(i, 0, 1), first_stage=phase(i, 1, 8), last_stage=phase(i, 1, 9), stages=phase(i, 1, 5),
                     partial=phase(i, 5, 6), wait=phase(i, 6, 7), merge=phase(i, 7, 2), l2_probe=phase(i, 10, 11))
        per_op.append(r)
        prev_end = en.max()
    table = {}
    for r in per_op:
        if r["op"] not in kinds or 5 <= r["i"] < 5 * (nl - 1):
            table.setdefault(r["op"], []).append(r)
    out = {k: {f: round(float(np.mean([r[f] for r in v])), 2) for f in v[0] if f not in ("op", "i")}
           for k, v in table.items()}
    layer_us = sum(out[k]["span"] for k in kinds)
    print(json.dumps({"profile": "timeline", "shape": args.shape, "ctx": args.ctx, "layers": nl, "vocab": args.vocab,
                      "event_ms": round(ms, 4),
                      "traced_us": round(prev_end / 1e3, 1), "layer_us": round(layer_us, 2), "per_op_us": out}))
    dec.close()


def profile_kernel(args):
    """Standalone launches of one hot kernel at its Llama-3-8B shape. Four
    weight sets rotate so no launch finds its weights in L2."""
    import torch
    import vbs_b200 as vbs
    if args.profile == "timeline":   # loads the profiling build instead of the product library
        profile_timeline(args)
        return
    torch.cuda.set_device(0)
    if not vbs.ops().init():
        raise SystemExit(vbs.last_error())
    sc = vbs.synth_scale(0.02)
    shapes = {"ffn_gate_up": (vbs.Q4_K, 14336, 4096), "down": (vbs.Q6_K, 4096, 14336),
              "output": (vbs.Q6_K, 128256, 4096), "qkv_like": (vbs.Q4_K, 6144, 4096)}
    st = torch.cuda.Stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    if args.profile == "sweep":
        # the BASELINE matvec sweep through vbs_cu_matvec: 4 shapes x {Q4_K,
        # Q6_K} x batch {1, 8}; weight sets rotate so no launch hits L2
        # (sets x bytes > 126 MB), one line per point
        peak, _ = peaks()
        for t in (vbs.Q4_K, vbs.Q6_K):
            for rows, cols in ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)):
                rb = vbs.row_bytes(t, cols)
                nset = max(2, min(8, -(-300_000_000 // (rows * rb))))
                ws = []
                for i in range(nset):
                    w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
                    vbs.synth(t, w.data_ptr(), rows, cols, 300 + i, sc)
                    ws.append(w)
                for b in (1, 8):
                    x = torch.randn((b, cols), device="cuda")
                    y = torch.empty((b, rows), device="cuda")
                    n = max(4, min(args.steps, 24))
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * n)]
                    torch.cuda.synchronize()
                    with torch.cuda.stream(st):
                        for i in range(n):
                            ev[2 * i].record(st)
                            vbs.matvec(t, ws[i % nset].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, batch=b,
                                       stream=st.cuda_stream)
                            ev[2 * i + 1].record(st)
                    torch.cuda.synchronize()
                    us = sorted(ev[2 * i].elapsed_time(ev[2 * i + 1]) * 1e3 for i in range(1, n))
                    med = us[len(us) // 2]
                    alg = rows * rb + b * cols * 4 + b * rows * 4
                    print(json.dumps({"profile": "sweep", "type": vbs.TYPE_NAMES[t], "rows": rows, "cols": cols, "batch": b,
                                      "median_us": round(med, 2), "algorithmic_bytes": alg,
                                      "gbs": round(alg / (med * 1e-6) / 1e9, 1),
                                      "frac_of_measured": round(alg / (med * 1e-6) / 1e9 / peak, 3)}), flush=True)
                del ws
        return
    if args.profile == "upload":
        # direct file -> device upload (vbs_cu_upload_file): a 2 GiB file of
        # seeded bytes in 64 ranges, read once to warm the page cache, then
        # timed (wall clock around the call; it returns after every copy)
        import tempfile
        import numpy as np
        n, size = 64, 32 << 20
        with tempfile.TemporaryDirectory() as td:
            path = Path(td) / "blob.bin"
            rng = np.random.default_rng(5)
            with open(path, "wb") as f:
                for _ in range(n):
                    f.write(rng.integers(0, 256, size, dtype=np.uint8).tobytes())
            bufs = [torch.empty(size, dtype=torch.uint8, device="cuda") for _ in range(n)]
            torch.cuda.synchronize()
            ranges = [(i * size, size, b.data_ptr()) for i, b in enumerate(bufs)]
            res = {}
            for threads in (1, 4, 8):
                vbs.upload_file(path, ranges, threads)   # warm: page cache, pinned allocations
                t0 = time.perf_counter()
                vbs.upload_file(path, ranges, threads)
                s = time.perf_counter() - t0
                res[f"threads_{threads}"] = {"s": round(s, 4), "gb_s": round(n * size / s / 1e9, 2)}
            ok = bool(np.array_equal(bufs[-1][:4096].cpu().numpy(),
                                     np.fromfile(path, dtype=np.uint8, count=4096, offset=(n - 1) * size)))
        print(json.dumps({"profile": "upload", "bytes": n * size, "ranges": n, "page_cache": "warm", "check": ok,
                          **res}))
        return
    if args.profile == "prefill":
        # the batched prompt pass: --ctx prompt tokens (chunks of 256 through
        # the tcgen05 GEMM) against the same prompt fed one token per step,
        # both timed with CUDA events on the decoder's stream; --layers and
        # --vocab cut the model for a small ncu case
        import models
        cfg = dict(models.L8B, n_layers=args.layers, vocab=args.vocab)
        model = vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=2024)
        prompt = models.splitmix_ints(4096, args.ctx, args.vocab)
        res = {}
        for mode in ("batched", "token-by-token"):
            dec = vbs.Decoder(model, args.ctx + 8, vbs.DEC_NO_PERSIST if args.per_op else 0)
            if mode == "batched":   # warm-up: buffers, workspaces, first launches
                dec.prefill(prompt[:8])
            else:
                dec.forward(prompt[:8], logits=False)
            dec.reset()
            s = torch.cuda.ExternalStream(dec.stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(s)
            if mode == "batched":
                dec.prefill(prompt)
            else:
                dec.forward(prompt, logits=False)
            e1.record(s)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            res[mode] = {"ms": round(ms, 2), "tok_s": round(args.ctx / (ms * 1e-3), 1)}
            dec.close()
        print(json.dumps({"profile": "prefill", "ctx": args.ctx, "layers": args.layers, "vocab": args.vocab,
                          "per_op": bool(args.per_op), **res}))
        return
    if args.profile == "stream":
        # slice streaming: the 8B shape's layer matrices in pinned host
        # memory, copied in layer by layer every step (PCIe-bound), against
        # the same model resident, per-op kernels, --steps steps each
        import models
        cfg = dict(models.L8B, n_layers=args.layers, vocab=args.vocab)
        model = vbs.synth_llama(models.shape_of(cfg), models.L8B_TYPES, seed=2024)
        host = vbs.streamed_model(model)
        layer_bytes = sum(t.numel() for n, t in host.tensors.items() if n.startswith("blk.0.") and not n.endswith("norm"))
        res = {}
        for mode, m, fl in (("streamed", host, vbs.DEC_STREAM), ("resident", model, vbs.DEC_NO_PERSIST)):
            dec = vbs.Decoder(m, args.ctx + args.steps + 16, fl)
            dec.forward([1], logits=False)
            dec.set_position(args.ctx - 1, 1)
            dec.enqueue_steps(2)
            torch.cuda.synchronize()
            s = torch.cuda.ExternalStream(dec.stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            dec.enqueue_steps(args.steps)
            e1.record(s)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            res[mode] = {"ms_per_step": round(ms, 3), "tok_s": round(1000.0 / ms, 2)}
            dec.close()
        gbs = layer_bytes * args.layers / (res["streamed"]["ms_per_step"] * 1e-3) / 1e9
        print(json.dumps({"profile": "stream", "layers": args.layers, "vocab": args.vocab, "ctx": args.ctx,
                          "host_bytes_per_step": layer_bytes * args.layers, "h2d_gb_s": round(gbs, 2), **res}))
        return
    if args.profile == "decode":
        # the full decode step at position --ctx (the cache rows before it
        # are zeros: same bytes and kernels as a prefilled cache), then
        # --steps graph replays timed with CUDA events; --layers/--vocab cut
        # the model for a small ncu case; --shape 70b: BASELINE config 4 on
        # one GPU (39 GB of Q4_K)
        import models
        base, types = (models.L70B, models.L70B_TYPES) if args.shape == "70b" else (models.L8B, models.L8B_TYPES)
        layers = args.layers if args.layers != 32 or args.shape == "8b" else base["n_layers"]
        cfg = dict(base, n_layers=layers, vocab=args.vocab)
        model = vbs.synth_llama(models.shape_of(cfg), types, seed=2024)
        B = max(1, args.batch)
        if B > 1:   # B sequences in lockstep: each step B tokens
            dec = vbs.BatchDecoder(model, args.ctx + args.steps + 8, B)
            dec.step(list(range(1, B + 1)), logits=False)
            dec.set_position(args.ctx - 1, list(range(1, B + 1)))
        else:
            dec = vbs.Decoder(model, args.ctx + args.steps + 8, vbs.DEC_NO_PERSIST if args.per_op else 0)
            dec.forward([1], logits=False)
            dec.set_position(args.ctx - 1, 1)
        dec.enqueue_steps(2)
        torch.cuda.synchronize()
        s = torch.cuda.ExternalStream(dec.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(args.steps):
            dec.enqueue_steps(1)
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / max(1, args.steps)
        wbytes = model.weight_bytes() - model.tensors["token_embd"].numel()
        kv = B * cfg["n_layers"] * cfg["n_kv_heads"] * (cfg["dim"] // cfg["n_heads"]) * 2 * 2 * (args.ctx + 2)
        peak, _ = peaks()
        print(json.dumps({"profile": "decode", "shape": args.shape, "ctx": args.ctx, "layers": cfg["n_layers"],
                          "vocab": args.vocab, "batch": B,
                          "kernels_per_step": dec.kernels_per_step if B == 1 else None, "steps": args.steps,
                          "ms_per_step": round(ms, 4), "tok_s": round(B * 1000.0 / ms, 2),
                          "bytes_per_step": int(wbytes + kv),
                          "frac_of_measured": round((wbytes + kv) / (ms * 1e-3) / 1e9 / peak, 4)}))
        dec.close()
        return
    if args.profile == "attention":
        nqh, nkh, hd, ctx = 32, 8, 128, args.ctx
        kc = [torch.randn((ctx, nkh * hd), device="cuda").half() for _ in range(4)]
        vc = [torch.randn((ctx, nkh * hd), device="cuda").half() for _ in range(4)]
        q = torch.randn(nqh * hd, device="cuda")
        out = torch.empty(nqh * hd, device="cuda")
        alg = 2 * ctx * nkh * hd * 2 + 2 * nqh * hd * 4

        def launch(i):
            vbs.attention(q.data_ptr(), kc[i % 4].data_ptr(), vc[i % 4].data_ptr(), out.data_ptr(), ctx, 0, ctx,
                          nqh, nkh, hd, 0.0883883, stream=st.cuda_stream)
    else:
        t, rows, cols = shapes[args.profile]
        nmat = 2 if args.profile == "ffn_gate_up" else 1
        ws = []
        for i in range(4 * nmat):
            w = torch.empty(rows * vbs.row_bytes(t, cols), dtype=torch.uint8, device="cuda")
            vbs.synth(t, w.data_ptr(), rows, cols, 100 + i, sc)
            ws.append(w)
        x = torch.randn(cols, device="cuda")
        nw = torch.ones(cols, device="cuda")
        y = torch.empty(rows, device="cuda")
        alg = nmat * rows * vbs.row_bytes(t, cols) + cols * 4 + rows * 4

        def launch(i):
            if nmat == 2:
                vbs.ffn_gate_up(t, ws[2 * (i % 4)].data_ptr(), ws[2 * (i % 4) + 1].data_ptr(), x.data_ptr(),
                                nw.data_ptr(), 1e-5, y.data_ptr(), rows, cols, st.cuda_stream)
            else:
                vbs.matvec(t, ws[i % 4].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, stream=st.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        for i in range(args.steps):
            evs[2 * i].record(st)
            launch(i)
            evs[2 * i + 1].record(st)
    torch.cuda.synchronize()
    us = [evs[2 * i].elapsed_time(evs[2 * i + 1]) * 1e3 for i in range(args.steps)]
    med = statistics.median(us[1:] if len(us) > 1 else us)
    print(json.dumps({"profile": args.profile, "launch_us": [round(u, 2) for u in us], "median_us": round(med, 2),
                      "algorithmic_bytes": alg, "gbs": round(alg / (med * 1e-6) / 1e9, 1)}), flush=True)


def peaks():
    try:
        j = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons during the timed region.

    NVML is polled every 5 ms from a thread (read-only queries); only the
    samples taken between mark() and stop() count. Without NVML it falls
    back to `nvidia-smi -lms 100`."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # nvmlClocksEventReason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index: int):
        self.idx, self.rows, self.proc, self.nvml = gpu_index, [], None, None
        self.t0 = self.t1 = None
        self.stop_evt = threading.Event()

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = None
            try:   # the CUDA device's own GPU: NVML indices ignore CUDA_VISIBLE_DEVICES
                import torch
                h = N.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(self.idx).uuid))
            except Exception:
                h = N.nvmlDeviceGetHandleByIndex(self.idx)
            self.nvml = (N, h)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def mark(self):
        self.t0 = time.monotonic()

    def stop(self):
        self.t1 = time.monotonic()

    def _poll(self):
        N, h = self.nvml
        get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            N.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_evt.is_set():
            try:
                t = time.monotonic()
                self.rows.append((t, float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)), int(get_reasons(h))))
            except Exception:
                pass
            time.sleep(0.005)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append((time.monotonic(), parts))

    def __exit__(self, *a):
        self.stop_evt.set()
        if self.nvml:
            self.t.join(1)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()

    def _window(self):
        t0 = self.t0 if self.t0 is not None else -1e30
        t1 = self.t1 if self.t1 is not None else 1e30
        inside = [r for r in self.rows if t0 <= r[0] <= t1]
        return inside or self.rows[-1:]

    def summary(self):
        rows = self._window() if self.rows else []
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        if self.nvml:
            sm = [r[1] for r in rows]
            reasons = sorted({k for r in rows for k, b in self.BITS.items() if r[2] & b})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.max_mhz), "reasons": reasons,
                    "samples": len(rows), "source": "nvml 5 ms"}
        rows = [r[1] for r in rows]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi 100 ms"}


# ---------------------------------------------------------------------------
# CPU: the reference's decode kernel on the host cores
# ---------------------------------------------------------------------------
def cpu_decode_sample(n_tokens: float, threads: int):
    """Time the reference CPU path's matvec work for n_tokens decode steps of
    the 8B shape: vbs_cpu requantizes K-quants to Q8_0 at load
    (src/vbs_cpu.c:312-346) and runs every projection through the hot-kernel
    table's matvec_q8_0 (src/hotkernels/vbs_hot_ref_impl.h:49-64), >97% of
    its per-token time. The kernel (the reference's own code from
    oracle/_ref when built, else the oracle's bit-identical port) streams a
    14336 x 4096 Q8_0 matrix in row shards, one shard per thread, as many
    times as a token's 7.50 G weights require. Returns (tokens/s, kind)."""
    import ctypes as C
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    R = orc.ref()
    if R is not None:
        fn, kind = R.ref_hot_matvec_q8_0, "reference"
    else:
        fn, kind = orc.lib().orc_cpu_matvec_q8_0, "port"
    rows, cols = 14336, 4096
    rng = np.random.default_rng(0)
    w = rng.integers(-127, 128, size=(rows, cols // 32, 34), dtype=np.int16).astype(np.int8).view(np.uint8)
    w[:, :, 0] = 0x00
    w[:, :, 1] = 0x1C       # fp16 scale 2^-8
    w = np.ascontiguousarray(w.reshape(-1))
    xq = rng.integers(-127, 128, size=cols, dtype=np.int8)
    qd = np.full(cols // 32, 0.01, np.float32)
    y = np.empty(rows, np.float32)
    weights_per_token = L8B_WEIGHTS
    passes = max(1, round(n_tokens * weights_per_token / (rows * cols)))
    shard = (rows + threads - 1) // threads
    rb = cols // 32 * 34

    def work(i):
        r0 = i * shard
        n = min(shard, rows - r0)
        if n > 0:
            fn(C.c_void_p(w.ctypes.data + r0 * rb), n, cols, orc.ptr(xq), orc.ptr(qd),
               C.c_void_p(y.ctypes.data + r0 * 4))

    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, range(threads)))          # warm-up pass
        t0 = time.perf_counter()
        for _ in range(passes):
            list(ex.map(work, range(threads)))
        dt = time.perf_counter() - t0
    tokens = passes * rows * cols / weights_per_token
    return tokens / dt, kind, passes


def write_l8b_gguf(path, model=None, n_layers: int = 32) -> None:
    """The bench's 8B-shaped model (seed 2024) as a GGUF file for the
    reference CPU path. From the device model's bytes when one is given
    (the synthesizers are bit-identical), else synthesized on the host
    cores."""
    import models
    cfg = dict(models.L8B, n_layers=n_layers)
    if model is not None:
        host = models.host_model_from_device(cfg, model).t
    else:
        host = models.host_tensors_parallel(cfg, models.L8B_TYPES, 2024)
    models.write_model_gguf(path, cfg, host, context_length=8192)


def ref_cpu_decode(gguf, n_prompt: int, n_warm: int, n_steps: int) -> dict:
    """Greedy decode through the reference's own CPU inference path,
    vbs_cpu_step_ex (src/vbs_cpu.c:572-639), as its vbs-cpu CLI runs it
    (src/vbs_cpu_main.c:70-86): load (K-quants requantized to Q8_0,
    src/vbs_cpu.c:312-346), an n_prompt-token prompt, n_warm untimed decode
    tokens, then n_steps timed decode tokens, each a full step with its
    logits and the first-maximum argmax. One host thread, as the reference
    runs (src/vbs_hotpath.c:3-5)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import models
    import oracle as orc
    t0 = time.perf_counter()
    cpu = orc.RefCpu(gguf, n_prompt + n_warm + n_steps + 1)
    t1 = time.perf_counter()
    prompt = models.splitmix_ints(4096, n_prompt, models.L8B["vocab"])
    for i, t in enumerate(prompt):
        cpu.step(t, i + 1 == len(prompt))
    t2 = time.perf_counter()
    tok = cpu.argmax()
    for _ in range(n_warm):
        cpu.step(tok)
        tok = cpu.argmax()
    t3 = time.perf_counter()
    for _ in range(n_steps):
        cpu.step(tok)
        tok = cpu.argmax()
    t4 = time.perf_counter()
    cpu.close()
    return {"tok_s": n_steps / (t4 - t3), "load_s": t1 - t0, "prompt_s": t2 - t1, "timed_s": t4 - t3,
            "position": n_prompt + n_warm}


def ref_cpu_tiny() -> dict:
    """BASELINE config 0 end to end through the reference CPU path: the tiny
    GGUF, its 16 seeded prompt tokens, 64 greedy tokens (the golden run)."""
    import tempfile
    sys.path.insert(0, str(ROOT / "oracle"))
    import models
    import oracle as orc
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "tiny.gguf"
        models.make_tiny_gguf(path)
        t0 = time.perf_counter()
        cpu = orc.RefCpu(path, 128)
        prompt = models.tiny_prompt()
        for i, t in enumerate(prompt):
            cpu.step(t, i + 1 == len(prompt))
        out = []
        for i in range(models.N_NEW):
            out.append(cpu.argmax())
            if i + 1 < models.N_NEW:
                cpu.step(out[-1])
        s = time.perf_counter() - t0
        cpu.close()
    golden = json.loads((ROOT / "tests" / "golden" / "tiny_greedy.json").read_text())
    return {"tok_s": (models.N_PROMPT + models.N_NEW - 1) / s, "s": round(s, 4),
            "tokens_match_golden": out == golden["generated"]}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


REF_PROMPT = 16   # prompt tokens before the reference path's timed decode steps


def reference_arm(args, rank):
    """--impl reference: the reference's own CPU decode path (vbs_cpu, from
    oracle/_ref, compiled from the reference's sources) on the 8B-shaped
    model, one decode token per step."""
    if rank != 0:
        return
    import tempfile
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    threads = os.cpu_count() or 1
    if orc.ref() is None:
        # the reference was not compiled here: its hot kernel's port over
        # one token's matvec work per step (the oracle's restatement)
        tok_s, kind, passes = cpu_decode_sample(max(1, args.steps) * 0.25, threads)
        sample = f"{passes} passes of the ported matvec_q8_0 over a 14336x4096 Q8_0 matrix, row-sharded"
        workload, cores, extra = "llama3-8b-shape decode matvec work, ported reference kernel", threads, {}
    else:
        with tempfile.TemporaryDirectory() as td:
            path = Path(td) / "l8b.gguf"
            write_l8b_gguf(path, n_layers=args.ref_layers)
            r = ref_cpu_decode(path, REF_PROMPT, min(args.warmup, 2), args.steps)
        tok_s, kind, cores = r["tok_s"], "reference", 1
        sample = (f"{args.steps} greedy decode steps of vbs_cpu_step_ex (the reference's CPU path) on the 8B-shaped "
                  f"GGUF at positions {r['position']}..{r['position'] + args.steps - 1}, after a {REF_PROMPT}-token "
                  f"prompt and {min(args.warmup, 2)} untimed steps (a 4096-token CPU prefill would take hours); "
                  f"load {r['load_s']:.0f} s")
        workload = (f"llama3-8b-shape decode ({args.ref_layers}L, dim 4096, 32/8 heads, ffn 14336, vocab 128256; "
                    "Q4_K attn+gate/up, Q6_K down/output/embd), reference vbs-cpu path (vbs_cpu_step_ex)")
        extra = {"tiny_e2e": ref_cpu_tiny()}
    line = {
        "impl": "reference", "metric": "decode tokens/s, Llama-3-8B Q4_K shape", "value": round(tok_s, 4),
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / tok_s, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8-dot/f32 (Q8_0 requant)", "data": "synthetic",
        "config": {"workload": workload, "ctx": REF_PROMPT if kind == "reference" else args.ctx, "batch": 1,
                   "parallelism": f"{cores} host thread(s) of {threads}", "cpu_model": cpu_model(), **extra},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if args.profile:
        profile_kernel(args)
        return

    import numpy as np
    import torch
    import models
    import vbs_b200 as vbs

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    if not vbs.ops().init():
        raise SystemExit(f"backend init failed: {vbs.last_error()}")
    if world > 1:
        import ctypes as C
        idb = (C.c_uint8 * 128)()
        if rank == 0:
            vbs.check(vbs.lib().vbs_cu_tp_unique_id(idb), "tp unique id")
        obj = [bytes(idb)]
        dist.broadcast_object_list(obj, src=0)
        idb = (C.c_uint8 * 128).from_buffer_copy(obj[0])
        vbs.check(vbs.lib().vbs_cu_tp_init(rank, world, idb), "tp init")

    shape = models.shape_of(models.L8B)
    model = vbs.synth_llama(shape, models.L8B_TYPES, seed=2024, tp_rank=rank, tp_world=world)
    torch.cuda.synchronize()
    max_ctx = args.ctx + args.warmup + args.steps + args.e2e_steps + 8
    dec = vbs.Decoder(model, max_ctx)
    kps = dec.kernels_per_step
    prompt = models.splitmix_ints(4096, args.ctx, shape.vocab)
    # the context: one GPU takes the batched prefill (chunks of 512 tokens
    # per pass over the weights), tensor parallelism one token per step like
    # the engine; either way the timed steps below start at position ctx
    prefill_mode = "token-by-token"
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if world == 1:
        try:
            dec.prefill(prompt)
            prefill_mode = "batched"
        except vbs.VbsError as e:
            print(f"batched prefill failed ({e}); feeding the prompt token by token", file=sys.stderr)
            vbs.clear_error()
            dec.reset()
    if prefill_mode != "batched":
        dec.forward(prompt, logits=False)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    stream = torch.cuda.ExternalStream(dec.stream)
    # Under tensor parallelism the last warm-up step is enqueued after the
    # barrier, just before the start event: it cannot finish on any rank
    # before every rank's exchange words arrived, so it lines the ranks up
    # on the device and the host-side skew of their launches stays out of
    # the timed steps.
    aligned = 1 if dist and args.warmup > 0 else 0
    dec.enqueue_steps(args.warmup - aligned)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = vbs.kernel_launches()
    with ClockSampler(local) as clk:
        time.sleep(0.3)
        torch.cuda.synchronize()
        clk.mark()
        if aligned:
            dec.enqueue_steps(1)
        ev0.record(stream)
        dec.enqueue_steps(args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.stop()
    launches = vbs.kernel_launches() - l0 - aligned * dec.kernels_per_step
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / args.steps
    tok_s = 1000.0 / ms_step
    ctx_mid = args.ctx + args.warmup + args.steps / 2

    # e2e: the reference-facing call (verum_forward's contract): host token
    # array in pinned memory -> device, one step, logits -> host, per step.
    tok_pinned = torch.empty(args.e2e_steps, dtype=torch.int32, pin_memory=True)
    tok_pinned.copy_(torch.tensor(models.splitmix_ints(99, args.e2e_steps, shape.vocab), dtype=torch.int32))
    logits_host = np.empty(shape.vocab, np.float32)
    import ctypes as C
    tp_ptr = C.cast(C.c_void_p(tok_pinned.data_ptr()), C.POINTER(C.c_uint32))
    lp = logits_host.ctypes.data_as(C.POINTER(C.c_float))
    dec.forward_into(tp_ptr, 1, lp)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(1, args.e2e_steps):
        dec.forward_into(C.cast(C.c_void_p(tok_pinned.data_ptr() + 4 * i), C.POINTER(C.c_uint32)), 1, lp)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_tok_s = (args.e2e_steps - 1) / e2e_s

    # roofline of the dominant kernel. One GPU: the persistent step kernel
    # is the whole step (one launch per token, timed above on its stream);
    # its algorithmic bytes are the step's weights + KV. Otherwise (the
    # per-op kernels under TP): fused norm + gate/up + SiLU, two Q4_K
    # [14336 x 4096] per layer (66 MB), timed live over all 32 layers'
    # weights (2.1 GB, so no launch finds its weights in L2).
    peak, peak_kind = peaks()
    roof = None
    step_bytes = L8B_WEIGHT_BYTES + KV_BYTES_PER_POS * ctx_mid

    def committed_traffic(name):
        # DRAM bytes of one launch (dram__bytes_read.sum + dram__bytes_write.sum)
        # from the committed ncu summary of that kernel
        tf = ROOT / "profiles" / name
        if tf.exists():
            import re
            mt = re.search(r"dram_bytes_per_launch:\s*(\d+)", tf.read_text())
            return int(mt.group(1)) if mt else None
        return None

    if world == 1 and kps == 1:
        achieved = step_bytes / (ms_step * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "step_kernel (persistent decode step: every op of a token, one launch)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_kind": peak_kind, "traffic": committed_traffic("step_kernel_decode_l8b_ctx4096.md"),
                "algorithmic_bytes": int(step_bytes), "launch_us": round(ms_step * 1e3, 2),
                "frac_of_8tbs": round(achieved / 8000.0, 4)}
    elif kps == 1:
        # tensor parallelism: each rank's step kernel streams its shard, 1/world
        # of the weights and of the KV rows (norm weights aside)
        achieved = step_bytes / world / (ms_step * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "step_kernel, tensor-parallel instance (per rank: its weight and KV shard)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_kind": peak_kind, "traffic": None, "algorithmic_bytes": int(step_bytes / world),
                "launch_us": round(ms_step * 1e3, 2), "frac_of_8tbs": round(achieved / 8000.0, 4),
                "per": "rank (the slowest rank's time)"}
    elif world == 1:
        x = torch.randn(shape.dim, device="cuda")
        h = torch.empty(shape.ffn, device="cuda")
        nrm = model.tensors["blk.0.ffn_norm"]
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            for l in range(2):
                vbs.ffn_gate_up(vbs.Q4_K, model.tensors[f"blk.{l}.ffn_gate"].data_ptr(),
                                model.tensors[f"blk.{l}.ffn_up"].data_ptr(), x.data_ptr(), nrm.data_ptr(), 1e-5,
                                h.data_ptr(), shape.ffn, shape.dim, st.cuda_stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for l in range(shape.n_layers):
                vbs.ffn_gate_up(vbs.Q4_K, model.tensors[f"blk.{l}.ffn_gate"].data_ptr(),
                                model.tensors[f"blk.{l}.ffn_up"].data_ptr(), x.data_ptr(), nrm.data_ptr(), 1e-5,
                                h.data_ptr(), shape.ffn, shape.dim, st.cuda_stream)
            e1.record(st)
        st.synchronize()
        k_ms = e0.elapsed_time(e1) / shape.n_layers
        alg = FFN_GATE_UP_BYTES + shape.dim * 4 + shape.ffn * 4
        achieved = alg / (k_ms * 1e-3) / 1e9
        traffic = committed_traffic("mv_fast_kernel_ffn_gate_up_q4k_8b.md")
        roof = {"bound": "hbm", "kernel": "mv_fast_kernel<Q4_K,dual,SILU> (norm+gate/up+SiLU)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_kind": peak_kind, "traffic": traffic, "algorithmic_bytes": alg, "launch_us": round(k_ms * 1e3, 2),
                "frac_of_8tbs": round(achieved / 8000.0, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as orc
        if orc.ref() is not None:
            import tempfile
            with tempfile.TemporaryDirectory() as td:
                path = Path(td) / "l8b.gguf"
                write_l8b_gguf(path, model)
                r = ref_cpu_decode(path, REF_PROMPT, 1, 8)
            cpu = {"value": round(r["tok_s"], 4), "unit": "tokens/s", "cores": 1, "kind": "reference",
                   "sample": f"8 greedy decode steps of the reference's vbs_cpu_step_ex on the same 8B-shaped model "
                             f"(GGUF of these weights; K-quants requantized to Q8_0 by the reference at load) at "
                             f"positions {r['position']}..{r['position'] + 7}, after a {REF_PROMPT}-token prompt; one "
                             f"host thread, as the reference runs; {cpu_model()}, {os.cpu_count()} host threads",
                   "timed_s": round(r["timed_s"], 2)}
        else:
            threads = os.cpu_count() or 1
            v, kind, passes = cpu_decode_sample(1.0, threads)
            cpu = {"value": round(v, 4), "unit": "tokens/s", "cores": threads, "kind": kind,
                   "sample": f"{passes} passes of the ported vbs_cpu hot kernel matvec_q8_0 over a 14336x4096 Q8_0 "
                             f"matrix = 1 token of 8B decode matvec work, row-sharded over {threads} threads"}
    if rank == 0:
        line = {
            "metric": "decode tokens/s, Llama-3-8B Q4_K shape", "value": round(tok_s, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-mma/f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized on device; seeded prompt ids)",
            "config": {"workload": "llama3-8b-shape decode (32L, dim 4096, 32/8 heads, ffn 14336, vocab 128256; "
                                   "Q4_K attn+gate/up, Q6_K down/output/embd)",
                       "ctx": args.ctx, "batch": 1, "parallelism": f"tp{world}" if world > 1 else "single",
                       "tp_sum": dec.tp_mode if world > 1 else None,
                       "l2": "inputs larger than L2 (4.84 GB weights per step)",
                       "kernels_per_step": kps, "prefill_s": round(prefill_s, 2), "prefill": prefill_mode,
                       "prefill_tok_s": round(args.ctx / prefill_s, 1)},
            "step_bandwidth": {"algorithmic_bytes": int(step_bytes),
                               "achieved_gbs": round(step_bytes * tok_s / 1e9, 1),
                               "frac_of_measured": round(step_bytes * tok_s / 1e9 / peak, 4),
                               "frac_of_8tbs": round(step_bytes * tok_s / 1e9 / 8000.0, 4)},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": shape.vocab * 4},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dec.close()
    if world > 1:
        vbs.lib().vbs_cu_tp_finalize()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
