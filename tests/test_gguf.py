"""The GGUF header parser behind the direct upload (no GPU): tensor offsets
and metadata, including the array-valued keys real model files carry
(src/vbs_gguf.c reads the same container), checked against the writer and
against the oracle's independent reader. The upload entry point itself
reports a missing device instead of touching one."""
import numpy as np
import pytest

import models


def test_layout_offsets_match_oracle_reader(vbs, orc, tiny_gguf):
    meta, lay = vbs.gguf_layout(tiny_gguf)
    hm = orc.load_gguf_host(tiny_gguf)
    data = tiny_gguf.read_bytes()
    assert int(meta["llama.block_count"]) == hm.cfg["n_layers"]
    for name, t in lay.items():
        key = name[:-len(".weight")] if name.endswith(".weight") else name
        ty, rows, cols, arr = hm.t[key]
        assert (t.type, t.dims[0]) == (ty, cols)
        assert data[t.offset:t.offset + t.nbytes] == arr.view(np.uint8).tobytes(), name
    _, tens = vbs.read_gguf(tiny_gguf)
    assert all(tens[k][2] == data[t.offset:t.offset + t.nbytes] for k, t in lay.items())


def test_layout_reads_arrays_alignment_and_types(vbs, tmp_path):
    rng = np.random.default_rng(3)
    blobs = {"a.weight": (vbs.Q4_K, (512, 3), rng.integers(0, 256, 3 * 2 * 144, dtype=np.uint8).tobytes()),
             "b.weight": (vbs.F32, (7,), rng.standard_normal(7).astype(np.float32).tobytes()),
             "c.weight": (vbs.Q6_K, (256, 5), rng.integers(0, 256, 5 * 210, dtype=np.uint8).tobytes()),
             "d.weight": (vbs.Q8_0, (64, 2), rng.integers(0, 256, 2 * 2 * 34, dtype=np.uint8).tobytes())}
    meta = {"general.alignment": 64, "general.architecture": "llama",
            "tokenizer.ggml.tokens": ["<s>", "</s>", "hello", ""], "tokenizer.ggml.token_type": [1, 3, 1, 1],
            "tokenizer.ggml.scores": [0.0, -1.5, 2.25, 0.5], "llama.context_length": 8192, "x.f": 0.5}
    path = tmp_path / "m.gguf"
    vbs.write_gguf(path, meta, [(k, t, d, b) for k, (t, d, b) in blobs.items()], alignment=64)
    got, lay = vbs.gguf_layout(path)
    assert got["tokenizer.ggml.tokens"] == meta["tokenizer.ggml.tokens"]
    assert got["tokenizer.ggml.token_type"] == meta["tokenizer.ggml.token_type"]
    assert got["tokenizer.ggml.scores"] == pytest.approx(meta["tokenizer.ggml.scores"])
    assert got["llama.context_length"] == 8192 and got["general.architecture"] == "llama"
    data = path.read_bytes()
    for k, (t, d, b) in blobs.items():
        g = lay[k]
        assert (g.type, g.dims, g.nbytes) == (t, d, len(b))
        assert g.offset % 64 == 0
        assert data[g.offset:g.offset + g.nbytes] == b


def test_layout_reads_only_the_header(vbs, tmp_path):
    """A file cut right after its header still yields the layout; reading
    the tensors from it fails."""
    path = tmp_path / "m.gguf"
    b = bytes(range(256)) * 9
    vbs.write_gguf(path, {"k": 1}, [("t.weight", vbs.Q8_0, (32, 64), b[:64 * 34])])
    _, lay = vbs.gguf_layout(path)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(path.read_bytes()[:lay["t.weight"].offset])
    _, lay2 = vbs.gguf_layout(cut)
    assert lay2["t.weight"].offset == lay["t.weight"].offset
    with pytest.raises(ValueError):
        vbs.read_gguf(cut)


def test_layout_rejects_bad_files(vbs, tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"GGUF\x02\x00\x00\x00" + bytes(16))
    with pytest.raises(ValueError):
        vbs.gguf_layout(p)
    p.write_bytes(b"GGUF\x03\x00\x00\x00")
    with pytest.raises(ValueError):
        vbs.gguf_layout(p)


def test_upload_without_gpu_reports_reason(vbs, tiny_gguf):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(vbs.VbsError):
        vbs.upload_file(tiny_gguf, [(0, 16, 1 << 40)])
    assert "device" in vbs.last_error()
