"""Direct file→device upload (vbs_cu_upload_file) on a B200: every byte of
every range lands at its destination whatever the thread count and chunk
size, a GGUF model uploads to the same bytes the file holds (plus the zero
tail padding the matvec kernels read past a row end), and bad ranges fail
with an error before anything is copied."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_upload_gguf_matches_file(vbs, gpu, tiny_gguf, clean_errors):
    import torch
    _, lay = vbs.gguf_layout(tiny_gguf)
    data = tiny_gguf.read_bytes()
    for n_threads in (1, 4):
        dm = vbs.upload_gguf(tiny_gguf, n_threads=n_threads)
        for key, t in dm.tensors.items():
            name = key + ".weight"
            if name not in lay:   # the output matrix shared with the embedding
                name = "token_embd.weight"
            g = lay[name]
            got = t.view(torch.uint8).cpu().numpy().tobytes()
            assert got[:g.nbytes] == data[g.offset:g.offset + g.nbytes], key
            assert not any(got[g.nbytes:]), key


@pytest.mark.parametrize("n_threads,chunk", [(1, 1 << 20), (3, 1 << 20), (8, 4 << 20), (0, 0)])
def test_upload_file_ranges(vbs, gpu, tmp_path, n_threads, chunk, clean_errors):
    import torch
    rng = np.random.default_rng(n_threads * 7 + 1)
    blob = rng.integers(0, 256, 23 * (1 << 20) + 12345, dtype=np.uint8)
    path = tmp_path / "blob.bin"
    path.write_bytes(blob.tobytes())
    # odd offsets and sizes, one empty range, one range to the last byte
    spec = [(0, 1), (7, 3 * (1 << 20) + 5), (5 << 20, 9 << 20), (blob.size - 777, 777), (123, 0),
            (17 << 20, (1 << 20) + 1)]
    bufs = [torch.full((max(s, 1) + 64,), 0xAB, dtype=torch.uint8, device="cuda") for _, s in spec]
    torch.cuda.synchronize()
    vbs.upload_file(path, [(o, s, b.data_ptr()) for (o, s), b in zip(spec, bufs)], n_threads, chunk)
    for (o, s), b in zip(spec, bufs):
        got = b.cpu().numpy()
        assert np.array_equal(got[:s], blob[o:o + s]), (o, s)
        assert (got[s:] == 0xAB).all(), (o, s)   # nothing past the range


def test_upload_file_rejects_bad_ranges(vbs, gpu, tmp_path, clean_errors):
    import torch
    path = tmp_path / "small.bin"
    path.write_bytes(bytes(range(256)) * 4)
    buf = torch.zeros(2048, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    # the library keeps the first error until it is cleared
    with pytest.raises(vbs.VbsError, match="outside"):
        vbs.upload_file(path, [(0, 16, buf.data_ptr()), (1000, 25, buf.data_ptr())])
    vbs.clear_error()
    with pytest.raises(vbs.VbsError, match="destination"):
        vbs.upload_file(path, [(0, 16, 0)])
    vbs.clear_error()
    with pytest.raises(vbs.VbsError, match="missing"):
        vbs.upload_file(tmp_path / "missing.bin", [(0, 1, buf.data_ptr())])
    assert not buf.cpu().numpy().any()   # nothing was copied
