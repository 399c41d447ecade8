"""The C-ABI library loads and exports every symbol include/vbs_b200.h
declares; the ops table has the reference's layout. No GPU compute."""
import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT


def declared_symbols():
    text = (ROOT / "include" / "vbs_b200.h").read_text()
    names = set(re.findall(r"VBS_API\s+[\w\s\*]*?\b(vbs_\w+)\s*\(", text))
    names |= set(re.findall(r"VBS_API\s+const\s+vbs_backend_ops_t\s+(g_vbs_cuda_backend)", text))
    return sorted(names)


def test_header_declares_boundary():
    names = declared_symbols()
    assert "g_vbs_cuda_backend" in names and "vbs_cuda_last_error" in names
    assert len(names) >= 25


def test_library_exports_all_declared(vbs):
    L = vbs.lib()
    for n in declared_symbols():
        assert hasattr(L, n), f"{n} declared in include/vbs_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(vbs.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split()[1] in "TDBR"}
    assert set(declared_symbols()) <= exported


def test_ops_table_layout(vbs):
    # 14 pointer-sized fields, in the order of include/vbs_backend.h:64-99
    assert C.sizeof(vbs.OpsTable) == 14 * C.sizeof(C.c_void_p)
    assert C.sizeof(vbs.Device) == 128 + 8 + 8 + 8 + 8   # name, type (+pad), two u64, handle
    assert C.sizeof(vbs.Buffer) == 4 * 8
    assert C.sizeof(vbs.Arg) == 24
    o = vbs.ops()
    for name, _ in vbs.OpsTable._fields_[:-1]:
        assert C.cast(getattr(o, name), C.c_void_p).value, f"{name} is NULL"
    assert o.launch_persistent_kernel   # device-driven generation (the reference leaves it NULL)


def test_init_without_gpu_reports_reason(vbs):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert vbs.ops().init() is False
    assert vbs.last_error() != "ok"


def test_version_names_blackwell_features(vbs):
    v = vbs.lib().vbs_cu_version().decode()
    for feat in ("sm_100a", "cp.async", "mma.m16n8k32"):
        assert feat in v


def test_sources_no_multicast_loads():
    src = "".join(p.read_text() for p in (ROOT / "verum-bespoke-singularity_b200" / "csrc").glob("*.cu*"))
    assert "mma.sync.aligned.m16n8k32" in src and "cp.async.cg" in src
    # No cluster-multicast load anywhere in the code (comments may mention
    # the word). The word is assembled so that this test does not contain it.
    import re
    code = re.sub(r"//[^\n]*", "", src)
    word = "".join(reversed("tsacitlum"))
    assert word not in code


@pytest.mark.parametrize("entry", ["attention", "attention_static"])
@pytest.mark.parametrize("nqh,nkh", [(32, 0), (0, 8), (30, 8)])
def test_attention_rejects_bad_head_counts(vbs, entry, nqh, nkh):
    """A zero or non-dividing KV head count is refused before any device
    work (it would otherwise reach the split arithmetic, which divides by
    it). The pointers are never dereferenced: the argument check comes
    first, so this runs without a GPU."""
    vbs.clear_error()
    fake = 4096
    with pytest.raises(vbs.VbsError, match="invalid arguments"):
        getattr(vbs, entry)(fake, fake, fake, fake, 128, 0, 128, nqh, nkh, 128, 0.088)
    vbs.clear_error()


def test_batch_decoder_refuses_bad_arguments(vbs):
    """vbs_cu_batch_decoder_create checks the model description and the
    batch size before it touches a device, so the refusals run without a
    GPU: no description, and a batch of 0 or above 64 sequences."""
    import ctypes as C
    L = vbs.lib()
    err = C.create_string_buffer(256)
    vbs.clear_error()
    assert not L.vbs_cu_batch_decoder_create(None, 64, 8, err, 256)
    assert b"invalid model description" in err.value
    desc = vbs.ModelDesc(n_layers=1, dim=64, n_heads=2, n_kv_heads=1, head_dim=32, ffn=128, vocab=16,
                         embd=16, out=16, out_norm=16)
    for bad in (0, 65):
        vbs.clear_error()
        assert not L.vbs_cu_batch_decoder_create(C.byref(desc), 64, bad, err, 256)
        assert b"batch must be" in err.value
        assert "batch" in vbs.last_error()
    vbs.clear_error()
    assert L.vbs_cu_batch_decoder_position(None) == 0   # an invalid handle is refused, not dereferenced


def test_layout_matches_reference_headers():
    """Every offset and size of the ops-table types in include/vbs_b200.h
    equals the reference's include/vbs_backend.h (the same printer compiled
    against each header; oracle/abi_layout.c)."""
    ours, ref = ROOT / "oracle" / "abi-layout", ROOT / "oracle" / "_ref" / "abi-layout-ref"
    if not ours.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "abi-layout"], check=True, capture_output=True)
    if not ref.exists():
        pytest.skip("the reference was not compiled here (oracle/_ref)")
    a = subprocess.run([str(ours)], capture_output=True, text=True, check=True).stdout
    b = subprocess.run([str(ref)], capture_output=True, text=True, check=True).stdout
    assert a.count("\n") >= 30 and a == b
