"""The reference's own backend self-test body run on this library.

oracle/_ref/cuda-backend-test is the reference's src/vbs_backend_test.c,
compiled unmodified (oracle/ref_backend_test.c includes it) and linked
against libvbs_b200.so in place of src/vbs_backend_cuda.c. Its
test_one_backend (src/vbs_backend_test.c:456-963) checks alloc/copy, every
primitive, linear tiles in both calling conventions and the quantized types
against the reference's own from-spec implementations; the reference runs
it for CPU, Vulkan and HIP and gives CUDA a smoke check only
(src/vbs_backend_test.c:1135-1147). Here every one of its checks must pass
on g_vbs_cuda_backend.
"""
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = ROOT / "oracle" / "_ref" / "cuda-backend-test"


def test_reference_backend_suite_on_cuda_table(gpu):
    assert BIN.exists(), "oracle/_ref/cuda-backend-test was not built (make -C oracle ref-backend-test)"
    out = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=600)
    text = out.stdout
    fails = [ln for ln in text.splitlines() if "[FAIL]" in ln]
    summary = [ln for ln in text.splitlines() if ln.startswith("cuda backend suite:")]
    assert out.returncode == 0 and not fails, "\n".join(fails) or text[-3000:] + out.stderr[-2000:]
    assert summary and summary[0].endswith(" 0 failures"), text[-2000:]
    n = int(summary[0].split(":")[1].split()[0])
    assert n >= 33, summary[0]   # the CPU table runs 33 checks of this suite (verum-slice --backend-test)
