"""Shared pytest setup. GPU tests carry @pytest.mark.gpu and run only on a
B200 box (`pytest -m gpu`); everything else runs on CPU."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def tiny_golden():
    return json.loads((GOLDEN / "tiny_greedy.json").read_text())


@pytest.fixture(scope="session")
def orc():
    import oracle
    if not oracle.LIB.exists():
        oracle.build(ref=False)
    return oracle


@pytest.fixture(scope="session")
def vbs():
    import vbs_b200
    if not vbs_b200.LIB_PATH.exists():
        vbs_b200.build()
    return vbs_b200


@pytest.fixture(scope="session")
def gpu(vbs):
    """The ops table, initialised on a B200. Fails (never skips) when the
    backend cannot come up: GPU tests must not pass on a fallback."""
    import torch
    assert torch.cuda.is_available(), "GPU test on a machine without CUDA"
    ops = vbs.ops()
    assert ops.init(), f"g_vbs_cuda_backend.init() failed: {vbs.last_error()}"
    return ops


@pytest.fixture()
def clean_errors(vbs):
    vbs.clear_error()
    yield
    vbs.clear_error()


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory, tiny_golden):
    import hashlib
    import models
    path = tmp_path_factory.mktemp("tiny") / "tiny.gguf"
    models.make_tiny_gguf(path)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == tiny_golden["gguf_sha256"], \
        "regenerated tiny model differs from the one the golden tokens were made with"
    return path
