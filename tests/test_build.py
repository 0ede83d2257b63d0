"""CPU checks of the native build: the sm_100a library compiles, loads without a GPU and
exports every entry point that include/llx.h declares; the compiled-in LUTs equal the
reference tables."""
from __future__ import annotations

import ctypes
import json
import re
import subprocess
import sys

import pytest

from conftest import GOLDEN, REPO


@pytest.fixture(scope="module")
def lib_path():
    from llaccel_b200 import build
    return build.build()


def declared_functions() -> list[str]:
    text = (REPO / "include" / "llx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llx_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib_path):
    lib = ctypes.CDLL(str(lib_path))
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    nm = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True).stdout
    for n in names:
        assert re.search(rf"\bT {n}\b", nm), n


def test_python_binding_covers_the_header(lib_path):
    from llaccel_b200 import cuda_backend
    assert sorted(cuda_backend.SIGNATURES) == declared_functions()
    lib = cuda_backend.load_library(lib_path)
    assert lib.llx_version().decode().startswith("llx")


def test_library_is_built_for_sm100a_only(lib_path):
    """The build targets sm_100a alone (no PTX, no other architecture).  The GPU test
    test_gpu_parity.py::test_kernels_are_sm100_binaries checks what the runtime loads."""
    from llaccel_b200 import build
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_lut_header_matches_reference_tables():
    sys.path.insert(0, str(REPO / "llaccel_b200" / "csrc"))
    import gen_luts
    ref = json.loads((GOLDEN / "luts.json").read_text())
    sig, expi, expf = gen_luts.tables()
    assert sig == ref["SIG"] and expi == ref["EXPI"] and expf == ref["EXPF"]
    assert (REPO / "llaccel_b200" / "csrc" / "luts_data.h").read_text() == gen_luts.render()


def test_model_load_without_gpu_fails_cleanly(lib_path):
    """No CUDA device here: loading must fail with a CUDA error code, never fall back."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from llaccel_b200 import cuda_backend
    with pytest.raises((cuda_backend.LlxError, ValueError)):
        cuda_backend.CudaModel(GOLDEN / "fx_v1")
