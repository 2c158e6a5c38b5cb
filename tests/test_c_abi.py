"""The C ABI from a plain C program (tests/c/abi_smoke.c): it compiles against include/emugen.h and
links libemugen.so on any machine; it runs on a GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
CUDA = Path("/usr/local/cuda")


def _build(tmp_path) -> Path:
    if shutil.which("gcc") is None or not (CUDA / "include" / "cuda_runtime.h").is_file():
        pytest.skip("gcc or the CUDA headers are not available")
    lib = REPO / "emugen_b200" / "libemugen.so"
    if not lib.is_file():
        pytest.skip("libemugen.so is not built")
    exe = tmp_path / "abi_smoke"
    cmd = ["gcc", "-std=c11", "-O1", "-Wall", "-Werror", str(REPO / "tests" / "c" / "abi_smoke.c"), "-I",
           str(REPO / "include"), "-I", str(CUDA / "include"), "-L", str(lib.parent), "-lemugen",
           "-Wl,-rpath," + str(lib.parent), "-L", str(CUDA / "lib64"), "-lcudart", "-Wl,-rpath," + str(CUDA / "lib64"),
           "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_program_compiles_and_links(tmp_path):
    assert _build(tmp_path).is_file()


@pytest.mark.gpu
def test_c_program_runs(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "c abi ok" in r.stdout
