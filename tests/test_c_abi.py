"""The C ABI from a C host with no Python or torch in the process
(tests/c_abi/linear_split_check.c): it compiles and links against
include/dak_b200.h, libdak_b200.so and the CUDA runtime here, and on a GPU it
runs split linears on both kernel paths and checks them against a double
precision product (max relative error <= 1e-2)."""
import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import REPO

CUDA = Path("/usr/local/cuda")
SRC = REPO / "tests" / "c_abi" / "linear_split_check.c"


def _build(tmp_path: Path) -> Path:
    cc = shutil.which("gcc")
    if cc is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("no C compiler or CUDA headers")
    lib_dir = REPO / "directaccesskernel_b200"
    if not (lib_dir / "libdak_b200.so").exists():
        pytest.fail("libdak_b200.so is not built")
    exe = tmp_path / "linear_split_check"
    subprocess.run([cc, "-O2", "-I", str(REPO / "include"), "-I", str(CUDA / "include"), str(SRC),
                    "-L", str(lib_dir), "-ldak_b200", "-L", str(CUDA / "lib64"), "-lcudart", "-lm",
                    f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)], check=True)
    return exe


def test_c_host_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
def test_c_host_runs_the_split_linear(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok")
