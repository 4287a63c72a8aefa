"""The C ABI from a plain C11 host (tests/c_abi_host.c): the header compiles as C with warnings
as errors and the program links against libmoe_b200.so (CPU); on a GPU it runs a layer, routing,
forwards at M = 1 and 64, the LM head and the error path (GPU)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIBDIR = ROOT / "moe-680m_b200" / "lib"
CC = shutil.which("cc") or shutil.which("gcc")


@pytest.fixture(scope="module")
def host_binary(tmp_path_factory):
    if CC is None:
        pytest.skip("no C compiler")
    if not (LIBDIR / "libmoe_b200.so").exists():
        pytest.fail("libmoe_b200.so is not built (python moe-680m_b200/build.py)")
    out = tmp_path_factory.mktemp("chost") / "c_abi_host"
    cmd = [CC, "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "c_abi_host.c"), "-L", str(LIBDIR), "-lmoe_b200", "-lm", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return out


def test_c_host_compiles_and_links(host_binary):
    assert host_binary.exists()


@pytest.mark.gpu
def test_c_host_runs(host_binary):
    env = dict(os.environ, LD_LIBRARY_PATH=f"{LIBDIR}:{os.environ.get('LD_LIBRARY_PATH', '')}")
    r = subprocess.run([str(host_binary)], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and "c host ok" in r.stdout, r.stdout + r.stderr
