"""The C ABI from plain C (tests/c/abi_from_c.c): include/tgcuda.h compiles as C11, libtgcuda.so
links, and the entry points that need no GPU give the reference's answers; on a machine without an
sm_100 GPU a context fails with TG_ENODEVICE rather than falling back."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_the_abi_works_from_c(pkg, tmp_path):
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    lib = pkg.LIB_PATH
    exe = tmp_path / "abi_from_c"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c" / "abi_from_c.c"), "-o", str(exe), f"-L{lib.parent}", "-ltgcuda",
                    f"-Wl,-rpath,{lib.parent}"], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, (res.returncode, res.stdout, res.stderr)
    assert res.stdout.strip().endswith("ok")
