"""The C ABI from a plain C program (no Python on the caller's side): compile
tests/c_client/fgt_client.c with gcc against include/fgt.h and libfgt.so, then
run it. It plans and specialises a softmax partition, reads info, ports and the
Execution Plan, and checks that invalid calls return statuses. No GPU needed."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

from fugatensor_b200 import _fgt

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_plain_c_caller(tmp_path):
    exe = tmp_path / "fgt_client"
    lib_dir = _fgt.LIB_PATH.parent
    subprocess.run(["gcc", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}", "-o", str(exe),
                    str(ROOT / "tests" / "c_client" / "fgt_client.c"), f"-L{lib_dir}", "-lfgt",
                    f"-Wl,-rpath,{lib_dir}"], check=True)
    env = dict(os.environ, FGT_CACHE_DIR=str(tmp_path / "cache"))
    out = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "ok"
