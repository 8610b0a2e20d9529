"""Collective failure handling: a rank that never joins ends in an error, not a wait.

The failure is made on the host, never by faulting or hanging a GPU: rank 0
of a two-rank communicator calls fgt_comm_create and rank 1 never does. The
communicator is non-blocking with a deadline (FGT_COMM_TIMEOUT_MS), so rank 0
must get FGT_ERR_NCCL within about the deadline. The attempt runs in a child
process on one GPU, under its own timeout, with NVLS off; no kernel is launched
and nothing waits on the GPU.
"""
import os
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu

CHILD = textwrap.dedent("""
    import ctypes, sys, time
    sys.path.insert(0, %r)
    import torch
    torch.cuda.set_device(0)
    torch.zeros(1, device="cuda")
    from fugatensor_b200 import _fgt
    uid = _fgt.Comm.unique_id()
    t0 = time.time()
    try:
        _fgt.Comm(uid, 2, 0)
        print("RESULT joined")
    except _fgt.NCCLError as e:
        print("RESULT nccl_error %%.2f %%s" %% (time.time() - t0, str(e).replace(chr(10), " ")))
    except Exception as e:
        print("RESULT other %%s %%s" %% (type(e).__name__, e))
""" % str(ROOT))


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_rank_that_never_joins_times_out_with_nccl_error():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", FGT_COMM_TIMEOUT_MS="3000", PYTHONUNBUFFERED="1")
    t0 = time.time()
    proc = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", CHILD], cwd=ROOT, env=env,
                          capture_output=True, text=True)
    elapsed = time.time() - t0
    out = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT")]
    assert proc.returncode == 0 and out, proc.stdout[-2000:] + proc.stderr[-2000:]
    _, kind, rest = out[-1].split(" ", 2)
    assert kind == "nccl_error", out[-1]
    waited = float(rest.split(" ", 1)[0])
    assert 2.5 <= waited <= 30.0, out[-1]
    assert "timed out" in out[-1]
    assert elapsed < 110
