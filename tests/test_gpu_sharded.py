"""Sharded execution on 2 GPUs (skipped when fewer are visible)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_two_rank_sharded_partitions_match_global_oracle(exchange):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONUNBUFFERED="1", FGT_EXCHANGE_WAIT_MS="1500",
               FGT_PEER_EXCHANGE="1" if exchange == "peer" else "0", FGT_TEST_EXCHANGE_TIMEOUT="1")
    port = 29531 if exchange == "peer" else 29533
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(ROOT / "tests" / "sharded_worker.py")]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert proc.stdout.count("ok (") == 10
    assert proc.stdout.count(f"exchange path {exchange}") == 2, proc.stdout[-2000:]
    if exchange == "peer":
        assert "exchange timeout reported" in proc.stdout
