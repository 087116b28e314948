"""Sharded engine on several GPUs (gpu; needs >= 2 devices).

Runs tests/mp_shard_worker.py under torchrun with NCCL, one process per GPU
on up to 8 GPUs of the box, and requires every rank's outputs to agree with
the fp64 CPU oracle on sampled rows (column-parallel layer, MLP and gated
FFN with the overlapped NVLink reduction and with NCCL, the NCCL fallback
for rows that do not split over the ranks, and output ownership).
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

WORKER = Path(__file__).resolve().parent / "mp_shard_worker.py"


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_sharded_engine_matches_oracle():
    n = min(torch.cuda.device_count(), 8)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(WORKER)]
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "0"))
    proc = subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True,
                          env=env)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    print(proc.stdout[-3000:])
