"""N-sharded SDOT matrix on 2 GPUs (openneedle_b200/sharded.py): the all-gather
fused into the GEMM epilogue and the NCCL form both equal the single-GPU
result.  Needs two GPUs; skipped otherwise."""
import os
import signal
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.gpu
def test_two_gpu_sharded_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from openneedle_b200 import build
    build.build()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "tests" / "sharded_worker.py")]
    proc = subprocess.Popen(cmd, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                            start_new_session=True)
    try:
        out, _ = proc.communicate(timeout=300)
    except subprocess.TimeoutExpired:
        os.killpg(proc.pid, signal.SIGKILL)
        out, _ = proc.communicate()
        pytest.fail("two-GPU run timed out:\n" + out[-3000:])
    assert proc.returncode == 0 and "sharded ok" in out, out[-3000:]
