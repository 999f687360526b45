"""One rank of the multi-GPU check of openneedle_b200.sharded (started by
tests/test_gpu_sharded.py through torch.distributed.run, one process per GPU).
Every rank's fused-epilogue and NCCL all-gather outputs must equal the
single-GPU result bit for bit (GEMM for batches >= 64, GEMV below)."""
import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from openneedle_b200.native import DeviceMatrix  # noqa: E402
from util import synthetic_matrix  # noqa: E402
from openneedle_b200.sharded import ShardedSdot  # noqa: E402


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank = dist.get_rank()
    ok = True
    for out, k, bits in ((1000, 512, 4), (2048, 1024, 2)):
        packed, norms, cb = synthetic_matrix(out, k, bits, 128, seed=5)
        full = DeviceMatrix(packed, norms, (out, k), bits, 128, cb)
        sh = ShardedSdot(packed, norms, (out, k), bits, 128, cb, max_batch=130)
        for m in (16, 64, 130):
            x = np.random.default_rng(m).normal(size=(m, k)).astype(np.float32)
            ref = full.sdot(x)
            xd = torch.from_numpy(x).cuda()
            y_fused = sh.forward(xd).cpu().numpy()
            y_nccl = sh.forward_nccl(xd).cpu().numpy()
            good = np.array_equal(y_fused, ref) and np.array_equal(y_nccl, ref)
            if not good:
                print(f"rank {rank}: mismatch out={out} k={k} bits={bits} m={m} "
                      f"fused {np.abs(y_fused - ref).max()} nccl {np.abs(y_nccl - ref).max()}", flush=True)
            ok = ok and good
        # back-to-back calls while a peer still reads the first output: rank 1
        # stalls its stream before copying its view of call 1, rank 0 issues
        # call 2 at once; the barrier before each GEMM keeps call 2's peer
        # stores out of rank 1's buffer until rank 1's copy has run
        m = 64
        x1 = np.random.default_rng(11).normal(size=(m, k)).astype(np.float32)
        x2 = np.random.default_rng(12).normal(size=(m, k)).astype(np.float32)
        y1 = sh.forward(torch.from_numpy(x1).cuda())
        if rank == 1:
            torch.cuda._sleep(200_000_000)
        first = y1.clone()
        y2 = sh.forward(torch.from_numpy(x2).cuda())
        good = (np.array_equal(first.cpu().numpy(), full.sdot(x1)) and
                np.array_equal(y2.cpu().numpy(), full.sdot(x2)))
        if not good:
            print(f"rank {rank}: back-to-back forward calls raced (out={out})", flush=True)
        ok = ok and good
        sh.close()
    flag = torch.tensor([1.0 if ok else 0.0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    all_ok = flag.item() == 1.0
    dist.destroy_process_group()
    if rank == 0:
        print("sharded ok" if all_ok else "sharded MISMATCH", flush=True)
    return 0 if all_ok else 1


if __name__ == "__main__":
    sys.exit(main())
