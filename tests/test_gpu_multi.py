"""Multi-GPU runs of the sharded CLI (two ranks under torchrun, NCCL).

The N-sharded run with --allgather gathers Y three ways: NCCL in place, the
4-round pipeline, and the fused GEMM + all-gather (gemm_run_gather over
IPC-mapped peer buffers). The CLI exits 3 unless each of them leaves exactly
the NCCL-gathered Y on every GPU and the sample points match the oracle's
dot products. Skipped on hosts with fewer than two GPUs.
"""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shard,shape", [("n", (512, 1024, 2048)), ("n", (300, 512, 1040)),
                                         ("m", (512, 1024, 2048))])
def test_two_rank_sharded_gather(shard, shape):
    N, K, M = shape
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), "mlp_bench.py", "--gpus", "2",
           "--shard", shard, "--allgather", "--N", str(N), "--K", str(K), "--M", str(M), "--iters", "3",
           "--warmup", "1", "--dtype", "all"]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.rstrip().endswith("ok")
    if shard == "n":
        # every dtype's default tile here has the fused gather: its column is a time
        rows = [l for l in r.stdout.splitlines() if l.startswith("custom") and "r " in l]
        assert rows and all(not l.rstrip().endswith("-") for l in rows), r.stdout
