#!/usr/bin/env python3
"""Command-line entry of the bench (the reference's `./run.sh [flags]`).

    python mlp_bench.py [--N n --K k --M m --iters i --warmup w]
                        [--dtype <name|all>] [--tile <name>] [--suite]
                        [--autotune] [--no-profile]
                        [--gpus 1|2|4|8] [--allgather] [--data ref|seeded]
                        [--seed s] [--rotate r] [--flush]
    python mlp_bench.py --peak [--iters i]     (tensor-core peak per MMA kind)

With --gpus N > 1 launch it under torchrun (one process per GPU):
    torchrun --nproc-per-node N --master-addr 127.0.0.1 mlp_bench.py --gpus N ...
"""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                "fp8-mlp-metal41-bench_b200"))

from mlpgemm.driver import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())
