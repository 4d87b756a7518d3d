"""Tensor-parallel decode on 2 GPUs (g4b.tp), when the box has them.

Runs tests/tp_worker.py under torch.distributed.run with 2 ranks: every rank
streams its column / row shards of a 2-layer stack with g4b_gemv_i4 and two
NCCL all-reduces per layer, rank 0 compares the gathered logits with the
unsharded chain on its own GPU (f32 summation order only: tests/util.py bar)
and checks that a CUDA-graph replay of the step reproduces them exactly.
Skipped on a one-GPU box (the round-end suite runs on one GPU).
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("fp8,allreduce", [(False, "nccl"), (True, "nccl"), (False, "peer"), (False, "chain"),
                                           (True, "chain")])
def test_tp_decode_two_gpus(fp8, allreduce):
    """allreduce="peer" also checks g4b_allreduce_f32 on its own: identical bits
    on both ranks, equal to NCCL's sum, across repeated calls.  allreduce="chain"
    runs each rank's token as one GEMV chain with the all-reduces inside it
    (g4b_gemv_chain_create_tp), eager and replayed in a graph."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, TP_FP8="1" if fp8 else "0", TP_ALLREDUCE=allreduce)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("world", [4, 8])
def test_tp_chain_decode_wider(world):
    """The in-chain all-reduce over 4 and 8 ranks (skipped on smaller boxes)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, TP_FP8="0", TP_ALLREDUCE="chain")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
