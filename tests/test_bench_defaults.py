"""bench.py's defaults for the schedule and the all-reduce (host logic, no GPU)."""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402


def _args(**kw):
    a = dict(workload="stream", parallel="auto", schedule=None, allreduce=None)
    a.update(kw)
    return argparse.Namespace(**a)


def test_one_gpu_runs_the_chain():
    a = _args()
    bench.resolve_defaults(a, 1)
    assert a.schedule == "chain" and a.allreduce == bench.TP_DEFAULT_ALLREDUCE


def test_tensor_parallel_defaults_follow_the_confirmed_worlds():
    for world in (2, 4, 8):
        a = _args()
        bench.resolve_defaults(a, world)
        assert a.schedule == ("chain" if world in bench.TP_CHAIN_CONFIRMED_WORLDS else "launches")


def test_explicit_choices_and_replicas_are_kept():
    a = _args(schedule="launches", allreduce="peer")
    bench.resolve_defaults(a, 2)
    assert (a.schedule, a.allreduce) == ("launches", "peer")
    a = _args(parallel="replicas")
    bench.resolve_defaults(a, 8)
    assert a.schedule == "chain"
