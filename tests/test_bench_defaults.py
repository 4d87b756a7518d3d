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


def _parsed(*argv):
    return bench.parse_args(list(argv))


def test_reference_arm_is_chosen_before_any_workload_dispatch():
    """--impl reference runs the reference's CPU path at every world size and
    workload; it never reaches the tensor-parallel or any other GPU runner."""
    for world in (1, 2, 4, 8):
        for wl in ["stream", "gemv", "prefill"] + list(bench.GEMM_WORKLOADS):
            a = _parsed("--impl", "reference", "--workload", wl)
            bench.resolve_defaults(a, world)
            assert bench.select_runner(a, world) is bench.run_reference_arm, (world, wl)
    a = _parsed()
    bench.resolve_defaults(a, 4)
    assert bench.select_runner(a, 4) is bench.run_tp
    a = _parsed()
    bench.resolve_defaults(a, 1)
    assert bench.select_runner(a, 1) is bench.run_stream
    a = _parsed("--parallel", "tp")
    assert bench.select_runner(a, 1) is bench.run_tp


def test_reference_arm_on_other_ranks_does_no_work(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "3")
    monkeypatch.setenv("WORLD_SIZE", "4")

    def boom(args):
        raise AssertionError("a non-zero rank must not run the reference sampler")

    monkeypatch.setattr(bench, "reference_sampler", boom)
    bench.run_reference_arm(_parsed("--impl", "reference"))
    assert capsys.readouterr().out == ""


def test_reference_arm_line_matches_the_config_of_our_arm(monkeypatch, capsys):
    """The reference arm prints the metric, unit and config our arm prints for
    the same workload and world size, tagged impl=reference, with its cpu_baseline."""
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setattr(bench, "reference_sampler",
                        lambda args: {"step": lambda: None, "work": 10 ** 9, "unit": "GB/s", "div": 1e9,
                                      "sample": "stub", "cores": 1})
    a = _parsed("--impl", "reference", "--steps", "2", "--warmup", "1")
    bench.resolve_defaults(a, 4)
    bench.run_reference_arm(a)
    import json
    line = json.loads(capsys.readouterr().out.strip())
    ours = bench.describe(_parsed(), 4)
    assert line["impl"] == "reference"
    assert (line["metric"], line["unit"], line["config"], line["scaling"]) == \
        (ours["metric"], ours["unit"], ours["config"], ours["scaling"])
    assert line["config"]["parallelism"] == "tp4"
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_sampler_runs_the_oracle_on_the_gemv_config():
    """The sampler really runs the oracle GEMV (configs[0] shape) on the host."""
    s = bench.reference_sampler(_parsed("--workload", "gemv"))
    assert s["unit"] == "GB/s" and s["work"] == bench.gemv_bytes(bench.FFN, bench.HIDDEN, False)
    s["step"]()
