"""bench.py's reference arm (--impl reference) on the CPU: for each workload it
times the matching CPU path (the oracle port, and for the network torch's CPU
Linear layers around it) under the same metric as that workload's b200 line,
with the contract's cpu_baseline and e2e objects; ranks other than 0 print
nothing."""
import json
import types

import pytest

import bench


def _args(workload):
    return types.SimpleNamespace(workload=workload, steps=1, warmup=0, gpus=1)


@pytest.mark.parametrize("workload,metric", [("c1", bench.C1_METRIC), ("affine", bench.AFF_METRIC),
                                             ("alif", bench.ALIF_METRIC), ("c3", bench.C3_METRIC)])
def test_reference_line_matches_the_workload(capsys, workload, metric):
    bench.run_reference(_args(workload), 1, 0)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == metric and line["unit"] == bench.UNIT
    assert line["value"] > 0 and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": bench.UNIT, "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_other_ranks_print_nothing(capsys):
    bench.run_reference(_args("c2"), 2, 1)
    assert capsys.readouterr().out == ""
