"""The reference arm of ``bench.py`` (the oracle port of the decode step, timed
on the host cores) at a shrunken shape on the CPU: one JSON line with the
driver's keys, the CPU baseline and e2e objects describing the run, a timed
region that holds the steps it reports, and no output from ranks other than
rank 0."""
from __future__ import annotations

import json

import bench

SMALL = ["--impl", "reference", "--layers", "2", "--width", "128", "--vocab", "1024", "--experts", "4",
         "--cpu-sample-streams", "2", "--steps", "3", "--warmup", "1"]


def _line(capsys) -> dict:
    lines = [line for line in capsys.readouterr().out.splitlines() if line.strip()]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_reference_arm_prints_one_contract_line(capsys, monkeypatch):
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    bench.main(SMALL)
    line = _line(capsys)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 1
    assert line["higher_is_better"] is True and line["vs_baseline"] is None and line["value"] > 0
    assert line["config"]["workload"] == "config5_herm_batched_decode" and line["config"]["layers"] == 2
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # ms_per_step is the median step, the timed region the sum of the steps
    assert line["timed_region_s"] * 1000.0 >= line["ms_per_step"] * 0.999
    # tokens/s of the sampled streams (one token per stream and step)
    assert abs(line["value"] - line["streams_sampled"] / (line["ms_per_step"] / 1000.0)) <= 1e-9 * line["value"]


def test_reference_arm_other_ranks_print_nothing(capsys, monkeypatch):
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    bench.main(SMALL)
    assert capsys.readouterr().out.strip() == ""
