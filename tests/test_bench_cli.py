"""The benchmark's command line and configuration table, checked without a GPU:
every configuration the headline line reports has a timing function and can be
run alone with ``--workload``."""

import sys

import pytest

import bench


def _parse(monkeypatch, *argv):
    monkeypatch.setattr(sys, "argv", ["bench.py", *argv])
    return bench.parse()


def test_every_reported_configuration_has_a_timing_function():
    assert set(bench.CONFIG_NAMES) <= set(bench.CONFIG_FNS)
    for name in bench.CONFIG_NAMES:
        assert bench.CONFIG_FNS[name].__doc__, f"{name}: timing function without a docstring"


@pytest.mark.parametrize("workload", ["preprocess", *bench.CONFIG_NAMES])
def test_each_configuration_runs_alone(monkeypatch, workload):
    args = _parse(monkeypatch, "--workload", workload, "--steps", "2", "--warmup", "3")
    assert args.workload == workload and args.steps == 2 and args.warmup == 3


def test_defaults_match_the_driver_contract(monkeypatch):
    args = _parse(monkeypatch)
    assert args.gpus == 1 and args.impl == "b200" and args.workload == "preprocess"
    assert args.steps >= 1 and args.warmup >= 3
    assert _parse(monkeypatch, "--impl", "reference").impl == "reference"
