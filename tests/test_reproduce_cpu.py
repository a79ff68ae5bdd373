"""The reproduction driver (benchmarks/reproduce.py): every command it would run names an
existing entry point with options that entry point accepts (checked with each entry
point's own argument parser, without running it)."""
import argparse
import importlib
import os
import sys

import pytest

from quantized_flash_communication_b200.benchmarks import reproduce

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class _Captured(Exception):
    def __init__(self, parser):
        self.parser = parser


def _parser_of(target):
    """The argparse parser an entry point builds, captured at its first parse_args call."""
    orig = argparse.ArgumentParser.parse_args

    def capture(self, *a, **k):
        raise _Captured(self)
    argparse.ArgumentParser.parse_args = capture
    try:
        if target[0] == "-m":
            mod = importlib.import_module(target[1])
            call = (lambda: mod.main([]))
        else:
            if ROOT not in sys.path:
                sys.path.insert(0, ROOT)
            mod = importlib.import_module(os.path.splitext(target[0])[0])
            call = mod.parse_args if hasattr(mod, "parse_args") else mod.main
        try:
            call()
        except _Captured as c:
            return c.parser
        raise AssertionError(f"{target[:2]} built no argument parser")
    finally:
        argparse.ArgumentParser.parse_args = orig


@pytest.mark.parametrize("gpus", [1, 2, 8])
def test_every_command_parses(gpus):
    table = reproduce.items(gpus)
    assert set(table) == {"flagship", "variants", "breakdown", "allreduce", "norm", "decode", "tables", "quant",
                          "kernels"}
    for item, cmds in table.items():
        for n, target in cmds:
            assert n <= gpus, (item, n)
            parser = _parser_of(target)
            args = target[2:] if target[0] == "-m" else target[1:]
            parser.parse_args(args)  # raises SystemExit on an unknown option or a bad value


def test_multi_gpu_commands_use_torchrun_on_localhost():
    for n, target in reproduce.items(8)["variants"]:
        cmd = reproduce._launch(n, target)
        assert "torch.distributed.run" in cmd and "127.0.0.1" in cmd and f"--nproc-per-node={n}" in cmd


def test_dry_run_lists_commands(capsys):
    assert reproduce.main(["--gpus", "2", "--only", "flagship,quant", "--dry-run"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert any("bench.py --gpus 2" in ln for ln in out) and any("bench_quant" in ln for ln in out)


def test_gpu_count_filter(capsys):
    assert reproduce.main(["--gpus", "8", "--only", "variants,flagship", "--ns", "8", "--dry-run"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert out and all("--nproc-per-node=8" in ln for ln in out)
