"""bench.py's command line (CPU): the driver's flags parse, the defaults are
the measured configuration, and the expert-parallel exchange mode defaults
to `auto` (each mode timed on the headline batch, the fastest kept)."""
from __future__ import annotations

import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_cli_under_test",
                                                  os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _parse(mod, argv):
    old = sys.argv
    sys.argv = ["bench.py"] + argv
    try:
        return mod.parse()
    finally:
        sys.argv = old


def test_driver_flags_parse_with_measured_defaults():
    b = _bench()
    a = _parse(b, ["--gpus", "1", "--steps", "20", "--warmup", "5"])
    assert (a.gpus, a.steps, a.warmup, a.impl) == (1, 20, 5, "ours")
    assert a.tokens == 64 and a.config == "1"       # BASELINE config 1 at T = 64
    assert a.prefill_tokens == 4096                 # config 3 sub-line
    assert a.ep_mode == "auto"


def test_reference_arm_and_modes_parse():
    b = _bench()
    assert _parse(b, ["--impl", "reference"]).impl == "reference"
    for mode in ("auto", "allgather", "nccl", "alltoall"):
        assert _parse(b, ["--ep-mode", mode]).ep_mode == mode
    # every fixed mode has a launch count for the gpu_launches claim
    assert set(b.LAUNCHES_PER_STEP_EP) == {"allgather", "nccl", "alltoall"}
