"""The measurement harness's host logic on CPU: the reference arm's JSON line (the CPU restatement of
the PGF step on a bounded prefix), and how the GPU arm names its workload, splits the sequence over
ranks and reports scaling."""
import argparse
import json
import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def _args(**kw):
    """bench.py's defaults (no command-line flags), with `kw` overriding."""
    bench = _bench()
    old = sys.argv
    sys.argv = ["bench.py"]
    try:
        a = bench.parse()
    finally:
        sys.argv = old
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_reference_arm_prints_one_line_with_the_contract_keys():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1",
                          "--cpu-sample-len", "64", "--layers", "2"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["steps"] == 1 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and "64 tokens" in cb["sample"]
    assert d["config"]["layers"] == 2 and d["config"]["seq_len"] == 1048576
    assert d["ms_per_step"] > 0


def test_reference_arm_under_torchrun_prints_once_from_rank_0():
    """Launched the way the multi-GPU runs launch both arms: rank 0 times and prints the one line,
    the other rank exits 0 without work."""
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "1", "--cpu-sample-len", "64", "--layers", "2"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["e2e"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"


@pytest.mark.parametrize("world,par,expect", [(1, "sp", 1048576), (2, "sp", 524288), (8, "sp", 131072),
                                              (8, "dp", 1048576)])
def test_sequence_split_over_ranks(world, par, expect):
    bench = _bench()
    a = _args(parallel=par)
    assert bench.per_rank_len(a, world) == expect
    assert bench.scaling_of(a, world) == ("strong" if par == "sp" else "weak")
    c = bench.config_of(a, world)
    assert c["seq_len"] == 1048576 and c["global_batch"] == (world if par == "dp" else 1)


def test_uneven_split_is_refused():
    bench = _bench()
    a = _args(seq_len=1000)
    with pytest.raises(SystemExit):
        bench.per_rank_len(a, 3)


def test_default_workload_and_variant_names():
    bench = _bench()
    a = _args()
    assert bench.default_workload(a, 1) and bench.default_workload(a, 8)
    assert "reference SSM variant" in bench.config_of(a, 1)["workload"]
    b = argparse.Namespace(**vars(a))
    b.variant = "std"
    assert not bench.default_workload(b, 1)
    assert "Mamba-standard" in bench.config_of(b, 1)["workload"]
