"""Tensor parallelism on 2+ GPUs of one node: tests/tp_worker.py under torch.distributed.run (one process per GPU),
checking the assembled logits of the sharded model against the FP64 oracle and a one-device model with the same
weights, and that every rank makes the same token choice. Skipped with fewer than two visible GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(case, world, mode="fused"):
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), "--case", case, "--mode", mode]
    p = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert p.returncode == 0, "tp worker failed (%d):\n%s\n%s" % (p.returncode, p.stdout[-3000:], p.stderr[-3000:])
    rep = json.loads(lines[-1])
    assert rep["ok"] and rep["tokens_agree"]
    assert rep["fused"] == (0 if mode == "nccl" else 1)
    return rep


@pytest.mark.parametrize("case,mode", [("small", "fused"), ("small", "nccl"), ("small", "two_shot"),
                                       ("small8", "fused")])
def test_tp2_small_against_oracle_and_one_device(case, mode):
    """The fused GEMM + peer-memory all-reduce and the NCCL all-reduce, each against the oracle and one device."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    rep = _run(case, 2, mode)
    assert rep["max_diff_vs_tp1"] < 0.02


def test_tp_internlm7b_shape_two_layers():
    n = _gpus()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    rep = _run("internlm7b", 8 if n >= 8 else 2)
    assert rep["max_diff_vs_tp1"] < 0.02


@pytest.mark.parametrize("mode", ["fused", "two_shot", "nccl"])
def test_tp4_internlm7b_shape(mode):
    """Four ranks: the fused one-shot all-reduce (the default there), the two-shot forced (reduce-scatter by the
    GEMMs' peer stores, a cooperative reduce + all-gather kernel; the default from 8 ranks) and NCCL."""
    if _gpus() < 4:
        pytest.skip("needs 4 GPUs")
    rep = _run("internlm7b", 4, mode)
    assert rep["max_diff_vs_tp1"] < 0.02
    assert rep["two_shot"] == (1 if mode == "two_shot" else 0)
