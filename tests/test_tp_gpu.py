"""Tensor-parallel decode on 2+ GPUs (skipped with fewer): tokens of the
sharded engine vs the golden vectors of the reference's eager path."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(world, config, tmp_path, nccl_only=False):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = str(tmp_path / f"tp{world}_{config}_{int(nccl_only)}.json")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", QB_TP_NCCL="1" if nccl_only else "0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "tp_gpu_worker.py"), out, config]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    with open(out) as f:
        return json.load(f)


@pytest.mark.parametrize("world", [2])
@pytest.mark.parametrize("nccl_only", [False, True], ids=["peer-reduction", "nccl-allreduce"])
def test_tp_small_matches_golden(world, nccl_only, tmp_path, built_lib):
    got = _run(world, "qwen3-small", tmp_path, nccl_only)
    gold = np.load(os.path.join(GOLDEN, "qwen3_small_greedy.npz"))["tokens"].tolist()
    assert got["tokens"] == gold
    assert got["again"] == gold


@pytest.mark.parametrize("world", [2, 4])
def test_tp_0p6b_matches_golden_until_reference_tie(world, tmp_path, built_lib):
    got = _run(world, "qwen3-0.6b", tmp_path)
    with open(os.path.join(GOLDEN, "qwen3_0p6b_greedy.json")) as f:
        g = json.load(f)
    first_tie = next(i for i, s in enumerate(g["steps"]) if s["margin"] == 0.0)
    assert got["tokens"][:first_tie] == g["tokens"][:first_tie]
