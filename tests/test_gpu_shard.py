"""KV-head sharded decode on 2+ GPUs (NCCL all-gather, and peer-memory output
assembly) against the unsharded result."""

import json
import os
import subprocess
import sys

import pytest
import torch

from tests.conftest import ROOT

pytestmark = pytest.mark.gpu


def _run(world):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHARD_BATCH="16")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "shard_worker.py")]
    proc = subprocess.run(["timeout", "-k", "30", "240", *cmd], capture_output=True, text=True,
                          env=env, cwd=ROOT)
    lines = [l for l in proc.stdout.splitlines() if l.startswith("SHARD_RESULT ")]
    assert proc.returncode == 0 and lines, proc.stdout[-2000:] + proc.stderr[-3000:]
    return json.loads(lines[0][len("SHARD_RESULT "):])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_matches_unsharded(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(world)
    assert res["peer_equal_nccl_all_ranks"], res
    assert res["pool_bit_exact"]
    assert res["within_tol"], res
    assert res["max_vs_single"] < 2e-2, res
