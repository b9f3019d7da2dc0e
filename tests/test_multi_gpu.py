"""Row-sharded ticks on 2 GPUs of one node (skipped with fewer GPUs).

The in-kernel peer exchange (nsb_dendritic_run_tiled_peers) and the NCCL
exchange are checked bit for bit against the single-GPU runtime, and a rank
that does not launch makes the other rank's cross-GPU barrier give up with a
status code instead of hanging.  The ranks run as child processes under
torch.distributed.run (tests/mgpu_worker.py).
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

WORKER = Path(__file__).resolve().parent / "mgpu_worker.py"


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(mode: str, timeout: int = 300) -> str:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), str(WORKER), mode]
    result = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout + 60)
    assert result.returncode == 0, result.stdout[-3000:] + result.stderr[-3000:]
    return result.stdout


needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


@pytest.mark.gpu
@needs_two
def test_sharded_exchanges_bitwise_equal_one_gpu():
    out = _run("parity")
    lines = [line.split() for line in out.splitlines() if line.startswith("PARITY")]
    assert len(lines) == 3, out
    for _, case, ok, *diffs in lines:
        assert ok == "True", (case, diffs)


@pytest.mark.gpu
@needs_two
def test_missing_rank_ends_the_cross_gpu_barrier_with_a_status():
    out = _run("timeout")
    codes = [int(line.split()[1]) for line in out.splitlines() if line.startswith("STATUS")]
    assert codes == [6], out


@pytest.mark.gpu
@needs_two
def test_sharded_checkpoint_restores_sharded_and_single_gpu():
    out = _run("checkpoint")
    lines = [line.split() for line in out.splitlines() if line.startswith("CHECKPOINT")]
    assert [case for _, case, _ in lines] == ["sharded", "single"], out
    for _, case, ok in lines:
        assert ok == "True", case


@pytest.mark.gpu
@needs_two
def test_sharded_pels_peer_and_nccl_exchanges_match_one_gpu():
    out = _run("pels")
    lines = [line.split() for line in out.splitlines() if line.startswith("PELS")]
    assert len(lines) == 5, out
    for _, case, ok, *diffs in lines:
        assert ok == "True", (case, diffs)


@pytest.mark.gpu
@needs_two
def test_missing_rank_ends_the_pels_delta_wait_with_a_status():
    out = _run("pels_timeout")
    codes = [int(line.split()[1]) for line in out.splitlines() if line.startswith("STATUS")]
    assert codes == [6], out


@pytest.mark.gpu
@needs_two
def test_sharded_stream_rollouts_equal_one_gpu_steps():
    """ShardedDendriticMatrixRuntime.stream(): rollout launches with the peer
    exchange, step() per tick with NCCL; every tick's rows equal one GPU's."""
    out = _run("stream")
    lines = [line.split() for line in out.splitlines() if line.startswith("STREAM")]
    assert [case for _, case, _ in lines] == ["peer", "nccl"], out
    for _, case, ok in lines:
        assert ok == "True", case
