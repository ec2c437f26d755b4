"""Multi-rank tests of the row-sharded path (one process per rank).

CPU (gloo, world size 2): the host-side decomposition -- shard ranges from
the C ABI, per-shard search, all-gather, merge -- equals the full search;
a rank that leaves is detected by the surviving rank's collective timing
out with an error.  GPU (2 GPUs, NCCL inside the engine): every rank gets the
merged global result, checked against the oracle.
"""
import os
import signal
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

WORKER = os.path.join(ROOT, "tests", "sharded_worker.py")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(mode, nproc, timeout):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", WORKER, mode]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="2")
    p = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         env=env, start_new_session=True)
    try:
        out, _ = p.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)
        out, _ = p.communicate()
        pytest.fail(f"{mode} workers timed out:\n{out[-3000:]}")
    return p.returncode, out


def test_cpu_shard_gather_merge_world2(engine):
    rc, out = _launch("cpu-merge", 2, 300)
    assert rc == 0, out[-3000:]


def test_cpu_lost_rank_is_detected(engine):
    rc, out = _launch("cpu-lost", 2, 120)
    assert "detected the lost peer" in out, out[-3000:]


@pytest.mark.gpu
def test_gpu_two_ranks_nccl(engine):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    rc, out = _launch("gpu", 2, 600)
    assert rc == 0, out[-4000:]
    assert "detected the missing peer list" in out, out[-4000:]


@pytest.mark.gpu
def test_gpu_two_ranks_exact_rerank_and_inner_product(engine):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    rc, out = _launch("gpu-exact", 2, 600)
    assert rc == 0, out[-4000:]
