"""Tensor-parallel dense decode on 2 GPUs (one process each, torchrun): attention heads, FFN
blocks and vocabulary rows sharded by the library, the attn_output / ffn_down partial sums
exchanged through the peers' memory inside the matvec kernels, greedy tokens identical on
every rank and to the CPU oracle's.  Needs two GPUs; skipped on a one-GPU box."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2])
def test_tp_greedy_matches_oracle(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "tp_worker.py"),
           "TINY", "48"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert '"matches_oracle": true' in r.stdout
