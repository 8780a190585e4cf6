"""Decode on 2 GPUs (one process each, torchrun), sharded by the library: attention heads,
dense FFN blocks and vocabulary rows (tensor parallelism; the attn_output / ffn_down partial
sums exchanged through the peers' memory inside the matvec kernels), and for the MoE and
MLA+MoE models the experts by ID (expert parallelism; each chosen expert's output sent to
its choice's slot on every rank).  Greedy tokens identical on every rank and to the CPU
oracle's.  Needs two GPUs; skipped on a one-GPU box."""
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


@pytest.mark.parametrize("cfg", ["TINY", "TINY_MOE", "TINY_MOE_NS", "TINY_MLA"])
@pytest.mark.parametrize("world", [2])
def test_tp_greedy_matches_oracle(world, cfg):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "tp_worker.py"),
           cfg, "48"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert '"matches_oracle": true' in r.stdout
