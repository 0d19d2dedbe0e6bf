"""GPU, 2 or more devices: tensor-parallel decode logits against the same model unsharded.

Runs bench.py's parity check under torchrun (one process per GPU, NCCL for the setup, the fused NVLink
peer all-reduce in the decode step): a 2-layer model of the 27B-class shapes with an 8-bpw head is
built sharded over the ranks and unsharded on each rank from the same seed over the same KV cache; one
decode step's gathered logits must agree with the unsharded ones to KL <= 1e-4 (the north-star logit
tolerance) and give the same greedy token. Skipped on a box with fewer GPUs."""
import json
import os
import signal
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_logits_match_unsharded(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "bench.py"),
           "--tp-parity-only", "--gpus", str(world)]
    # NVLS off: a rank that fails must not leave NVLink multicast objects bound on the others
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                         start_new_session=True)
    try:
        out, err = p.communicate(timeout=600)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)
        out, err = p.communicate()
        pytest.fail(f"TP{world} parity run timed out:\n{err[-3000:]}")
    assert p.returncode == 0, err[-3000:]
    line = [ln for ln in out.splitlines() if ln.startswith("{")][-1]
    res = json.loads(line)["tp_parity"]
    print(f"TP{world}: {res}")
    assert res["argmax_equal"], res
    assert res["kl"] <= 1e-4, res
