"""Multi-GPU clause sharding over NCCL (needs >= 2 GPUs): a torchrun-style
2-process run must give exactly the single-process result."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, sys.argv[1])
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
if world > 1:
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
from ytm_b200.cutm import MultiClassTM
from ytm_b200 import synthetic
X, y = synthetic.prototypes(600, seed=3)
tm = MultiClassTM(number_of_clauses_per_class=300, T=100, s=8.0, dim=(28, 28, 1), n_classes=10, seed=9)
tm.fit(X[:512], y[:512], batch_size=64)
tm.fit(X[:512], y[:512], batch_size=64)
ta, w = tm.get_ta_state(), tm.get_weights()
pred, cs = tm.predict(X[512:])          # sample-sharded inference (default)
tm.inference_sharding = "clauses"
pred2, cs2 = tm.predict(X[512:])        # clause-sharded inference
if rank == 0:
    np.savez(sys.argv[2], ta=ta, w=w, cs=cs, cs2=cs2)
if world > 1:
    dist.destroy_process_group()
"""


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(world, out, tmp):
    script = tmp / "worker.py"
    script.write_text(WORKER)
    procs = []
    port = _port()
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, str(script), ROOT, str(out)], env=env))
    for p in procs:
        assert p.wait(timeout=600) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharding_equals_one_gpu(tmp_path):
    _run(1, tmp_path / "one.npz", tmp_path)
    _run(2, tmp_path / "two.npz", tmp_path)
    a, b = np.load(tmp_path / "one.npz"), np.load(tmp_path / "two.npz")
    for k in ("ta", "w", "cs", "cs2"):
        np.testing.assert_array_equal(a[k], b[k])
