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


def _run(world, out, tmp, extra_env=None, script=None, text=WORKER):
    if script is None:
        script = tmp / "worker.py"
        script.write_text(text)
    procs = []
    port = _port()
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", **(extra_env or {}))
        procs.append(subprocess.Popen([sys.executable, str(script), ROOT, str(out)], env=env))
    for p in procs:
        assert p.wait(timeout=600) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("allreduce", ["peer", "nccl"])
def test_two_gpu_sharding_equals_one_gpu(tmp_path, allreduce):
    """Clause-sharded training with the class sums summed by the NVLink peer
    all-reduce (default) or by NCCL equals one GPU bit for bit."""
    _run(1, tmp_path / "one.npz", tmp_path)
    _run(2, tmp_path / "two.npz", tmp_path, {"YTM_ALLREDUCE": allreduce})
    a, b = np.load(tmp_path / "one.npz"), np.load(tmp_path / "two.npz")
    for k in ("ta", "w", "cs", "cs2"):
        np.testing.assert_array_equal(a[k], b[k])


ENCODE = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, sys.argv[1])
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
if world > 1:
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
from ytm_b200.cutm import MultiClassTM
from ytm_b200 import synthetic
X, y = synthetic.prototypes(101, seed=4)
out = {}
for name, pd in (("single", (28, 28)), ("conv", (10, 10))):
    tm = MultiClassTM(number_of_clauses_per_class=20, T=10, s=5.0, dim=(28, 28, 1), n_classes=10, patch_dim=pd,
                      seed=2)
    for n in (101, 3, 2):  # ragged shares, the last one padded; one row per rank
        out[f"{name}_{n}"] = tm._literals_device(X[:n], False).cpu().numpy()
        out[f"{name}_{n}_pinned"] = tm._literals_device(torch.from_numpy(X[:n].view(np.int32)).pin_memory(),
                                                        False).cpu().numpy()
if rank == world - 1:
    np.savez(sys.argv[2], **out)
if world > 1:
    dist.destroy_process_group()
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_host_input_rows_sharded(tmp_path):
    """Host inputs on 2 GPUs: each rank copies and encodes half of the rows and
    the encoded rows are all-gathered; the result equals one GPU's encoding
    of all rows (literal words and packed bit images, ragged row counts)."""
    s1, s2 = tmp_path / "e1.py", tmp_path / "e2.py"
    s1.write_text(ENCODE)
    s2.write_text(ENCODE)
    _run(1, tmp_path / "one.npz", tmp_path, script=s1)
    _run(2, tmp_path / "two.npz", tmp_path, script=s2)
    a, b = np.load(tmp_path / "one.npz"), np.load(tmp_path / "two.npz")
    assert set(a.files) == set(b.files)
    for k in a.files:
        np.testing.assert_array_equal(a[k], b[k])


PEER = r"""
import os, sys, ctypes as ct, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, sys.argv[1])
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
from ytm_b200 import _lib
lib = _lib.load()
ctx = ct.c_void_p(); h = (ct.c_uint8 * 64)()
_lib.check(lib.ytm_peer_ar_create(rank, world, 5000, ct.byref(ctx), h))
hs = [None] * world
dist.all_gather_object(hs, bytes(h))
_lib.check(lib.ytm_peer_ar_open(ctx, (ct.c_uint8 * (64 * world)).from_buffer_copy(b"".join(hs))))
dist.barrier()
mode = sys.argv[3]
st = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
ok = True
if mode == "sum":
    for it in range(7):  # several calls: both data slots, ragged sizes
        n = 5000 - 613 * it
        g = torch.Generator().manual_seed(it)
        allv = torch.randint(-10**6, 10**6, (world, n), generator=g, dtype=torch.int32)
        x = allv[rank].cuda()
        _lib.check(lib.ytm_peer_allreduce_i32(ctx, ct.c_void_p(x.data_ptr()), n, 0, st))
        ok &= bool(torch.equal(x.cpu(), allv.sum(0, dtype=torch.int32)))
    s = ct.c_int32(-1); _lib.check(lib.ytm_peer_ar_status(ctx, ct.byref(s)))
    ok &= s.value == 0
else:  # rank 1 never arrives: rank 0 must give up after its short limit and say which peer
    if rank == 0:
        x = torch.arange(10, dtype=torch.int32, device="cuda")
        _lib.check(lib.ytm_peer_allreduce_i32(ctx, ct.c_void_p(x.data_ptr()), 10, 1 << 14, st))
        s = ct.c_int32(-1); _lib.check(lib.ytm_peer_ar_status(ctx, ct.byref(s)))
        ok &= s.value == 2 and bool(torch.equal(x.cpu(), torch.arange(10, dtype=torch.int32)))
    dist.barrier()
dist.barrier()
lib.ytm_peer_ar_destroy(ctx)
if rank == 0:
    open(sys.argv[2], "w").write("ok" if ok else "bad")
dist.destroy_process_group()
"""


def _run_peer(tmp, mode):
    script = tmp / "peer.py"
    script.write_text(PEER)
    out = tmp / f"peer_{mode}.txt"
    port = _port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, str(script), ROOT, str(out), mode], env=env))
    for p in procs:
        assert p.wait(timeout=300) == 0
    return out.read_text()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_sums(tmp_path):
    assert _run_peer(tmp_path, "sum") == "ok"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_reports_missing_rank(tmp_path):
    """A rank that never arrives: the waiting rank's bounded spin ends, the
    status names the missing peer, and the data are left as they were."""
    assert _run_peer(tmp_path, "timeout") == "ok"
