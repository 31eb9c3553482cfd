"""Multi-GPU cases (cross-process NVLink PUT/GET, PXN forward, NVLS) under
torch.distributed.run; skipped on hosts with fewer than 2 GPUs."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["putget", "pxn", "nvls", "gather_bcast", "peer_exit", "engine_bcast",
                                  "engine_pxn"])
def test_multigpu_case(case):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    n = 2 if case == "peer_exit" else min(n, 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "mp_cases.py"), case]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, f"{case} failed:\n{r.stdout[-4000:]}\n{r.stderr[-4000:]}"
    assert f"case {case} ok" in r.stdout


def test_pxn_proxy_rails_single_process():
    """MPCOMM_PXN_ENABLE=1: one process opens a GPU-fabric rail per visible
    GPU, and a PUT/GET between GPU 0's HBM and pinned host memory is striped
    over them (peers read/write GPU 0 over NVLink); the bytes round-trip
    bit-exact and more than one rail carries traffic."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    code = r"""
import os, torch, mpcomm
os.environ["MPCOMM_PXN_ENABLE"] = "1"
os.environ["MPCOMM_NVL_CHUNK_SIZE"] = str(4 << 20)
torch.cuda.set_device(0)
n = torch.cuda.device_count()
size = 64 << 20
src = torch.randint(0, 256, (size,), dtype=torch.uint8, device="cuda:0")
dst = torch.zeros(size, dtype=torch.uint8, device="cuda:0")
pool = torch.zeros(size, dtype=torch.uint8, pin_memory=True)
c = mpcomm.MPComm()
assert c.init("pxn-test") == 0 and c.start_accept_thread() == 0
assert len(c.get_active_devices()) == n, c.get_active_devices()
for t in (src, dst, pool):
    assert c.register_memory(t.data_ptr(), size) == 0
assert c.publish_buffer(pool.data_ptr(), size) == 0
port = c.get_tcp_port()
assert c.connect("pool", "127.0.0.1", port) == 0 and c.query_remote_buffers("pool", "127.0.0.1", port)
h = c.put_async(src.data_ptr(), "pool", pool.data_ptr(), size)
assert c.wait_transfer(h, 60000) == 0
c.release_transfer(h)
assert torch.equal(pool, src.cpu())
h = c.get_async(dst.data_ptr(), "pool", pool.data_ptr(), size)
assert c.wait_transfer(h, 60000) == 0
c.release_transfer(h)
torch.cuda.synchronize()
assert torch.equal(dst, src)
per_rail = c.get_rail_completed_bytes()
assert sum(per_rail) == 2 * size, per_rail
busy = [b for b in per_rail if b > 0]
assert len(busy) >= 2, per_rail
c.shutdown()
print("pxn rails ok", len(busy))
"""
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-c", code], capture_output=True,
                       text=True, cwd=ROOT, env=dict(os.environ, MPCOMM_LOG_LEVEL="1"))
    assert r.returncode == 0, f"{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    assert "pxn rails ok" in r.stdout
