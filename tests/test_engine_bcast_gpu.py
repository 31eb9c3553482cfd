"""Fused broadcast through the MPComm engine on one GPU.

broadcast_async to several destinations reachable through one GPU-fabric
rail is posted as one one-to-many WRITE per chunk: a single gather_bcast
launch that reads each source tile once and stores it to every destination
(instead of a copy per destination). A host-memory source is an H2D read
and carries a QoS window like tmaGather. Runs in a child process so the
kernel trace ring (MPCOMM_KERNEL_TRACE) is configured from its start.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CODE = r"""
import os, torch, mpcomm
torch.cuda.set_device(0)
n = (24 << 20) + 4096  # two 16 MiB chunks
src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
hsrc = torch.randint(0, 256, (n,), dtype=torch.uint8).pin_memory()
d1 = torch.zeros(n, dtype=torch.uint8, device="cuda")
d2 = torch.zeros(n, dtype=torch.uint8, device="cuda")
c = mpcomm.MPComm()
assert c.init("bc") == 0 and c.start_accept_thread() == 0 and c.get_fabric_name() == "nvl"
for t in (src, hsrc, d1, d2):
    assert c.register_memory(t.data_ptr(), n) == 0
for t in (d1, d2):
    assert c.publish_buffer(t.data_ptr(), n) == 0
port = c.get_tcp_port()
assert c.connect("self", "127.0.0.1", port) == 0 and c.query_remote_buffers("self", "127.0.0.1", port)

def bcast(local):
    mpcomm._native.kernel_trace_reset()
    h = c.broadcast_async(local, n, ["self", "self"], [d1.data_ptr(), d2.data_ptr()])
    assert h != mpcomm.INVALID_TRANSFER_HANDLE
    assert c.wait_transfer(h, 60000) == 0
    r = c.get_transfer_result(h)
    c.release_transfer(h)
    assert r["bytes_transferred"] == 2 * n, r
    return [t["kind"] for t in mpcomm._native.kernel_trace()]

kinds = bcast(src.data_ptr())
torch.cuda.synchronize()
assert torch.equal(d1, src) and torch.equal(d2, src)
fused = os.environ.get("MPCOMM_FUSED_BROADCAST", "1") != "0"
if fused:
    assert kinds.count("gather_bcast_p2p") == 2 and "copy_batch" not in kinds, kinds
else:
    assert "gather_bcast_p2p" not in kinds and "copy_batch" in kinds, kinds

# Host-memory source: an H2D read, inside a QoS window when QoS is on.
c.enable_h2d_qos(0, 0)
d1.zero_(); d2.zero_(); torch.cuda.synchronize()
kinds = bcast(hsrc.data_ptr())
torch.cuda.synchronize()
assert torch.equal(d1.cpu(), hsrc) and torch.equal(d2.cpu(), hsrc)
if fused:
    w = c.get_last_h2d_window(0)
    assert w is not None and w["end_ns"] > w["begin_ns"] > 0, w
c.disable_h2d_qos()
c.shutdown()
print("engine bcast ok", kinds)
"""


@pytest.mark.parametrize("fused", ["1", "0"])
def test_engine_broadcast_one_gpu(fused):
    env = dict(os.environ, MPCOMM_KERNEL_TRACE="1024", MPCOMM_NVL_CHUNK_SIZE=str(16 << 20),
               MPCOMM_FUSED_BROADCAST=fused, MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-c", CODE], capture_output=True, text=True,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, f"{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    assert "engine bcast ok" in r.stdout


PAGED = r"""
import os, torch, mpcomm
torch.cuda.set_device(0)
bs, pages, n = 65536, 96, 40  # MPCOMM_NVL_CHUNK_SIZE=1 MiB: 16 pages per chunk, 3 chunks
pool = torch.randint(0, 256, (pages, bs), dtype=torch.uint8).pin_memory()
idx_cpu = torch.randperm(pages, generator=torch.Generator().manual_seed(3))[:n]
idx = idx_cpu.cuda()
dst = torch.zeros(n * bs, dtype=torch.uint8, device="cuda")
c = mpcomm.MPComm()
assert c.init("pg") == 0 and c.start_accept_thread() == 0 and c.get_fabric_name() == "nvl"
dram = c.map_dram_to_gpu(pool.data_ptr(), pool.numel())
assert dram
assert c.register_memory(dst.data_ptr(), dst.numel()) == 0
assert c.publish_buffer(dst.data_ptr(), dst.numel()) == 0
port = c.get_tcp_port()
assert c.connect("self", "127.0.0.1", port) == 0 and c.query_remote_buffers("self", "127.0.0.1", port)
c.enable_h2d_qos(0, 0)
mpcomm._native.kernel_trace_reset()
h = c.put_pages_async(dram, idx.data_ptr(), n, bs, "self", dst.data_ptr())
assert h != mpcomm.INVALID_TRANSFER_HANDLE
assert c.wait_transfer(h, 60000) == 0
r = c.get_transfer_result(h)
c.release_transfer(h)
assert r["bytes_transferred"] == n * bs, r
torch.cuda.synchronize()
assert torch.equal(dst.view(n, bs).cpu(), pool[idx_cpu])
kinds = [t["kind"] for t in mpcomm._native.kernel_trace()]
assert kinds.count("pxn_gather_forward") == 3, kinds
w = c.get_last_h2d_window(0)
assert w is not None and w["end_ns"] > w["begin_ns"] > 0, w
# Indices in host memory: no GPU holds them, so no rail can run the gather.
assert c.put_pages_async(dram, idx_cpu.data_ptr(), n, bs, "self", dst.data_ptr()) == mpcomm.INVALID_TRANSFER_HANDLE
c.disable_h2d_qos()
c.unmap_dram_from_gpu(pool.data_ptr())
c.shutdown()
print("paged put ok")
"""


def test_engine_paged_put_one_gpu():
    """put_pages_async: the fused PXN gather + forward as an engine transfer
    (one pxn_gather_forward launch per chunk of pages, with an H2D window)."""
    env = dict(os.environ, MPCOMM_KERNEL_TRACE="1024", MPCOMM_NVL_CHUNK_SIZE=str(1 << 20), MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-c", PAGED], capture_output=True, text=True,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, f"{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    assert "paged put ok" in r.stdout
