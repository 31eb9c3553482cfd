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
bs, pages, n = 65536, 96, 40  # MPCOMM_PAGED_CHUNK_SIZE=1 MiB: 16 pages per launch, 3 launches
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
    env = dict(os.environ, MPCOMM_KERNEL_TRACE="1024", MPCOMM_PAGED_CHUNK_SIZE=str(1 << 20), MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-c", PAGED], capture_output=True, text=True,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, f"{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    assert "paged put ok" in r.stdout


MIXED = r"""
import os, torch, mpcomm
torch.cuda.set_device(0)
n = 24 << 20
src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
dsts = [torch.zeros(n, dtype=torch.uint8, device="cuda") for _ in range(3)]
host = torch.zeros(n, dtype=torch.uint8).pin_memory()
back = torch.zeros(n, dtype=torch.uint8, device="cuda")
bs, pages, k = 16384, 8192, 4096
pool = torch.randint(0, 256, (pages, bs), dtype=torch.uint8).pin_memory()
idx_cpu = torch.randperm(pages, generator=torch.Generator().manual_seed(9))[:k]
idx = idx_cpu.cuda()
out = torch.empty(k * bs, dtype=torch.uint8, device="cuda")
c = mpcomm.MPComm()
assert c.init("mix") == 0 and c.start_accept_thread() == 0 and c.get_fabric_name() == "nvl"
for t in [src, back, host] + dsts:
    assert c.register_memory(t.data_ptr(), n) == 0
for t in dsts + [host]:
    assert c.publish_buffer(t.data_ptr(), n) == 0
port = c.get_tcp_port()
assert c.connect("self", "127.0.0.1", port) == 0 and c.query_remote_buffers("self", "127.0.0.1", port)
dram = c.map_dram_to_gpu(pool.data_ptr(), pool.numel())
assert dram
c.enable_h2d_qos(0, 0)  # READ posts pause while an H2D window is open
gs = torch.cuda.Stream()
assert c.tma_gather(dram, idx.data_ptr(), out.data_ptr(), k, bs, 0, 0, gs.cuda_stream) == 0
half = n // 2
hs = [c.broadcast_async(src.data_ptr(), n, ["self"] * 3, [d.data_ptr() for d in dsts]),
      c.scatter_async(src.data_ptr(), ["self", "self"], [host.data_ptr(), host.data_ptr() + half], [half, n - half])]
for h in hs:
    assert h != mpcomm.INVALID_TRANSFER_HANDLE
    assert c.wait_transfer(h, 60000) == 0
    c.release_transfer(h)
h = c.get_async(back.data_ptr(), "self", host.data_ptr(), n)  # READ over PCIe, gated by the QoS engine
assert c.wait_transfer(h, 60000) == 0
c.release_transfer(h)
torch.cuda.synchronize()
for d in dsts:
    assert torch.equal(d, src)
assert torch.equal(host.cuda(), src) and torch.equal(back, src)
assert torch.equal(out.view(k, bs).cpu(), pool[idx_cpu])
w = c.get_last_h2d_window(0)
assert w is not None and w["end_ns"] > w["begin_ns"] > 0, w
c.disable_h2d_qos()
c.unmap_dram_from_gpu(pool.data_ptr())
c.shutdown()
print("mixed ok")
"""


def test_broadcast_and_scatter_under_qos_window_with_pxn_rails():
    """broadcast_async to three destinations and scatter_async to two, with
    MPCOMM_PXN_ENABLE=1 (a rail per visible GPU) and H2D QoS on while a
    tmaGather's window is open on the same GPU, then a GET the QoS engine
    gates: every transfer completes bit-exact and the window is recorded."""
    env = dict(os.environ, MPCOMM_PXN_ENABLE="1", MPCOMM_NVL_CHUNK_SIZE=str(4 << 20), MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(["timeout", "-k", "30", "240", sys.executable, "-c", MIXED], capture_output=True, text=True,
                       cwd=ROOT, env=env)
    assert r.returncode == 0, f"{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    assert "mixed ok" in r.stdout
