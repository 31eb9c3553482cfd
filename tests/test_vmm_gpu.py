"""VMM (cuMemCreate) memory between processes over the GPU fabric.

CUDA IPC cannot export VMM allocations (NVLS group copies, GPUDirect
buffers from gdr_alloc, PyTorch's expandable segments), so the nvl fabric
offers such a registration as the POSIX handles of the allocations behind
it on the owner's descriptor server; a peer fetches them over the Unix
socket, maps them back to back, and its kernels then PUT/GET the range like
cudaMalloc memory. Two processes on one GPU: the target serves a gdr_alloc
buffer (one allocation) or a tensor of an expandable segment (several
allocations), the initiator writes it, reads it back, and the target checks
its own bytes.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

TARGET = r"""
import os, sys, time, zlib, torch, mpcomm
from mpcomm import parallel
d, kind = sys.argv[1], sys.argv[2]
torch.cuda.set_device(0)
n = 64 << 20
if kind == "gdr":
    err, ptr, size = mpcomm._native.gdr_alloc(0, n)
    assert err == 0 and size >= n, (err, size)
    buf = parallel.device_view(ptr, n)
else:  # PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True
    torch.empty(3 << 20, dtype=torch.uint8, device="cuda")  # start mid-page
    buf = torch.empty(n, dtype=torch.uint8, device="cuda")
    ptr = buf.data_ptr()
    err, segs = mpcomm._native.vmm_segments(ptr, n)
    assert err == 0 and len(segs) >= 2, (err, segs)
buf.zero_(); torch.cuda.synchronize()
c = mpcomm.MPComm()
assert c.init("vt") == 0 and c.get_fabric_name() == "nvl"
assert c.register_memory(ptr, n) == 0 and c.publish_buffer(ptr, n) == 0
assert c.start_accept_thread() == 0
open(os.path.join(d, "port.tmp"), "w").write(str(c.get_tcp_port()))
os.rename(os.path.join(d, "port.tmp"), os.path.join(d, "port"))
deadline = time.time() + 120
while not os.path.exists(os.path.join(d, "crc")):
    assert time.time() < deadline, "initiator never finished"
    time.sleep(0.05)
want = int(open(os.path.join(d, "crc")).read())
torch.cuda.synchronize()
got = zlib.crc32(buf.cpu().numpy().tobytes())
c.unpublish_buffer(ptr); c.unregister_memory(ptr)
c.shutdown()
if kind == "gdr":
    mpcomm._native.gdr_free(ptr, size)
assert got == want, (got, want)
print("target bytes ok")
"""

INITIATOR = r"""
import os, sys, time, zlib, torch, mpcomm
d = sys.argv[1]
torch.cuda.set_device(0)
n = 64 << 20
deadline = time.time() + 120
while not os.path.exists(os.path.join(d, "port")):
    assert time.time() < deadline, "target never served"
    time.sleep(0.05)
port = int(open(os.path.join(d, "port")).read())
src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
back = torch.zeros(n, dtype=torch.uint8, device="cuda")
c = mpcomm.MPComm()
assert c.init("vi") == 0 and c.get_fabric_name() == "nvl"
for t in (src, back):
    assert c.register_memory(t.data_ptr(), n) == 0
assert c.connect("vt", "127.0.0.1", port) == 0
raddr = c.query_remote_buffers("vt", "127.0.0.1", port)["buffers"][0]["addr"]
h = c.put_async(src.data_ptr(), "vt", raddr, n)
assert h != mpcomm.INVALID_TRANSFER_HANDLE and c.wait_transfer(h, 60000) == 0
c.release_transfer(h)
h = c.get_async(back.data_ptr(), "vt", raddr, n)
assert h != mpcomm.INVALID_TRANSFER_HANDLE and c.wait_transfer(h, 60000) == 0
c.release_transfer(h)
torch.cuda.synchronize()
assert torch.equal(back, src), "GET of the VMM buffer differs from the PUT"
crc = zlib.crc32(src.cpu().numpy().tobytes())
open(os.path.join(d, "crc.tmp"), "w").write(str(crc))
os.rename(os.path.join(d, "crc.tmp"), os.path.join(d, "crc"))
c.shutdown()
print("initiator vmm ok")
"""


@pytest.mark.parametrize("kind", ["gdr", "expandable"])
def test_put_get_vmm_buffer_of_another_process(tmp_path, kind):
    env = dict(os.environ, MPCOMM_LOG_LEVEL="1", MPCOMM_FABRIC="nvl")
    tenv = dict(env, PYTORCH_CUDA_ALLOC_CONF="expandable_segments:True") if kind == "expandable" else env
    t = subprocess.Popen(["timeout", "-k", "10", "180", sys.executable, "-c", TARGET, str(tmp_path), kind], cwd=ROOT,
                         env=tenv, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    try:
        r = subprocess.run(["timeout", "-k", "10", "180", sys.executable, "-c", INITIATOR, str(tmp_path)], cwd=ROOT,
                           env=env, capture_output=True, text=True)
        assert r.returncode == 0 and "initiator vmm ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
        out, _ = t.communicate(timeout=120)
        assert t.returncode == 0 and "target bytes ok" in out, out[-3000:]
    finally:
        if t.poll() is None:
            t.kill()
            t.wait()


PEERS = r"""
import os, sys, torch, torch.distributed as dist
from mpcomm import _native, parallel
rank, world = int(sys.argv[1]), 2
dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{sys.argv[2]}", rank=rank, world_size=world)
torch.cuda.set_device(0)
torch.empty(5 << 20, dtype=torch.uint8, device="cuda")  # start mid-page
pb = parallel.PeerBuffers(48 << 20)
err, segs = _native.vmm_segments(pb.local.data_ptr(), pb.nbytes)
assert err == 0 and len(segs) >= 2, (err, segs)
pb.local.copy_(torch.arange(pb.nbytes, device="cuda", dtype=torch.int64).to(torch.uint8) ^ (rank + 1))
torch.cuda.synchronize()
dist.barrier()
peer = 1 - rank
# The library's own copy kernel moves bytes to and from the peer's mapping.
got = torch.empty(pb.nbytes, dtype=torch.uint8, device="cuda")
assert _native.copy_spans([pb.ptrs[peer]], [got.data_ptr()], [pb.nbytes]) == 0
want = torch.arange(pb.nbytes, device="cuda", dtype=torch.int64).to(torch.uint8) ^ (peer + 1)
torch.cuda.synchronize()
assert torch.equal(got, want), "peer view differs"
mark = torch.full((4096,), 0xA0 + rank, dtype=torch.uint8, device="cuda")
assert _native.copy_spans([mark.data_ptr()], [pb.ptrs[peer]], [4096]) == 0  # a store into the peer's buffer
torch.cuda.synchronize()
dist.barrier()
assert bool((pb.local[:4096] == 0xA0 + peer).all()), "the peer's store did not land"
dist.barrier()
pb.close()
dist.destroy_process_group()
print(f"rank {rank} peer buffers ok")
"""


def test_peer_buffers_over_expandable_segments():
    """PeerBuffers when the allocator hands out expandable-segment memory
    (CUDA IPC cannot export it): two ranks on one GPU share their buffers
    through the descriptor servers, read each other's bytes and store into
    each other's buffers."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, PYTORCH_CUDA_ALLOC_CONF="expandable_segments:True", MPCOMM_LOG_LEVEL="1")
    ps = [subprocess.Popen(["timeout", "-k", "10", "180", sys.executable, "-c", PEERS, str(r), str(port)], cwd=ROOT,
                           env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = [p.communicate(timeout=240)[0] for p in ps]
    for r, (p, out) in enumerate(zip(ps, outs)):
        assert p.returncode == 0 and f"rank {r} peer buffers ok" in out, out[-3000:]
