"""Multi-GPU cases (cross-process NVLink PUT/GET, PXN forward, NVLS) under
torch.distributed.run; skipped on hosts with fewer than 2 GPUs."""
import json
import os
import socket
import subprocess
import sys
import time

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


def test_scatter_test_broadcast_across_gpus(tmp_path):
    """The C++ API end to end: scatter_test serves a buffer in the HBM of
    every GPU but 0; the initiator on GPU 0 broadcasts to all of them
    (--test-type broadcast), reads every slot back and compares it
    (--verify). Each request of 2 chunks is 2 fused launches whatever the
    number of targets."""
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    exe = os.path.join(ROOT, "examples", "bin", "scatter_test")
    env = dict(os.environ, MPCOMM_LOG_LEVEL="1", MPCOMM_NVL_CHUNK_SIZE=str(16 << 20))
    procs, targets = [], []
    try:
        for r in range(1, n):
            ready = tmp_path / f"t{r}.ready"
            procs.append(subprocess.Popen([exe, "--mode", "target", "--host-id", f"t{r}", "--gpu", str(r),
                                           "--buffer-size", "64M", "--ready-file", str(ready)],
                                          stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL, env=env))
        deadline = time.time() + 60
        for r in range(1, n):
            ready = tmp_path / f"t{r}.ready"
            while not ready.exists():
                assert time.time() < deadline, f"target {r} not ready"
                assert procs[r - 1].poll() is None, f"target {r} exited"
                time.sleep(0.1)
            targets += ["--target", f"t{r}:127.0.0.1:{int(ready.read_text().split()[0])}"]
        r = subprocess.run(["timeout", "-k", "10", "240", exe, "--gpu", "0", *targets, "--size", "32M",
                            "--batch-size", "2", "--iterations", "2", "--warmup", "1", "--test-type", "broadcast",
                            "--verify", "--json"], capture_output=True, text=True, env=env, cwd=ROOT)
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
        bench = next(x for x in lines if x.get("test") == "broadcast")
        check = next(x for x in lines if "verify" in x)
        assert check["bad"] == 0 and check["slots"] == 2 * (n - 1)
        assert bench["kernel_launches"] == 2 * 2 * 2, bench  # iterations x batch x chunks
    finally:
        for p in procs:
            p.terminate()
        for p in procs:
            try:
                p.wait(timeout=20)
            except subprocess.TimeoutExpired:
                p.kill()


def test_scatter_test_nvls_broadcast_across_gpus():
    """scatter_test --nvls: the initiator on GPU 0 creates an NVLS multicast
    group (native createMulticastGroup, no launcher) that a target process
    on every other GPU joins and serves its copy of; a broadcast to all the
    targets then goes out as multicast stores, one gather_bcast_nvls launch
    per chunk, and every copy (the initiator's own included) reads back
    bit-exact: the targets' copies are VMM memory, reached by the GETs
    through their descriptor servers. Targets leave on SIGTERM after
    releasing their copies."""
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    from mpcomm import _native
    if not all(_native.multicast_supported(d) for d in range(n)):
        pytest.skip("no NVLS multicast on these GPUs")
    exe = os.path.join(ROOT, "examples", "bin", "scatter_test")
    env = dict(os.environ, MPCOMM_LOG_LEVEL="1", MPCOMM_NVL_CHUNK_SIZE=str(16 << 20), MPCOMM_KERNEL_TRACE="256")
    group = f"scatter-test-{os.getpid()}"
    procs, targets, outs = [], [], []
    try:
        for r in range(1, n):
            port = _free_port()
            procs.append(subprocess.Popen([exe, "--mode", "target", "--host-id", f"t{r}", "--gpu", str(r),
                                           "--tcp-port", str(port), "--buffer-size", "64M",
                                           "--nvls", f"{group}:{n}"],
                                          stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env))
            targets += ["--target", f"t{r}:127.0.0.1:{port}"]
        r = subprocess.run(["timeout", "-k", "10", "240", exe, "--gpu", "0", *targets, "--size", "32M",
                            "--batch-size", "2", "--iterations", "2", "--warmup", "1", "--test-type", "broadcast",
                            "--nvls", f"{group}:{n}", "--nvls-create", "--verify", "--json"],
                           capture_output=True, text=True, env=env, cwd=ROOT)
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
        bench = next(x for x in lines if x.get("test") == "broadcast")
        check = next(x for x in lines if "verify" in x)
        assert check["bad"] == 0 and check["slots"] == 2 * n, check  # n - 1 targets + own copy
        assert bench["nvls_member"] and bench["kernel_kinds"] == {"gather_bcast_nvls": 8}, bench
    finally:
        for p in procs:
            p.terminate()
        for p in procs:
            try:
                outs.append(p.communicate(timeout=30)[0])
            except subprocess.TimeoutExpired:
                p.kill()
                outs.append(p.communicate()[0])
    for p, out in zip(procs, outs):
        assert p.returncode == 0 and "stopping" in out, out[-2000:]
