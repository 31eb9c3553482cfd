"""Multi-process CPU tests: the "sock" fabric between processes, and failure
detection on the host (a peer that exits, a refused connect, a peer that
drops the control connection mid-handshake). No GPU is touched."""
import ctypes
import json
import os
import socket
import struct
import subprocess
import sys
import time

import pytest

N = 4 << 20


ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class Target:
    def __init__(self, fabric="sock"):
        env = dict(os.environ, MPCOMM_FABRIC=fabric, MPCOMM_LOG_LEVEL="0")
        self.proc = subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "mp_cpu_target.py"), str(N)],
                                     stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True, env=env)
        line = self.proc.stdout.readline()
        assert line, "target did not start"
        info = json.loads(line)
        self.port, self.addr = info["port"], info["addr"]

    def cmd(self, c):
        self.proc.stdin.write(c + "\n")
        self.proc.stdin.flush()

    def crc(self):
        self.cmd("crc")
        return int(self.proc.stdout.readline())

    def close(self):
        if self.proc.poll() is None:
            try:
                self.cmd("stop")
                self.proc.wait(20)
            except (BrokenPipeError, subprocess.TimeoutExpired):
                self.proc.kill()


@pytest.fixture
def target():
    t = Target()
    yield t
    t.close()


@pytest.fixture
def initiator(monkeypatch):
    monkeypatch.setenv("MPCOMM_FABRIC", "sock")
    monkeypatch.setenv("MPCOMM_LOG_LEVEL", "0")
    import mpcomm

    c = mpcomm.MPComm()
    assert c.init("initiator") == 0
    yield c
    c.shutdown()


def test_sock_fabric_cross_process_put_get(target, initiator):
    import mpcomm

    port, raddr = target.port, target.addr
    c = initiator
    assert c.connect("T", "127.0.0.1", port) == 0
    info = c.query_remote_buffers("T", "127.0.0.1", port)
    assert info["buffers"][0]["addr"] == raddr
    src = ctypes.create_string_buffer(os.urandom(N), N)
    assert c.register_memory(ctypes.addressof(src), N) == 0
    h = c.put_async(ctypes.addressof(src), "T", raddr, N)
    assert c.wait_transfer(h, 30000) == 0
    c.release_transfer(h)
    assert target.crc() == mpcomm.ops.crc32_host(src.raw)
    back = ctypes.create_string_buffer(N)
    assert c.register_memory(ctypes.addressof(back), N) == 0
    h = c.get_async(ctypes.addressof(back), "T", raddr, N)
    assert c.wait_transfer(h, 30000) == 0
    c.release_transfer(h)
    assert back.raw == src.raw


def test_peer_exit_fails_transfer_without_hanging(target, initiator):
    import mpcomm

    port, raddr = target.port, target.addr
    c = initiator
    assert c.connect("T", "127.0.0.1", port) == 0
    assert c.query_remote_buffers("T", "127.0.0.1", port)
    src = ctypes.create_string_buffer(N)
    assert c.register_memory(ctypes.addressof(src), N) == 0
    target.cmd("die")
    assert target.proc.wait(30) == 3
    t0 = time.time()
    h = c.put_async(ctypes.addressof(src), "T", raddr, N)
    rc = c.wait_transfer(h, 20000)
    assert rc == int(mpcomm.MPCommError.ERR_TRANSFER), rc
    assert time.time() - t0 < 20
    c.release_transfer(h)


def test_connect_refused(initiator):
    import mpcomm

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]  # closed again: nothing listens here
    assert initiator.connect("nobody", "127.0.0.1", port) == int(mpcomm.MPCommError.ERR_CONNECTION)


def test_peer_drops_mid_handshake(initiator):
    import threading

    import mpcomm

    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    port = srv.getsockname()[1]

    def serve():
        conn, _ = srv.accept()
        conn.recv(4)                               # active side's NIC count
        conn.sendall(struct.pack("<I", 1))         # our NIC count, then vanish
        conn.close()

    t = threading.Thread(target=serve)
    t.start()
    assert initiator.connect("flaky", "127.0.0.1", port) == int(mpcomm.MPCommError.ERR_CONNECTION)
    t.join(10)
    srv.close()


HOST_BARRIER = r"""
import os, sys, time
import torch.distributed as dist
sys.path.insert(0, os.environ["ROOT"])
from mpcomm.bench.multigpu import _host_barrier
dist.init_process_group("gloo")
rank = dist.get_rank()
if rank == 1:
    time.sleep(1.0)  # arrives late
t0 = time.time()
_host_barrier(timeout_s=30)
_host_barrier(timeout_s=30)
waited = time.time() - t0
print(f"rank {rank} waited {waited:.2f}", flush=True)
assert rank == 1 or waited > 0.8, waited
dist.destroy_process_group()
"""


def test_bench_host_barrier_two_ranks(tmp_path):
    """The benchmark's store-based barrier (no device work) holds an early
    rank until the late one arrives, call after call."""
    script = tmp_path / "hb.py"
    script.write_text(HOST_BARRIER)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, ROOT=ROOT, MPCOMM_LOG_LEVEL="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", f"--master-port={port}", str(script)],
                       capture_output=True, text=True, env=env, timeout=180)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("waited") == 2
