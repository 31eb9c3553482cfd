"""Control-plane handshakes do not wait on the caller's device work.

A peer's connect() reaches this process on its accept thread, which creates
the GPU-fabric queue pairs. The process's own device work may be queued
behind something that waits for that very handshake (a collective the peer
has not joined yet, for instance). Queue-pair creation therefore issues no
call that runs on, or waits for, the legacy default stream: with a long
kernel pending there, connect() still completes at once.
"""
import time

import pytest
import torch

import mpcomm

pytestmark = pytest.mark.gpu


def test_connect_while_default_stream_is_busy(monkeypatch):
    monkeypatch.setenv("MPCOMM_LOG_LEVEL", "1")
    torch.cuda.set_device(0)
    buf = torch.zeros(1 << 20, dtype=torch.uint8).pin_memory()
    c = mpcomm.MPComm()
    assert c.init("busy") == 0 and c.start_accept_thread() == 0 and c.get_fabric_name() == "nvl"
    assert c.register_memory(buf.data_ptr(), buf.numel()) == 0
    assert c.publish_buffer(buf.data_ptr(), buf.numel()) == 0
    torch.cuda.synchronize()
    # About 3 s of device time queued on the legacy default stream.
    torch.cuda._sleep(int(3.0 * 1.9e9))
    t0 = time.perf_counter()
    assert c.connect("self", "127.0.0.1", c.get_tcp_port()) == 0
    assert c.query_remote_buffers("self", "127.0.0.1", c.get_tcp_port())
    took = time.perf_counter() - t0
    torch.cuda.synchronize()
    c.shutdown()
    assert took < 1.0, f"connect waited {took:.2f} s behind the default stream"


def test_pcie_affinity_self_check_gpu_fabric(monkeypatch):
    """On the GPU fabric every rail is a GPU: the sysfs affinity of GPU g is
    its own rail nvl_g, which the suffix heuristic also picks."""
    monkeypatch.setenv("MPCOMM_LOG_LEVEL", "1")
    c = mpcomm.MPComm()
    assert c.init("affinity") == 0 and c.get_fabric_name() == "nvl"
    rows = c.get_pcie_affinity_self_check()
    assert len(rows) == torch.cuda.device_count()
    row0 = rows[0]
    assert row0["gpu"] == 0 and "nvl_0" in row0["sysfs_rails"], row0
    assert row0["suffix_rail"] == "nvl_0" and row0["agrees"], row0
    c.shutdown()
