"""QoS control channel on the CPU (in-process loopback fabric): a gathering
host (B) opens a channel to a writer (A) and pauses, paces and clears A's
WRITEs into it; GETs are never held; a closed channel lifts the policy
(fail-open); frames in the reference's byte layout from a raw socket are
honoured."""
import ctypes
import socket
import struct
import time

import pytest

import mpcomm

N = 4 << 20


class Buf:
    def __init__(self, n, fill=b"\0"):
        self.raw = ctypes.create_string_buffer(fill * n if len(fill) == 1 else fill, n)
        self.ptr = ctypes.addressof(self.raw)


@pytest.fixture
def pair(lo_env):
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0
    assert a.start_accept_thread() == 0 and b.start_accept_thread() == 0
    tb, sa = Buf(N), Buf(N, b"\x5a")
    assert b.register_memory(tb.ptr, N) == 0 and b.publish_buffer(tb.ptr, N) == 0
    assert a.register_memory(sa.ptr, N) == 0
    assert a.connect("B", "127.0.0.1", b.get_tcp_port()) == 0
    assert a.query_remote_buffers("B", "127.0.0.1", b.get_tcp_port())
    assert b.connect("A", "127.0.0.1", a.get_tcp_port()) == 0
    yield a, b, sa, tb
    a.shutdown()
    b.shutdown()


def _wait(pred, timeout=5.0):
    t0 = time.time()
    while time.time() - t0 < timeout:
        if pred():
            return True
        time.sleep(0.005)
    return False


def test_pause_pace_clear(pair):
    a, b, sa, tb = pair
    assert b.open_qos_channel("A") == 0
    assert b.send_qos_policy("A", -1, 0) == 0
    assert _wait(lambda: len(a.get_remote_qos_policies()) == 1)
    pol = a.get_remote_qos_policies()[0]
    assert pol["peer_host_id"] == "B" and pol["gpu_device_id"] == -1 and pol["rate_bytes_per_sec"] == 0
    h = a.put_async(sa.ptr, "B", tb.ptr, N)
    time.sleep(0.3)
    assert not a.is_transfer_complete(h), "WRITE posted while paused"
    assert a.get_remote_qos_defer_count() > 0
    # A GET from B is a READ: never held by the peer's pause.
    back = Buf(1 << 20)
    assert a.register_memory(back.ptr, 1 << 20) == 0
    g = a.get_async(back.ptr, "B", tb.ptr, 1 << 20)
    assert a.wait_transfer(g, 5000) == 0
    a.release_transfer(g)
    assert b.clear_qos_policy("A") == 0
    assert a.wait_transfer(h, 10000) == 0
    a.release_transfer(h)
    assert ctypes.string_at(tb.ptr, N) == b"\x5a" * N
    assert _wait(lambda: a.get_remote_qos_policies() == [])
    # Paced: 16 MB/s with a 64 KiB burst -> 4 MiB takes >= ~0.2 s.
    assert b.send_qos_policy("A", -1, 16 << 20, 64 << 10) == 0
    assert _wait(lambda: len(a.get_remote_qos_policies()) == 1)
    t0 = time.time()
    h = a.put_async(sa.ptr, "B", tb.ptr, N)
    assert a.wait_transfer(h, 20000) == 0
    a.release_transfer(h)
    assert time.time() - t0 >= 0.15
    assert b.clear_qos_policy("A", -1) == 0


def test_channel_close_fails_open(pair):
    a, b, sa, tb = pair
    assert b.open_qos_channel("A") == 0 and b.send_qos_policy("A", -1, 0) == 0
    assert _wait(lambda: len(a.get_remote_qos_policies()) == 1)
    h = a.put_async(sa.ptr, "B", tb.ptr, N)
    time.sleep(0.1)
    assert not a.is_transfer_complete(h)
    assert b.close_qos_channel("A") == 0
    assert a.wait_transfer(h, 10000) == 0, "policy not lifted when the channel closed"
    a.release_transfer(h)
    assert a.get_remote_qos_policies() == []
    assert b.send_qos_policy("A", -1, 0) != 0  # channel gone


def test_policy_for_another_gpu_does_not_hold_host_writes(pair):
    a, b, sa, tb = pair
    assert b.open_qos_channel("A") == 0 and b.send_qos_policy("A", 3, 0) == 0  # B's GPU 3 only
    assert _wait(lambda: len(a.get_remote_qos_policies()) == 1)
    h = a.put_async(sa.ptr, "B", tb.ptr, N)  # into B's host memory
    assert a.wait_transfer(h, 10000) == 0
    a.release_transfer(h)


def test_reference_layout_frames_from_raw_socket(pair):
    """Hello + frames packed by hand (host-endian, 132 and 112 bytes)."""
    a, b, sa, tb = pair
    s = socket.create_connection(("127.0.0.1", a.get_tcp_port()))
    s.sendall(struct.pack("=I", 0x4D505143) + struct.pack("=I128s", 1, b"B"))

    def frame(kind, gpu, rate, burst, gen):
        return struct.pack("=IIIiI16I", 0x4D505146, 1, kind, gpu, 0, *([0] * 16)) + \
            struct.pack("=4xQQQ", rate, burst, gen)

    assert len(frame(1, -1, 0, 0, 1)) == 112
    s.sendall(frame(1, -1, 0, 4096, 7))
    assert _wait(lambda: a.get_remote_qos_policies() and a.get_remote_qos_policies()[0]["generation"] == 7)
    h = a.put_async(sa.ptr, "B", tb.ptr, N)
    time.sleep(0.2)
    assert not a.is_transfer_complete(h)
    s.sendall(frame(1, -1, 0, 4096, 3))  # stale generation: ignored
    time.sleep(0.05)
    assert a.get_remote_qos_policies()[0]["generation"] == 7
    s.sendall(frame(2, -1, 0, 0, 8))
    assert a.wait_transfer(h, 10000) == 0
    a.release_transfer(h)
    s.sendall(frame(1, -1, 0, 0, 9))
    assert _wait(lambda: len(a.get_remote_qos_policies()) == 1)
    s.sendall(b"\x00" * 112)  # bad magic: channel closed, policies lifted
    assert _wait(lambda: a.get_remote_qos_policies() == [])
    s.close()
