"""CPU tests of the public API on the in-process loopback fabric.

Mirrors the reference's correctness harness (user_examples/test_mpcomm.py:
scatter/gather/broadcast/put/get with read-back verification) without NICs:
two MPComm objects in one process talk through the real TCP control plane
and the "lo" fabric.
"""
import ctypes
import os
import subprocess
import sys
import zlib

import pytest

import mpcomm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class Buf:
    def __init__(self, n, fill=None):
        self.raw = ctypes.create_string_buffer(n)
        self.n = n
        if fill is not None:
            ctypes.memmove(self.ptr, fill, n)

    @property
    def ptr(self):
        return ctypes.addressof(self.raw)

    def bytes(self, off=0, n=None):
        n = self.n - off if n is None else n
        return ctypes.string_at(self.ptr + off, n)


@pytest.fixture
def pair(lo_env):
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0
    assert b.start_accept_thread() == 0
    yield a, b
    a.shutdown()
    b.shutdown()


def connect(a, b, tbuf, n):
    assert b.register_memory(tbuf.ptr, n) == 0
    assert b.publish_buffer(tbuf.ptr, n) == 0
    port = b.get_tcp_port()
    assert a.connect("B", "127.0.0.1", port) == 0
    info = a.query_remote_buffers("B", "127.0.0.1", port)
    assert info["buffers"][0]["addr"] == tbuf.ptr
    return port


def test_module_surface():
    for name in ["SUCCESS", "ERR_DEVICE", "ERR_CONTEXT", "ERR_MEMORY", "ERR_CONNECTION", "ERR_TRANSFER",
                 "ERR_TIMEOUT", "ERR_INVALID_ARG", "ERR_INVALID_HANDLE", "ERR_PENDING"]:
        assert hasattr(mpcomm.MPCommError, name)
    assert int(mpcomm.MPCommError.ERR_PENDING) == -9
    assert mpcomm.INVALID_TRANSFER_HANDLE == 0
    assert (mpcomm.H2D_MODE_AUTO, mpcomm.H2D_MODE_SM, mpcomm.H2D_MODE_TMA) == (0, 1, 2)
    assert mpcomm.MPComm.get_nic_filter_env_var_name() == "MPCOMM_NIC_FILTER"
    assert mpcomm.MPComm.get_qps_per_connection_env_var_name() == "MPCOMM_QPS_PER_CONNECTION"
    for m in ["init", "shutdown", "register_memory", "unregister_memory", "connect", "start_accept_thread",
              "stop_accept_thread", "update_remote_memory_info", "get_rkey", "get_all_rkeys", "scatter_async",
              "gather_async", "broadcast_async", "put_async", "get_async", "mp_replicate_async",
              "is_transfer_complete", "wait_transfer", "get_transfer_result", "release_transfer",
              "get_num_nics", "get_local_host_id", "get_tcp_port", "get_gid", "get_device_name",
              "get_active_devices", "get_qps_per_connection", "set_nic_throttle", "clear_nic_throttle",
              "enable_h2d_qos", "set_h2d_qos_policy", "is_h2d_qos_enabled", "disable_h2d_qos",
              "get_nic_completed_bytes", "get_rail_completed_bytes", "get_pcie_domain_stats", "reset_pcie_domain_stats",
              "is_pcie_domain_stat_enabled", "get_throttle_latency", "write_bytes_to_buffer",
              "read_bytes_from_buffer", "publish_buffer", "unpublish_buffer", "unpublish_all_buffers",
              "get_published_buffer_count", "query_remote_buffers", "query_remote_buffer_by_numa",
              "query_remote_buffer", "get_published_buffer_info", "map_dram_to_gpu", "unmap_dram_from_gpu",
              "tma_gather", "tma_scatter"]:
        assert hasattr(mpcomm.MPComm, m), m


def test_not_initialized_errors(lo_env):
    c = mpcomm.MPComm()
    buf = Buf(64)
    assert c.register_memory(buf.ptr, 64) == int(mpcomm.MPCommError.ERR_CONTEXT)
    assert c.put_async(buf.ptr, "x", 0, 64) == mpcomm.INVALID_TRANSFER_HANDLE
    assert c.wait_transfer(12345, 0) == int(mpcomm.MPCommError.ERR_INVALID_HANDLE)
    assert c.is_transfer_complete(12345)  # unknown handle counts as complete


def test_put_get_roundtrip(pair):
    a, b = pair
    n = 3 << 20
    t = Buf(n)
    s = Buf(n, os.urandom(n))
    connect(a, b, t, n)
    assert a.register_memory(s.ptr, n) == 0
    h = a.put_async(s.ptr, "B", t.ptr, n)
    assert h != 0 and a.wait_transfer(h, 10000) == 0
    r = a.get_transfer_result(h)
    assert r["error_code"] == 0 and r["bytes_transferred"] == n and r["elapsed_ms"] >= 0
    a.release_transfer(h)
    assert t.bytes() == s.bytes()
    d = Buf(n)
    assert a.register_memory(d.ptr, n) == 0
    h = a.get_async(d.ptr, "B", t.ptr, n)
    assert a.wait_transfer(h) == 0
    a.release_transfer(h)
    assert d.bytes() == s.bytes()
    assert a.get_nic_completed_bytes() == 2 * n
    per_rail = a.get_rail_completed_bytes()
    assert len(per_rail) == a.get_num_nics() and sum(per_rail) == 2 * n


def test_scatter_gather_broadcast(pair):
    a, b = pair
    seg, hosts = 100_000, 3
    t = Buf(seg * hosts)
    connect(a, b, t, seg * hosts)
    s = Buf(seg * hosts, os.urandom(seg * hosts))
    assert a.register_memory(s.ptr, seg * hosts) == 0
    raddrs = [t.ptr + (hosts - 1 - i) * seg for i in range(hosts)]
    h = a.scatter_async(s.ptr, ["B"] * hosts, raddrs, [seg] * hosts)
    assert a.wait_transfer(h) == 0
    a.release_transfer(h)
    for i in range(hosts):
        assert t.bytes((hosts - 1 - i) * seg, seg) == s.bytes(i * seg, seg)
    g = Buf(seg * hosts)
    assert a.register_memory(g.ptr, seg * hosts) == 0
    h = a.mp_replicate_async("gather", ["B"] * hosts, g.ptr, raddrs, [seg] * hosts)
    assert a.wait_transfer(h) == 0
    a.release_transfer(h)
    assert g.bytes() == s.bytes()
    # broadcast one segment to all three slots
    h = a.broadcast_async(s.ptr, seg, ["B"] * hosts, [t.ptr + i * seg for i in range(hosts)])
    assert a.wait_transfer(h) == 0
    a.release_transfer(h)
    for i in range(hosts):
        assert t.bytes(i * seg, seg) == s.bytes(0, seg)


@pytest.mark.parametrize("fused", ["1", "0"])
def test_broadcast_fused_and_per_destination(lo_env, monkeypatch, fused):
    """broadcast_async gives the same bytes at every destination whether the
    rail writes all of them in one operation per chunk (fused) or one WR per
    destination; a rail that fails a fused chunk is quarantined and the rest
    of the broadcast moves to a healthy rail."""
    monkeypatch.setenv("MPCOMM_FUSED_BROADCAST", fused)
    monkeypatch.setenv("MPCOMM_MAX_RDMA_TRANSFER_SIZE", str(64 << 10))
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0 and b.start_accept_thread() == 0
    try:
        seg, hosts = 300_000, 4
        t = Buf(seg * hosts)
        connect(a, b, t, seg * hosts)
        s = Buf(seg, os.urandom(seg))
        assert a.register_memory(s.ptr, seg) == 0
        rails = a.get_active_devices()
        # One completion error on every rail but the last.
        for i in range(len(rails) - 1):
            assert mpcomm._native._lo_inject_wc_errors(a.get_gid(i), 1) == 0
        h = a.broadcast_async(s.ptr, seg, ["B"] * hosts, [t.ptr + i * seg for i in range(hosts)])
        assert a.wait_transfer(h, 30000) == 0
        r = a.get_transfer_result(h)
        a.release_transfer(h)
        assert r["bytes_transferred"] == seg * hosts
        for i in range(hosts):
            assert t.bytes(i * seg, seg) == s.bytes(), i
    finally:
        a.shutdown()
        b.shutdown()


def test_pcie_affinity_self_check_without_gpus(lo_env):
    """The GPU <-> rail affinity table has a row per visible GPU; none here."""
    c = mpcomm.MPComm()
    assert c.init("aff") == 0
    assert c.get_pcie_affinity_self_check() == []
    c.shutdown()


def test_staging_refuses_unmapped_local_range(pair):
    """An unregistered local range that is neither device memory nor mapped
    host memory is refused at submit (no handle, nothing touched)."""
    a, b = pair
    t = Buf(1 << 20)
    connect(a, b, t, 1 << 20)
    libc = ctypes.CDLL(None)
    libc.mmap.restype = ctypes.c_void_p
    libc.mmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_long]
    libc.munmap.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    addr = libc.mmap(None, 1 << 20, 3, 0x22, -1, 0)  # PROT_READ|WRITE, MAP_PRIVATE|ANONYMOUS
    assert addr and addr != ctypes.c_void_p(-1).value
    assert libc.munmap(addr, 1 << 20) == 0  # the range is unmapped from here on
    assert a.put_async(addr, "B", t.ptr, 1 << 20) == mpcomm.INVALID_TRANSFER_HANDLE
    assert a.get_async(addr, "B", t.ptr, 1 << 20) == mpcomm.INVALID_TRANSFER_HANDLE


def test_staging_config1_put_get_crc(pair):
    """Config 1: 64 x 1 MiB host->host PUT then GET through the staging pool."""
    import random

    a, b = pair
    nb, bs = 64, 1 << 20
    rng = random.Random(0)
    payload = bytes(rng.getrandbits(8) for _ in range(4096)) * (nb * bs // 4096)
    t = Buf(nb * bs)
    connect(a, b, t, nb * bs)
    src = Buf(nb * bs, payload)  # NOT registered: staging path
    hs = [a.put_async(src.ptr + i * bs, "B", t.ptr + i * bs, bs) for i in range(nb)]
    assert all(hs)
    for h in hs:
        assert a.wait_transfer(h, 30000) == 0
        a.release_transfer(h)
    back = Buf(nb * bs)
    hs = [a.get_async(back.ptr + i * bs, "B", t.ptr + i * bs, bs) for i in range(nb)]
    for h in hs:
        assert a.wait_transfer(h, 30000) == 0
        a.release_transfer(h)
    for i in range(nb):
        want = zlib.crc32(payload[i * bs:(i + 1) * bs])
        assert mpcomm.ops.crc32_host(back.bytes(i * bs, bs)) == want


def test_wait_timeout_and_pending_result(pair):
    a, b = pair
    n = 1 << 20
    t = Buf(n)
    connect(a, b, t, n)
    s = Buf(n)
    assert a.register_memory(s.ptr, n) == 0
    for i in range(a.get_num_nics()):
        mpcomm._native._lo_set_wr_delay_us(a.get_gid(i), 200_000)
    h = a.put_async(s.ptr, "B", t.ptr, n)
    assert a.wait_transfer(h, 10) == int(mpcomm.MPCommError.ERR_TIMEOUT)
    assert not a.is_transfer_complete(h)
    assert a.get_transfer_result(h)["error_code"] == int(mpcomm.MPCommError.ERR_PENDING)
    for i in range(a.get_num_nics()):
        mpcomm._native._lo_set_wr_delay_us(a.get_gid(i), 0)
    assert a.wait_transfer(h, 20000) == 0
    a.release_transfer(h)


def test_injected_wc_errors_repost_on_healthy_rail(pair, monkeypatch):
    a, b = pair
    n = 4 << 20
    t = Buf(n)
    connect(a, b, t, n)
    s = Buf(n, os.urandom(n))
    assert a.register_memory(s.ptr, n) == 0
    assert a.get_num_nics() == 2
    mpcomm._native._lo_inject_wc_errors(a.get_gid(0), 3)
    h = a.put_async(s.ptr, "B", t.ptr, n)
    assert a.wait_transfer(h, 20000) == 0  # chunks re-posted on lo_1
    a.release_transfer(h)
    assert t.bytes() == s.bytes()


def test_all_rails_down_fails_transfer(pair):
    a, b = pair
    n = 1 << 20
    t = Buf(n)
    connect(a, b, t, n)
    s = Buf(n)
    assert a.register_memory(s.ptr, n) == 0
    for i in range(a.get_num_nics()):
        mpcomm._native._lo_set_port_active(a.get_gid(i), False)
    h = a.put_async(s.ptr, "B", t.ptr, n)
    assert a.wait_transfer(h, 20000) == int(mpcomm.MPCommError.ERR_TRANSFER)
    a.release_transfer(h)


def test_publish_registry_and_rkeys(pair):
    a, b = pair
    x, y = Buf(4096), Buf(8192)
    assert b.publish_buffer(x.ptr, 4096) == int(mpcomm.MPCommError.ERR_MEMORY)  # not registered
    assert b.register_memory(x.ptr, 4096) == 0 and b.register_memory(y.ptr, 8192) == 0
    assert b.publish_buffer(x.ptr, 4096, (7 << 16) | 1) == 0  # numa tag overloaded by callers
    assert b.publish_buffer(y.ptr, 8192, 0) == 0
    assert b.get_published_buffer_count() == 2
    assert b.publish_buffer(x.ptr, 4096, 3) == 0  # republish updates
    assert b.get_published_buffer_count() == 2
    info = b.get_published_buffer_info()["buffers"]
    assert info[0]["numa_node"] == 3 and len(info[0]["rkeys"]) == b.get_num_nics()
    assert b.get_all_rkeys(x.ptr) == info[0]["rkeys"]
    port = b.get_tcp_port()
    assert a.connect("B", "127.0.0.1", port) == 0
    e = a.query_remote_buffer_by_numa("B", "127.0.0.1", port, 0)
    assert e["addr"] == y.ptr
    e = a.query_remote_buffer_by_numa("B", "127.0.0.1", port, 42)  # falls back to the first
    assert e["addr"] == x.ptr
    assert b.unpublish_buffer(x.ptr) == 0 and b.unpublish_buffer(x.ptr) != 0
    b.unpublish_all_buffers()
    assert b.get_published_buffer_count() == 0
    assert a.query_remote_buffers("B", "127.0.0.1", port) == {}


def test_update_remote_memory_info(pair):
    a, b = pair
    n = 65536
    t = Buf(n)
    assert b.register_memory(t.ptr, n) == 0
    port = b.get_tcp_port()
    assert a.connect("B", "127.0.0.1", port) == 0  # no query: rkeys unknown
    s = Buf(n, os.urandom(n))
    assert a.register_memory(s.ptr, n) == 0
    assert a.update_remote_memory_info("B", [1]) == int(mpcomm.MPCommError.ERR_INVALID_ARG)
    assert a.update_remote_memory_info("B", b.get_all_rkeys(t.ptr)) == 0
    h = a.put_async(s.ptr, "B", t.ptr, n)
    assert a.wait_transfer(h, 10000) == 0
    a.release_transfer(h)
    assert t.bytes() == s.bytes()


def test_throttle_latency_and_qos_flags(pair):
    a, b = pair
    a.set_nic_throttle(1, 65536)
    lat = a.get_throttle_latency()
    assert lat["set_ns"] > 0 and set(lat) >= {"worker_us", "drain_us", "effective_us", "drained"}
    a.clear_nic_throttle()
    assert not a.is_h2d_qos_enabled()
    a.enable_h2d_qos(1 << 30)
    assert a.is_h2d_qos_enabled()
    a.set_h2d_qos_policy(0)
    a.disable_h2d_qos()
    assert not a.is_h2d_qos_enabled()
    assert a.get_pcie_domain_stats() == [] and not a.is_pcie_domain_stat_enabled()


def test_topology_introspection(pair):
    a, _ = pair
    topo = a.get_numa_topology()
    assert topo and topo[0]["numa_node"] == 0
    assert {n["nic_name"] for n in a.get_nic_topology()} == set(a.get_active_devices())
    assert a.get_nic_numa_node(a.get_device_name(0)) >= 0
    assert a.get_local_nic_indices_for_numa(0) == list(range(a.get_num_nics()))
    buf = Buf(4096)
    assert a.get_numa_node_for_addr(buf.ptr) >= -1


def test_handle_recycling(pair):
    a, b = pair
    t = Buf(4096)
    connect(a, b, t, 4096)
    s = Buf(4096)
    assert a.register_memory(s.ptr, 4096) == 0
    seen = set()
    for _ in range(200):
        h = a.put_async(s.ptr, "B", t.ptr, 4096)
        assert a.wait_transfer(h) == 0
        a.release_transfer(h)
        seen.add(h)
    assert len(seen) <= 2  # released handles are reused


def test_kernel_trace_off_by_default():
    assert mpcomm._native.kernel_trace_slots() == 0
    assert mpcomm._native.kernel_trace() == []
    assert mpcomm.MPComm.get_kernel_launch_count() >= 0


@pytest.mark.parametrize("name", ["test_core", "test_engine", "test_engine_san", "test_engine_tsan", "test_core_san",
                                  "test_core_tsan"])
def test_native_binaries(name):
    """Core unit tests, the multi-threaded engine stress, and both built
    with AddressSanitizer + UBSan (memory errors in the engine's lifetime and
    completion protocol abort with a report) and with ThreadSanitizer (any
    data race between the submitting threads, the worker, the publish/query
    thread and the throttle toggler, or in the descriptor server and the
    multicast-group protocol threads, fails it)."""
    exe = os.path.join(ROOT, "tests", "native", "bin", name)
    if name.endswith("_tsan") and not os.path.exists(exe):
        pytest.skip("toolchain has no ThreadSanitizer runtime")
    assert os.path.exists(exe), "native tests not built (run __graft_entry__.build())"
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0:abort_on_error=1", MPCOMM_LOG_LEVEL="1",
               TSAN_OPTIONS="halt_on_error=1:exitcode=66:second_deadlock_stack=1",
               MPCOMM_STRESS_ROUNDS="40" if name == "test_engine_tsan" else "12")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "ERROR: AddressSanitizer" not in r.stderr
    assert "WARNING: ThreadSanitizer" not in r.stderr


def test_type_stub_covers_the_native_module():
    """mpcomm/_mpcomm.pyi declares every public method of MPComm and every
    module function, so IDEs and type checkers see the whole API."""
    import ast

    import mpcomm

    tree = ast.parse(open(os.path.join(ROOT, "mpcomm", "_mpcomm.pyi")).read())
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "MPComm")
    stub_methods = {f.name for f in cls.body if isinstance(f, ast.FunctionDef)}
    native = {n for n in dir(mpcomm._mpcomm.MPComm) if not n.startswith("_")}
    assert native <= stub_methods, sorted(native - stub_methods)
    stub_funcs = {f.name for f in tree.body if isinstance(f, ast.FunctionDef)}
    funcs = {n for n in dir(mpcomm._mpcomm) if not n.startswith("_") and callable(getattr(mpcomm._mpcomm, n))
             and n not in ("MPComm", "MPCommError")}
    assert funcs <= stub_funcs, sorted(funcs - stub_funcs)


def test_sock_fabric_marks_data_connections_with_dscp():
    """MPCOMM_ROCE_DSCP marks the sock fabric's TCP data connections (both
    ends) with that DSCP, as it sets the traffic class of RDMA QPs."""
    code = r"""
import ctypes, os, mpcomm
n = 1 << 16
a, b = mpcomm.MPComm(), mpcomm.MPComm()
assert a.init("A") == 0 and b.init("B") == 0 and b.start_accept_thread() == 0
t = ctypes.create_string_buffer(n); s = ctypes.create_string_buffer(os.urandom(n), n)
assert b.register_memory(ctypes.addressof(t), n) == 0 and b.publish_buffer(ctypes.addressof(t), n) == 0
assert a.register_memory(ctypes.addressof(s), n) == 0
port = b.get_tcp_port()
assert a.connect("B", "127.0.0.1", port) == 0 and a.query_remote_buffers("B", "127.0.0.1", port)
h = a.put_async(ctypes.addressof(s), "B", ctypes.addressof(t), n)
assert a.wait_transfer(h, 10000) == 0 and t.raw == s.raw
a.release_transfer(h); a.shutdown(); b.shutdown()
print("dscp case ok")
"""
    env = dict(os.environ, MPCOMM_FABRIC="sock", MPCOMM_ROCE_DSCP="46", MPCOMM_LOG_LEVEL="3", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                       timeout=120)
    assert r.returncode == 0 and "dscp case ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
    marked = r.stdout.count("traffic class 0xb8 (DSCP 46)")
    assert marked >= 2, r.stdout[-3000:]  # initiator and target ends
    assert "cannot set traffic class" not in r.stderr


def test_sock_fabric_rejected_write_is_drained_without_allocating_its_length():
    """A write that fails the sock fabric's rkey check is answered with a
    remote-access error and its payload drained in bounded pieces: a peer
    announcing a 3 GiB payload cannot make the target allocate 3 GiB, and
    the connection keeps serving requests."""
    import socket
    import struct

    code = r"""
import os, socket, struct, mpcomm
def rss():
    for line in open("/proc/self/status"):
        if line.startswith("VmRSS:"):
            return int(line.split()[1]) * 1024
b = mpcomm.MPComm()
assert b.init("B") == 0
gid = b.get_gid(0)                       # sock:<ip>:<port>:<n>
_, ip, port, _ = gid.split(":")
s = socket.create_connection((ip, int(port)))
s.sendall(struct.pack("<III", 0x4D505348, 0, 0))          # hello
def req(op, rkey, length, addr=0):
    return struct.pack("<IIIIQ", 0x4D505352, op, rkey, length, addr)
def status():
    b_ = b""
    while len(b_) < 4:
        c = s.recv(4 - len(b_)); assert c; b_ += c
    return struct.unpack("<i", b_)[0]
s.sendall(req(0, 0xBAD, 1 << 20) + os.urandom(1 << 20))   # rejected 1 MiB write
assert status() != 0
s.sendall(req(1, 0xBAD, 4096))                           # rejected read: status only
assert status() != 0
before = rss()
s.sendall(req(0, 0xBAD, 3 << 30) + b"x" * 4096)          # 3 GiB announced, 4 KiB sent
import time; time.sleep(0.5)
grown = rss() - before
s.close()
b.shutdown()
assert grown < (256 << 20), grown
print("drain ok", grown)
"""
    env = dict(os.environ, MPCOMM_FABRIC="sock", MPCOMM_LOG_LEVEL="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0 and "drain ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_multicast_group_bounded_without_peers():
    """createMulticastGroup / joinMulticastGroup fail within their timeout:
    a joiner with no creator gets MPCOMM_ERR_CONNECTION, a creator on a
    host without a multicast-capable GPU MPCOMM_ERR_DEVICE (with one, it
    times out waiting for the second member), bad arguments INVALID_ARG."""
    import time

    from mpcomm import _native
    name = f"mpcomm-cpu-test-{os.getpid()}"
    t0 = time.monotonic()
    err, g = _native.multicast_group(name, 1 << 20, 2, False, 300)
    assert err == -4 and g == {} and time.monotonic() - t0 < 10
    err, g = _native.multicast_group(name, 1 << 20, 2, True, 300)
    assert err in (-1, -4) and g == {}
    assert _native.multicast_group(name, 1 << 20, 1, True, 300)[0] == -7
    assert _native.multicast_group(name, 0, 2, False, 300)[0] == -7
    assert _native.multicast_group("", 1 << 20, 2, False, 300)[0] == -7


def test_nvls_group_from_name_fails_cleanly_without_gpus():
    """NvlsGroup.from_name raises (never hangs) where no group can form: on a
    host without multicast-capable GPUs the creator fails at once, a joiner
    after its timeout."""
    import time

    from mpcomm import parallel
    name = f"mpcomm-cpu-from-name-{os.getpid()}"
    t0 = time.monotonic()
    for create in (True, False):
        with pytest.raises(RuntimeError):
            parallel.NvlsGroup.from_name(name, 1 << 20, 2, create=create, timeout_ms=300)
    assert time.monotonic() - t0 < 10


def test_bench_comparators_fail_cleanly_without_gpus():
    """The bench comparators report failure, never crash, on a host without
    a usable GPU: the copy engine call returns a CUDA error and the
    round-trip floor an empty list."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from mpcomm import _native
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    assert _native.copy_engine_async(p, p + 2048, 1024, 0) != 0
    assert _native.copy_roundtrip_us(p, p + 2048, 1024, 4) == []
    err, segs = _native.vmm_segments(p, 4096)
    assert err != 0 and segs == []
