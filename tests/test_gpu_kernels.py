"""GPU tests of the sm_100a kernels against plain PyTorch / zlib references.

Every comparison is bit-exact: these kernels move bytes. Cases mirror the
reference's user_examples/test_tma.py (gather, per-block scatter, round
trip, alignment sweep 16..1024 B) plus the B200 additions (64 KiB pages,
index bound check, bounded waits, CRC-32, fabric copies).
"""
import random
import time
import zlib

import pytest
import torch

pytestmark = pytest.mark.gpu

import mpcomm  # noqa: E402
from mpcomm import ops  # noqa: E402


def _pool(pages, bs, seed=0, pinned=True):
    g = torch.Generator().manual_seed(seed)
    t = torch.randint(0, 256, (pages, bs), dtype=torch.uint8, generator=g)
    return t.pin_memory() if pinned else t.cuda()


@pytest.mark.parametrize("bs", [16, 272, 1024, 4096, 65536, 65536 + 48])
@pytest.mark.parametrize("mode", [ops.MODE_AUTO, ops.MODE_SM, ops.MODE_TMA])
def test_paged_gather_bitexact(bs, mode):
    pages, n = 64, 40
    pool = _pool(pages, bs, seed=bs)
    idx = torch.randperm(pages, generator=torch.Generator().manual_seed(1))[:n].cuda()
    out = ops.paged_gather(pool, idx, mode=mode)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), pool[idx.cpu()])


@pytest.mark.parametrize("bs", [16, 1040, 65536])
@pytest.mark.parametrize("mode", [ops.MODE_AUTO, ops.MODE_SM, ops.MODE_TMA])
def test_paged_scatter_bitexact(bs, mode):
    pages, n = 48, 20
    pool = _pool(pages, bs, seed=3)
    before = pool.clone()
    idx = torch.randperm(pages, generator=torch.Generator().manual_seed(2))[:n].cuda()
    src = torch.randint(0, 256, (n, bs), dtype=torch.uint8, device="cuda")
    ops.paged_scatter(src, idx, pool, mode=mode)
    torch.cuda.synchronize()
    expect = before.clone()
    expect[idx.cpu()] = src.cpu()
    assert torch.equal(pool, expect)


def test_gather_scatter_round_trip_device_pool():
    pages, bs, n = 128, 8192, 128
    pool = _pool(pages, bs, seed=5, pinned=False)
    idx = torch.randperm(pages, device="cuda")
    staged = ops.paged_gather(pool, idx)
    back = torch.zeros_like(pool)
    ops.paged_scatter(staged, idx, back)
    torch.cuda.synchronize()
    assert torch.equal(back, pool)


@pytest.mark.parametrize("offset", [1, 4, 8, 12])
def test_sm_mode_handles_unaligned_blocks(offset):
    pages, bs, n = 16, 1000, 10
    raw = torch.randint(0, 256, (pages * bs + 64,), dtype=torch.uint8).pin_memory()
    base = raw.data_ptr() + offset
    idx = torch.randperm(pages)[:n].cuda()
    out = torch.empty(n * bs, dtype=torch.uint8, device="cuda")
    err, _, path = mpcomm._native.paged_gather(base, pages, idx.data_ptr(), out.data_ptr(), n, bs,
                                               ops.MODE_AUTO, 0, torch.cuda.current_stream().cuda_stream)
    assert err == 0 and path == 2  # AUTO falls back to the vector kernel
    torch.cuda.synchronize()
    ref = raw[offset:offset + pages * bs].view(pages, bs)[idx.cpu()].reshape(-1)
    assert torch.equal(out.cpu(), ref)


def test_tma_mode_rejects_misaligned():
    pool = torch.zeros(4 * 1024 + 16, dtype=torch.uint8).pin_memory()
    idx = torch.zeros(2, dtype=torch.int64, device="cuda")
    out = torch.empty(2 * 1000, dtype=torch.uint8, device="cuda")
    err, _, _ = mpcomm._native.paged_gather(pool.data_ptr(), 4, idx.data_ptr(), out.data_ptr(), 2, 1000,
                                            ops.MODE_TMA, 0, 0)
    assert err != 0  # misaligned block size: refused, not silently rerouted


def test_out_of_range_index_is_skipped():
    pages, bs = 8, 4096
    pool = _pool(pages, bs)
    idx = torch.tensor([0, 99, 2, -1], dtype=torch.int64, device="cuda")
    out = torch.full((4, bs), 7, dtype=torch.uint8, device="cuda")
    ops.paged_gather(pool, idx, out=out)
    torch.cuda.synchronize()
    o = out.cpu()
    assert torch.equal(o[0], pool[0]) and torch.equal(o[2], pool[2])
    assert (o[1] == 7).all() and (o[3] == 7).all()  # bad indices never touch memory


@pytest.mark.parametrize("n,bs", [(5, 1), (5, 15), (5, 4096), (5, (512 << 10) + 3), (5, 3 << 20),
                                  (3, (5 << 20) + 16 * 37), (2, 96 << 20), (700, 4096 + 512 + 48)])
def test_crc32_matches_zlib(n, bs):
    """Spans of rows, the two-chain split, row tails, unaligned blocks (odd
    block sizes) and multi-span blocks against zlib."""
    data = torch.randint(0, 256, (n * bs,), dtype=torch.uint8, generator=torch.Generator().manual_seed(bs))
    got = ops.crc32_blocks(data.cuda(), n).cpu().tolist()
    raw = data.numpy().tobytes()
    want = [zlib.crc32(raw[i * bs:(i + 1) * bs]) for i in range(n)]
    assert [g & 0xFFFFFFFF for g in got] == want


def test_copy_spans_mixed_alignment():
    src = torch.randint(0, 256, (1 << 22,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros_like(src)
    spans = [(0, 0, 1 << 20), ((1 << 20) + 3, (1 << 20) + 3, 65537), (2 << 20, (3 << 20) + 5, 1000)]
    ops.copy_spans([src.data_ptr() + a for a, _, _ in spans], [dst.data_ptr() + b for _, b, _ in spans],
                   [n for _, _, n in spans])
    torch.cuda.synchronize()
    for a, b, n in spans:
        assert torch.equal(dst[b:b + n], src[a:a + n])


@pytest.mark.parametrize("mode", [ops.MODE_AUTO, ops.MODE_SM])
def test_copy_gate_pauses_then_fails_open(mode):
    """A copy given a QoS gate pauses before each tile while the gate word
    is non-zero, for at most gate_budget_ns per pipeline, then finishes the
    copy anyway (bit-exact); with the gate at zero it does not pause."""
    src = torch.randint(0, 256, (8 << 20,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros_like(src)
    gate = torch.zeros(32, dtype=torch.int32, device="cuda")
    budget = 40_000_000  # 40 ms

    def timed():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.copy_spans([src.data_ptr()], [dst.data_ptr()], [src.numel()], max_ctas=8, mode=mode,
                       gate=gate.data_ptr(), gate_budget_ns=budget)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    timed()  # warm-up
    open_ms = timed()
    assert open_ms < 20, open_ms
    gate[0] = 1
    dst.zero_()
    held_ms = timed()
    assert torch.equal(dst, src)
    assert 0.9 * budget / 1e6 <= held_ms < 20 * budget / 1e6, held_ms


def test_bounded_flag_wait_times_out_and_context_survives():
    """A wait on a flag nothing sets ends with a status bit, not a hang."""
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.wait_flag(flag.data_ptr(), 1, budget_ns=50_000_000, status_ptr=status.data_ptr())
    torch.cuda.synchronize()
    assert status.item() & 8  # kStatusFlagTimeout
    # The context is still usable.
    x = torch.arange(1024, device="cuda")
    assert int(x.sum().item()) == 1024 * 1023 // 2
    flag.fill_(1)
    status.zero_()
    ops.wait_flag(flag.data_ptr(), 1, budget_ns=50_000_000, status_ptr=status.data_ptr())
    torch.cuda.synchronize()
    assert status.item() == 0


def test_pxn_forward_local_flag():
    """Fused gather + forward into a (here local) destination with a done flag."""
    pages, bs, n = 32, 65536, 12
    pool = _pool(pages, bs, seed=9)
    idx = torch.randperm(pages)[:n].cuda()
    dst = torch.empty((n, bs), dtype=torch.uint8, device="cuda")
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.pxn_gather_forward(pool.data_ptr(), pages, idx, dst.data_ptr(), bs, done_flag=flag.data_ptr(),
                           flag_value=77, counter=ctr.data_ptr())
    torch.cuda.synchronize()
    assert flag.item() == 77 and ctr.item() == 0
    assert torch.equal(dst.cpu(), pool[idx.cpu()])


def test_gather_bcast_p2p_local_destinations_and_flags():
    """Fused gather + fan-out (P2P sink) to two local buffers: both receive
    the gathered pages bit-exact, both flags are published, the counter
    resets, a repeat launch works, and an out-of-range index is skipped and
    flagged."""
    pages, bs, n = 48, 65536 + 4096, 20
    pool = _pool(pages, bs, seed=21)
    idx = torch.randperm(pages, generator=torch.Generator().manual_seed(3))[:n].cuda()
    a = torch.zeros((n, bs), dtype=torch.uint8, device="cuda")
    b = torch.zeros((n, bs), dtype=torch.uint8, device="cuda")
    flags = torch.zeros(2, dtype=torch.int64, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    expect = pool[idx.cpu()]
    for rep in (1, 2):
        ops.gather_bcast(pool.data_ptr(), pages, idx, bs, dst_ptrs=[a.data_ptr(), b.data_ptr()],
                         flags=[flags.data_ptr(), flags.data_ptr() + 8], flag_value=10 + rep,
                         counter=ctr.data_ptr(), status_ptr=status.data_ptr())
        torch.cuda.synchronize()
        assert flags.tolist() == [10 + rep, 10 + rep] and ctr.item() == 0 and status.item() == 0
        assert torch.equal(a.cpu(), expect) and torch.equal(b.cpu(), expect)
    bad = idx.clone()
    bad[3] = pages + 5
    a.fill_(9)
    ops.gather_bcast(pool.data_ptr(), pages, bad, bs, dst_ptrs=[a.data_ptr()], status_ptr=status.data_ptr())
    torch.cuda.synchronize()
    assert status.item() & 4  # kStatusBadIndex
    got = a.cpu()
    assert (got[3] == 9).all()
    keep = [i for i in range(n) if i != 3]
    assert torch.equal(got[keep], expect[keep])


def test_gather_bcast_rejects_misaligned():
    pool = _pool(8, 4096)
    idx = torch.arange(4, device="cuda")
    out = torch.zeros(4 * 4096 + 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        ops.gather_bcast(pool.data_ptr(), 8, idx, 4096, dst_ptrs=[out.data_ptr() + 8])
    with pytest.raises(RuntimeError):
        ops.gather_bcast(pool.data_ptr(), 8, idx, 4088, dst_ptrs=[out.data_ptr()])


def _fabric_pair():
    comm = mpcomm.MPComm()
    assert comm.init("gpu-test") == 0
    assert comm.get_fabric_name() == "nvl"
    assert comm.start_accept_thread() == 0
    return comm


@pytest.mark.parametrize("nbytes", [4096, (1 << 20) + 13, 96 << 20])
def test_fabric_put_get_hbm_dram(nbytes):
    comm = _fabric_pair()
    try:
        src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
        back = torch.zeros_like(src)
        pool = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
        for t in (src, back, pool):
            assert comm.register_memory(t.data_ptr(), t.numel()) == 0
        assert comm.publish_buffer(pool.data_ptr(), nbytes) == 0
        port = comm.get_tcp_port()
        assert comm.connect("pool", "127.0.0.1", port) == 0
        assert comm.query_remote_buffers("pool", "127.0.0.1", port)
        torch.cuda.synchronize()
        h = comm.put_async(src.data_ptr(), "pool", pool.data_ptr(), nbytes)
        assert comm.wait_transfer(h, 60000) == 0
        r = comm.get_transfer_result(h)
        assert r["bytes_transferred"] == nbytes
        comm.release_transfer(h)
        h = comm.get_async(back.data_ptr(), "pool", pool.data_ptr(), nbytes)
        assert comm.wait_transfer(h, 60000) == 0
        comm.release_transfer(h)
        torch.cuda.synchronize()
        assert torch.equal(pool.cuda(), src)
        assert torch.equal(back, src)
    finally:
        comm.shutdown()


def test_fabric_scatter_gather_hbm_to_hbm():
    comm = _fabric_pair()
    try:
        n, seg = 4, (8 << 20) + 16
        src = torch.randint(0, 256, (n * seg,), dtype=torch.uint8, device="cuda")
        remote = torch.zeros(n * seg, dtype=torch.uint8, device="cuda")
        back = torch.zeros_like(src)
        for t in (src, remote, back):
            assert comm.register_memory(t.data_ptr(), t.numel()) == 0
        assert comm.publish_buffer(remote.data_ptr(), remote.numel()) == 0
        port = comm.get_tcp_port()
        assert comm.connect("peer", "127.0.0.1", port) == 0
        assert comm.query_remote_buffers("peer", "127.0.0.1", port)
        torch.cuda.synchronize()
        hosts = ["peer"] * n
        # scatter segments in reverse order
        raddrs = [remote.data_ptr() + (n - 1 - i) * seg for i in range(n)]
        h = comm.scatter_async(src.data_ptr(), hosts, raddrs, [seg] * n)
        assert comm.wait_transfer(h, 60000) == 0
        comm.release_transfer(h)
        h = comm.gather_async(back.data_ptr(), hosts, raddrs, [seg] * n)
        assert comm.wait_transfer(h, 60000) == 0
        comm.release_transfer(h)
        torch.cuda.synchronize()
        assert torch.equal(back, src)
        for i in range(n):
            assert torch.equal(remote[(n - 1 - i) * seg:(n - i) * seg], src[i * seg:(i + 1) * seg])
    finally:
        comm.shutdown()


def test_h2d_qos_pauses_read_posts_during_gather_windows(monkeypatch):
    """A background GET (pool -> HBM) shares the PCIe link with tmaGather.
    With QoS at rate 0 its chunk posts are deferred while a gather kernel's
    window is open (PCIe-domain defer_count rises) and it still completes
    bit-exact; posted == completed bytes at the end."""
    monkeypatch.setenv("MPCOMM_PCIE_STAT_ENABLE", "1")
    monkeypatch.setenv("MPCOMM_NVL_CHUNK_SIZE", str(1 << 20))
    comm = mpcomm.MPComm()
    assert comm.init("qos-test") == 0 and comm.start_accept_thread() == 0
    try:
        n = 512 << 20
        pool = torch.randint(0, 256, (n,), dtype=torch.uint8).pin_memory()
        dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
        for t in (pool, dst):
            assert comm.register_memory(t.data_ptr(), n) == 0
        assert comm.publish_buffer(pool.data_ptr(), n) == 0
        port = comm.get_tcp_port()
        assert comm.connect("pool", "127.0.0.1", port) == 0 and comm.query_remote_buffers("pool", "127.0.0.1", port)
        pages, bs, m = 4096, 65536, 2048
        kv = _pool(pages, bs, seed=4)
        dram = comm.map_dram_to_gpu(kv.data_ptr(), kv.numel())
        idx = torch.randperm(pages)[:m].cuda()
        out = torch.empty(m * bs, dtype=torch.uint8, device="cuda")
        comm.enable_h2d_qos(0, 0)
        assert comm.is_pcie_domain_stat_enabled()
        stream = torch.cuda.Stream()
        h = comm.get_async(dst.data_ptr(), "pool", pool.data_ptr(), n)
        while not comm.is_transfer_complete(h):
            assert comm.tma_gather(dram, idx.data_ptr(), out.data_ptr(), m, bs, 0, 0, stream.cuda_stream) == 0
            stream.synchronize()
        assert comm.wait_transfer(h, 60000) == 0
        comm.release_transfer(h)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), pool)
        assert torch.equal(out.view(m, bs).cpu(), kv[idx.cpu()])
        stats = {s["gpu"]: s for s in comm.get_pcie_domain_stats()}
        s0 = stats[torch.cuda.current_device()]
        assert s0["defer_count"] > 0, s0
        assert s0["posted_bytes"] == s0["completed_bytes"] == n and s0["in_flight_bytes"] == 0
        assert 0 < s0["in_flight_bytes_max"] <= n
        comm.reset_pcie_domain_stats()
        assert comm.get_pcie_domain_stats()[0]["post_count"] == 0
        comm.unmap_dram_from_gpu(kv.data_ptr())
    finally:
        comm.shutdown()


def test_tma_gather_api_with_mapping_and_qos_window():
    """tmaGather through MPComm with H2D QoS on: the kernel opens and closes its window."""
    comm = mpcomm.MPComm()
    assert comm.init("qos") == 0
    try:
        comm.enable_h2d_qos(0, 0)
        pages, bs, n = 256, 65536, 64
        kv = _pool(pages, bs, seed=11)
        dram = comm.map_dram_to_gpu(kv.data_ptr(), kv.numel())
        assert dram
        idx = torch.tensor(random.Random(1).sample(range(pages), n), dtype=torch.int64, device="cuda")
        out = torch.empty(n * bs, dtype=torch.uint8, device="cuda")
        assert comm.tma_gather(dram, idx.data_ptr(), out.data_ptr(), n, bs) == 0
        torch.cuda.synchronize()
        assert torch.equal(out.view(n, bs).cpu(), kv[idx.cpu()])
        assert comm.unmap_dram_from_gpu(kv.data_ptr()) == 0
    finally:
        comm.shutdown()


def test_kernel_trace_ring_records_launches():
    """MPCOMM_KERNEL_TRACE=<slots>: gather, scatter and fabric copies stamp
    their device start/end into the ring; durations agree with CUDA events
    and the ring wraps without a reset."""
    import os
    import subprocess
    import sys
    code = r"""
import torch, mpcomm
from mpcomm import ops
n_pages, bs = 512, 65536
pool = torch.randint(0, 256, (n_pages, bs), dtype=torch.uint8).pin_memory()
idx = torch.randperm(n_pages)[:256].cuda()
out = torch.empty(256 * bs, dtype=torch.uint8, device="cuda")
e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
e0.record(); ops.paged_gather(pool, idx, out); e1.record(); torch.cuda.synchronize()
ev_us = e0.elapsed_time(e1) * 1e3
ops.paged_scatter(out, idx, pool)
src = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, device="cuda"); dst = torch.empty_like(src)
ops.copy_spans([src.data_ptr()], [dst.data_ptr()], [src.numel()])
torch.cuda.synchronize()
tr = mpcomm._native.kernel_trace()
kinds = [r["kind"] for r in tr]
assert kinds[-3:] == ["h2d_gather", "h2d_scatter", "copy_batch"], kinds
g = tr[-3]
assert g["bytes"] == 256 * bs and 0 < g["duration_us"] <= ev_us * 1.05 + 5, (g, ev_us)
assert tr[-1]["bytes"] == 64 << 20 and tr[-1]["duration_us"] > 0
for _ in range(10):  # wrap the 8-slot ring
    ops.copy_spans([src.data_ptr()], [dst.data_ptr()], [1 << 20])
torch.cuda.synchronize()
tr = mpcomm._native.kernel_trace()
assert len(tr) == 8 and all(r["kind"] == "copy_batch" and r["bytes"] == 1 << 20 and r["duration_us"] > 0 for r in tr)
assert [r["seq"] for r in tr] == sorted(r["seq"] for r in tr)
mpcomm._native.kernel_trace_reset()
assert mpcomm._native.kernel_trace() == []
print("trace ok", round(g["duration_us"], 1), round(ev_us, 1))
"""
    env = dict(os.environ, MPCOMM_KERNEL_TRACE="8")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and "trace ok" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_qos_remote_pause_around_gather_windows(monkeypatch):
    """MPCOMM_QOS_REMOTE=1: B's QoS-windowed tma_gather on its GPU sends a
    pause to A over B's control channel before the kernel starts and the
    clear once the window closes; A's PUTs into B's GPU are deferred
    meanwhile and complete bit-exact, and no policy is left behind."""
    monkeypatch.setenv("MPCOMM_QOS_REMOTE", "1")
    monkeypatch.setenv("MPCOMM_NVL_CHUNK_SIZE", str(1 << 20))
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0
    try:
        assert a.start_accept_thread() == 0 and b.start_accept_thread() == 0
        n = 256 << 20
        inbox = torch.zeros(n, dtype=torch.uint8, device="cuda")
        src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
        assert b.register_memory(inbox.data_ptr(), n) == 0 and b.publish_buffer(inbox.data_ptr(), n) == 0
        assert a.register_memory(src.data_ptr(), n) == 0
        assert a.connect("B", "127.0.0.1", b.get_tcp_port()) == 0
        assert a.query_remote_buffers("B", "127.0.0.1", b.get_tcp_port())
        assert b.connect("A", "127.0.0.1", a.get_tcp_port()) == 0
        assert b.open_qos_channel("A") == 0
        b.enable_h2d_qos(0, 0)
        pages, bs, m = 4096, 65536, 2048
        kv = _pool(pages, bs, seed=9)
        dram = b.map_dram_to_gpu(kv.data_ptr(), kv.numel())
        idx = torch.randperm(pages)[:m].cuda()
        out = torch.empty(m * bs, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.Stream()
        h = a.put_async(src.data_ptr(), "B", inbox.data_ptr(), n)
        gathers = 0
        while not a.is_transfer_complete(h) and gathers < 200:
            assert b.tma_gather(dram, idx.data_ptr(), out.data_ptr(), m, bs, 0, 0, stream.cuda_stream) == 0
            stream.synchronize()
            gathers += 1
        assert a.wait_transfer(h, 60000) == 0
        a.release_transfer(h)
        torch.cuda.synchronize()
        assert torch.equal(inbox, src)
        assert torch.equal(out.view(m, bs).cpu(), kv[idx.cpu()])
        assert a.get_remote_qos_defer_count() > 0, gathers
        t0 = time.time()
        while a.get_remote_qos_policies() and time.time() - t0 < 2:
            time.sleep(0.01)
        assert a.get_remote_qos_policies() == []
        b.unmap_dram_from_gpu(kv.data_ptr())
    finally:
        b.shutdown()
        a.shutdown()


def test_copy_roundtrip_floor_copies_and_times():
    """copy_roundtrip_us (the latency bench's floor): every launch copies the
    bytes and is timed to its host-visible done word."""
    n = 64 << 10
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n, dtype=torch.uint8).pin_memory()
    us = mpcomm._native.copy_roundtrip_us(src.data_ptr(), dst.data_ptr(), n, 20)
    assert len(us) == 20 and all(0 < u < 1e6 for u in us), us
    assert torch.equal(dst, src.cpu())
