"""Staging pool with device memory: PUT/GET from HBM that was never
registered goes through slabs in the same GPU's HBM, filled and drained by
the sm_100a bulk-copy kernel, then through the zero-copy engine."""
import pytest
import torch

import mpcomm

pytestmark = pytest.mark.gpu


@pytest.fixture
def comm_pool(monkeypatch):
    monkeypatch.setenv("MPCOMM_LOG_LEVEL", "1")
    monkeypatch.setenv("MPCOMM_STAGING_DEVICE_SLAB_BYTES", str(4 << 20))  # several pieces per transfer
    monkeypatch.setenv("MPCOMM_STAGING_SLABS", "4")
    torch.cuda.set_device(0)
    size = 48 << 20
    pool = torch.zeros(size, dtype=torch.uint8).pin_memory()
    c = mpcomm.MPComm()
    assert c.init("staging-gpu") == 0 and c.start_accept_thread() == 0
    assert c.get_fabric_name() == "nvl"
    assert c.register_memory(pool.data_ptr(), size) == 0
    assert c.publish_buffer(pool.data_ptr(), size) == 0
    port = c.get_tcp_port()
    assert c.connect("pool", "127.0.0.1", port) == 0
    assert c.query_remote_buffers("pool", "127.0.0.1", port)
    yield c, pool
    c.shutdown()


def _wait(c, h):
    assert h != mpcomm.INVALID_TRANSFER_HANDLE
    assert c.wait_transfer(h, 60000) == 0
    r = c.get_transfer_result(h)
    c.release_transfer(h)
    return r


def test_put_get_from_unregistered_hbm(comm_pool):
    c, pool = comm_pool
    n = 40 << 20
    g = torch.Generator(device="cuda").manual_seed(5)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)  # not registered
    back = torch.zeros(n, dtype=torch.uint8, device="cuda")  # not registered
    torch.cuda.synchronize()
    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    r = _wait(c, c.put_async(src.data_ptr(), "pool", pool.data_ptr(), n))
    assert r["bytes_transferred"] == n
    assert torch.equal(pool[:n], src.cpu())
    r = _wait(c, c.get_async(back.data_ptr(), "pool", pool.data_ptr(), n))
    assert r["bytes_transferred"] == n
    torch.cuda.synchronize()
    assert torch.equal(back, src)
    # 10 pieces of 4 MiB each way: a stage copy and a fabric copy per piece.
    assert mpcomm.MPComm.get_kernel_launch_count() - launches0 >= 40


def test_unaligned_staged_ranges(comm_pool):
    """Odd offsets and a length that is not a multiple of 16 (the copy
    kernel's inline path for unaligned tiles)."""
    c, pool = comm_pool
    n = (9 << 20) + 5
    base = torch.randint(0, 256, (n + 64,), dtype=torch.uint8, device="cuda")
    src_ptr = base.data_ptr() + 3
    r = _wait(c, c.put_async(src_ptr, "pool", pool.data_ptr() + 7, n))
    assert r["bytes_transferred"] == n
    assert torch.equal(pool[7:7 + n], base[3:3 + n].cpu())
    out = torch.zeros(n + 64, dtype=torch.uint8, device="cuda")
    _wait(c, c.get_async(out.data_ptr() + 11, "pool", pool.data_ptr() + 7, n))
    torch.cuda.synchronize()
    assert torch.equal(out[11:11 + n], base[3:3 + n])
    assert int(out[:11].sum()) == 0 and int(out[11 + n:].sum()) == 0


def test_staged_range_past_allocation_refused(comm_pool):
    """A device range that runs past the end of its allocation is refused at
    submit (no handle, nothing copied)."""
    c, pool = comm_pool
    t = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    seg = next(s for s in torch.cuda.memory_snapshot()
               if s["address"] <= t.data_ptr() < s["address"] + s["total_size"])
    end = seg["address"] + seg["total_size"]
    h = c.put_async(end - 4096, "pool", pool.data_ptr(), 64 << 10)
    assert h == mpcomm.INVALID_TRANSFER_HANDLE
