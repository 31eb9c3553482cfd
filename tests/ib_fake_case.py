"""Runs the "ib" fabric against the fake libibverbs provider (env
MPCOMM_IBVERBS_LIB) in one process: handshake with suffix pairing (mlx5_0 ->
mlx5_0 + cross-NUMA mlx5_4 is absent, so mlx5_0 <-> mlx5_0 and mlx5_1 <->
mlx5_1), buffer query, PUT/GET/scatter with byte checks. With
MPCOMM_FAULT_INJECT_* set, the QPs of rail 0 go to ERR and the transfer must
still complete (completions flush, rail 0 is quarantined, chunks re-post on
rail 1). With --gpu the buffers are B200 HBM (torch CUDA tensors): the
backend must register them through GPUDirect dma-buf
(cuMemGetHandleForAddressRange -> ibv_reg_dmabuf_mr; the fake moves their
bytes with the driver's UVA copy) and the PUT/GET must round-trip
bit-exact. Prints "ib fake ok" on success."""
import ctypes
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import mpcomm  # noqa: E402


def main():
    n = 6 << 20
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0
    assert a.get_fabric_name() == "ib", a.get_fabric_name()
    prefix = os.environ.get("FAKE_IBV_DEVICE_PREFIX", "mlx5_")
    assert a.get_active_devices() == [prefix + "0", prefix + "1"], a.get_active_devices()
    gid = a.get_gid(0)
    assert gid.startswith("fe:80:") and len(gid) == 47, gid
    t = ctypes.create_string_buffer(n)
    s = ctypes.create_string_buffer(os.urandom(n), n)
    d = ctypes.create_string_buffer(n)
    assert b.register_memory(ctypes.addressof(t), n) == 0
    assert b.publish_buffer(ctypes.addressof(t), n) == 0
    assert b.start_accept_thread() == 0
    for x in (s, d):
        assert a.register_memory(ctypes.addressof(x), n) == 0
    rk = b.get_all_rkeys(ctypes.addressof(t))
    assert len(rk) == 2 and all(rk), rk
    port = b.get_tcp_port()
    assert a.connect("B", "127.0.0.1", port) == 0
    info = a.query_remote_buffers("B", "127.0.0.1", port)
    assert info["buffers"][0]["rkeys"] == rk
    h = a.put_async(ctypes.addressof(s), "B", ctypes.addressof(t), n)
    assert a.wait_transfer(h, 20000) == 0, "PUT failed"
    a.release_transfer(h)
    assert t.raw == s.raw
    h = a.get_async(ctypes.addressof(d), "B", ctypes.addressof(t), n)
    assert a.wait_transfer(h, 20000) == 0, "GET failed"
    a.release_transfer(h)
    assert d.raw == s.raw
    seg = n // 3
    h = a.scatter_async(ctypes.addressof(s), ["B"] * 3, [ctypes.addressof(t) + (2 - i) * seg for i in range(3)],
                        [seg] * 3)
    assert a.wait_transfer(h, 20000) == 0
    a.release_transfer(h)
    for i in range(3):
        assert t.raw[(2 - i) * seg:(3 - i) * seg] == s.raw[i * seg:(i + 1) * seg]
    sport_check(a)
    a.shutdown()
    b.shutdown()
    print("ib fake ok", flush=True)


def sport_check(comm):
    """With MPCOMM_IBV_DV_LIB pointing at this provider, every RTS transition
    set a UDP source port through the device vendor's call."""
    want = os.environ.get("EXPECT_SPORT_VENDOR")
    if not want:
        return
    lib = ctypes.CDLL(os.environ["MPCOMM_IBVERBS_LIB"])
    calls = [lib.fake_ibv_sport_calls(0), lib.fake_ibv_sport_calls(1)]
    vendor = {"mlx5": 0, "bnxt_re": 1}[want]
    assert calls[vendor] > 0 and calls[1 - vendor] == 0, calls
    ports = (ctypes.c_uint16 * 256)()
    n = lib.fake_ibv_sports(ports, 256)
    got = {ports[i] for i in range(min(n, 256))}
    allowed = {int(x) for x in os.environ.get("MPCOMM_UDP_SPORTS", "").split(",") if x}
    if allowed:
        assert got <= allowed and len(got) == len(allowed), (got, allowed)
    else:
        assert all(49152 <= p <= 65535 for p in got) and len(got) > 1, got
    print(f"sport calls {calls} ports {sorted(got)}", flush=True)


def main_gpu():
    import torch

    lib = ctypes.CDLL(os.environ["MPCOMM_IBVERBS_LIB"])
    lib.fake_ibv_dmabuf_registrations.restype = ctypes.c_int
    n = (24 << 20) + 4096
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(3)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    tgt = torch.zeros(n, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("A") == 0 and b.init("B") == 0
    assert a.get_fabric_name() == "ib", a.get_fabric_name()
    # What the driver offers: dma-buf support of the device, and an export
    # of this exact range (the backend exports 64 KiB-aligned spans).
    cuda = ctypes.CDLL("libcuda.so.1")
    dev = ctypes.c_int()
    assert cuda.cuDeviceGet(ctypes.byref(dev), 0) == 0
    sup = ctypes.c_int(-1)
    cuda.cuDeviceGetAttribute(ctypes.byref(sup), 124, dev)  # CU_DEVICE_ATTRIBUTE_DMA_BUF_SUPPORTED
    def export_rc(a0, span, flags=0):
        fd = ctypes.c_int(-1)
        rc = cuda.cuMemGetHandleForAddressRange(ctypes.byref(fd), ctypes.c_uint64(a0), ctypes.c_size_t(span),
                                                1, ctypes.c_ulonglong(flags))  # CU_MEM_RANGE_HANDLE_TYPE_DMA_BUF_FD
        if rc == 0:
            os.close(fd.value)
        return rc

    base, size = ctypes.c_uint64(0), ctypes.c_size_t(0)
    assert cuda.cuMemGetAddressRange_v2(ctypes.byref(base), ctypes.byref(size), ctypes.c_uint64(src.data_ptr())) == 0
    rc = export_rc(base.value, size.value)  # the whole allocation, as the backend exports it
    sub = export_rc(src.data_ptr() & ~0xFFFF, ((src.data_ptr() + n + 0xFFFF) & ~0xFFFF) - (src.data_ptr() & ~0xFFFF))
    pcie = export_rc(base.value, size.value, 1)  # CU_MEM_RANGE_FLAG_DMA_BUF_MAPPING_TYPE_PCIE
    print(f"driver: dma_buf_supported={sup.value} export_rc={rc} subrange_rc={sub} pcie_flag_rc={pcie} "
          f"allocation={size.value} bytes", flush=True)
    before = lib.fake_ibv_dmabuf_registrations()
    assert b.register_memory(tgt.data_ptr(), n) == 0
    assert b.publish_buffer(tgt.data_ptr(), n) == 0
    assert b.start_accept_thread() == 0
    for x in (src, dst):
        assert a.register_memory(x.data_ptr(), n) == 0
    regs = lib.fake_ibv_dmabuf_registrations() - before
    if sup.value == 1 and rc == 0:
        # every buffer on every NIC went through the dma-buf path
        assert regs == 3 * len(a.get_active_devices()), regs
    else:
        # no dma-buf export here: the backend falls back to ibv_reg_mr
        # (nvidia-peermem style); the transfers below still run on HBM
        assert regs == 0, regs
    port = b.get_tcp_port()
    assert a.connect("B", "127.0.0.1", port) == 0
    assert a.query_remote_buffers("B", "127.0.0.1", port)
    h = a.put_async(src.data_ptr(), "B", tgt.data_ptr(), n)
    assert a.wait_transfer(h, 20000) == 0, "PUT into HBM failed"
    a.release_transfer(h)
    torch.cuda.synchronize()
    assert torch.equal(tgt, src), "PUT mismatch"
    h = a.get_async(dst.data_ptr() + 4096, "B", tgt.data_ptr() + 4096, n - 4096)
    assert a.wait_transfer(h, 20000) == 0, "GET from HBM failed"
    a.release_transfer(h)
    torch.cuda.synchronize()
    assert torch.equal(dst[4096:], src[4096:]) and not dst[:4096].any(), "GET mismatch"
    # HBM allocated for GPUDirect RDMA (VMM allocation with the
    # gpuDirectRDMACapable flag): the driver's dma-buf export of it, and its
    # registration + a PUT into it through the fake provider.
    from mpcomm.parallel import device_view

    err, gptr, gsize = mpcomm._native.gdr_alloc(0, n)
    gdr = {"alloc_rc": err}
    if err == 0:
        gdr["export_rc"] = mpcomm._native.dmabuf_export_rc(gptr, gsize, 0)
        gdr["export_pcie_rc"] = mpcomm._native.dmabuf_export_rc(gptr, gsize, 1)
        before = lib.fake_ibv_dmabuf_registrations()
        assert b.register_memory(gptr, n) == 0 and b.publish_buffer(gptr, n) == 0
        gdr["dmabuf_registrations"] = lib.fake_ibv_dmabuf_registrations() - before
        if gdr["export_rc"] == 0 or gdr["export_pcie_rc"] == 0:
            assert gdr["dmabuf_registrations"] == len(b.get_active_devices()), gdr
        assert a.query_remote_buffers("B", "127.0.0.1", port)
        h = a.put_async(src.data_ptr(), "B", gptr, n)
        assert a.wait_transfer(h, 20000) == 0, "PUT into GPUDirect HBM failed"
        a.release_transfer(h)
        torch.cuda.synchronize()
        assert torch.equal(device_view(gptr, n), src), "PUT into GPUDirect HBM mismatch"
        b.unpublish_buffer(gptr)
        b.unregister_memory(gptr)
        assert mpcomm._native.gdr_free(gptr, gsize) == 0
    print(f"gdr: {gdr}", flush=True)
    a.shutdown()
    b.shutdown()
    print(f"ib fake ok (dma-buf registrations: {regs}, dma_buf_supported={sup.value}, export_rc={rc})",
          flush=True)


if __name__ == "__main__":
    main_gpu() if "--gpu" in sys.argv else main()
