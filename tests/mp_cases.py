"""Multi-GPU test cases, one process per GPU (run by tests/test_multigpu.py
under torch.distributed.run). Each case verifies bit-exactly and exits
non-zero on any mismatch.

  putget  GPU fabric PUT/GET/scatter between processes: rank r writes into
          rank r^1's published HBM buffer over NVLink (CUDA IPC).
  pxn     fused gather + forward: pages of a host pool shared by all ranks are
          gathered by rank (r+1)%N and stored into rank r's HBM; a done flag
          lands in rank r's memory.
  nvls    NVLS multicast broadcast from rank 0 (falls back to P2P fan-out
          where multicast is unavailable) of a rollout-style batch.
  gather_bcast  fused host-page gather + broadcast from rank 0 in one kernel
          (NVLS multimem stores where supported, then P2P bulk stores),
          completed by a device flag every rank waits on with a bounded wait.
  peer_exit  (2 ranks) rank 1 leaves between steps; rank 0's next PUT to it
          fails on the host, fast, and its engine keeps working.
  engine_bcast  MPComm.broadcast_async from rank 0 to every other rank: one
          fused launch per chunk (bulk stores to each peer's published
          buffer), then to the other members' copies of an NVLS group
          (multicast stores); the kernel trace shows which launch ran.
  engine_pxn  MPComm.put_pages_async: rank r gathers the pages rank
          (r-1)%N wants from a host pool shared by all ranks and writes them
          into that rank's published HBM buffer (fused PXN gather + forward as
          an engine transfer).
"""
import argparse
import datetime
import os
import sys
import time
import zlib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import mpcomm  # noqa: E402
from mpcomm import ops, parallel  # noqa: E402


def case_putget(rank, world):
    peer = rank ^ 1
    if peer >= world:
        return
    n = (48 << 20) + 64
    mine = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda",
                         generator=torch.Generator(device="cuda").manual_seed(100 + rank))
    inbox = torch.zeros(n, dtype=torch.uint8, device="cuda")
    back = torch.zeros(n, dtype=torch.uint8, device="cuda")
    comm = mpcomm.MPComm()
    assert comm.init(f"r{rank}") == 0 and comm.get_fabric_name() == "nvl"
    assert comm.start_accept_thread() == 0
    for t in (mine, inbox, back):
        assert comm.register_memory(t.data_ptr(), t.numel()) == 0
    assert comm.publish_buffer(inbox.data_ptr(), n) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    dist.barrier()
    assert comm.connect("peer", "127.0.0.1", ports[peer]) == 0
    info = comm.query_remote_buffers("peer", "127.0.0.1", ports[peer])
    remote = info["buffers"][0]["addr"]
    torch.cuda.synchronize()
    h = comm.put_async(mine.data_ptr(), "peer", remote, n)
    assert comm.wait_transfer(h, 60000) == 0, "cross-process PUT failed"
    comm.release_transfer(h)
    dist.barrier()  # both PUTs done
    crcs = [None] * world
    dist.all_gather_object(crcs, (zlib.crc32(mine.cpu().numpy().tobytes()),
                                  zlib.crc32(inbox.cpu().numpy().tobytes())))
    assert crcs[rank][1] == crcs[peer][0], "peer data did not arrive intact"
    h = comm.get_async(back.data_ptr(), "peer", remote, n)
    assert comm.wait_transfer(h, 60000) == 0, "cross-process GET failed"
    comm.release_transfer(h)
    torch.cuda.synchronize()
    assert torch.equal(back, mine)  # what we wrote to the peer reads back
    dist.barrier()
    comm.shutdown()


def case_pxn(rank, world):
    bs, pages, n = 65536, 4096, 256
    name = "mpcomm-test-pxn"
    if rank == 0:
        pool = parallel.SharedHostPool(name, pages * bs, create=True)
        g = torch.Generator().manual_seed(7)
        pool.tensor.copy_(torch.randint(0, 256, (pages * bs,), dtype=torch.uint8, generator=g))
    dist.barrier()
    if rank != 0:
        pool = parallel.SharedHostPool(name, pages * bs, create=False)
    dist.barrier()
    bufs = parallel.PeerBuffers(n * bs)
    flags = parallel.PeerBuffers(64)
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    # what every rank wants
    wants = [torch.randperm(pages, generator=torch.Generator().manual_seed(3 + r))[:n] for r in range(world)]
    requester = (rank - 1) % world  # this rank gathers for requester
    idx = wants[requester].cuda()
    dist.barrier()
    ops.pxn_gather_forward(pool.dev_ptr, pages, idx, bufs.ptrs[requester], bs,
                           done_flag=flags.ptrs[requester], flag_value=42, counter=ctr.data_ptr())
    torch.cuda.synchronize()
    dist.barrier()
    got = bufs.local.view(n, bs).cpu()
    ref = pool.tensor.view(pages, bs)[wants[rank]]
    assert torch.equal(got, ref), "forwarded pages differ"
    assert flags.local.view(torch.int64)[0].item() == 42, "done flag not published"
    dist.barrier()
    bufs.close()
    flags.close()
    pool.close(unlink=(rank == 0))


def case_nvls(rank, world):
    nbytes = 8 << 20
    src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(5))
    try:
        grp = parallel.NvlsGroup(nbytes)
        used = "nvls"
    except RuntimeError as e:
        grp = None
        used = f"fanout ({e})"
    if grp is not None:
        grp.uc[:nbytes].zero_()
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            ops.nvls_broadcast(src, grp.mc_ptr, nbytes)
            torch.cuda.synchronize()
        dist.barrier()
        assert torch.equal(grp.uc[:nbytes], src), "NVLS broadcast mismatch"
        dist.barrier()
        # All-source broadcast: every rank pulls its slice from rank 0's HBM.
        root = parallel.PeerBuffers(nbytes)
        if rank == 0:
            root.local.copy_(torch.flip(src, [0]))
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        grp.broadcast_from(root.ptrs[0], nbytes)
        torch.cuda.synchronize()
        dist.barrier()
        assert torch.equal(grp.uc[:nbytes], torch.flip(src, [0])), "all-source NVLS broadcast mismatch"
        dist.barrier()
        # The same with bulk copies of each slice into shared memory.
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        grp.broadcast_from(root.ptrs[0], nbytes, method="bulk")
        torch.cuda.synchronize()
        dist.barrier()
        assert torch.equal(grp.uc[:nbytes], torch.flip(src, [0])), "all-source bulk NVLS broadcast mismatch"
        dist.barrier()
        root.close()
        grp.close()
    bufs = parallel.PeerBuffers(nbytes)
    dist.barrier()
    if rank == 0:
        ops.p2p_fanout(src, [bufs.ptrs[r] for r in range(1, world)], nbytes)
        torch.cuda.synchronize()
    dist.barrier()
    if rank != 0:
        assert torch.equal(bufs.local, src), "P2P fan-out mismatch"
    dist.barrier()
    bufs.close()
    if rank == 0:
        print(f"nvls case used: {used}", flush=True)


def case_gather_bcast(rank, world):
    bs, pages, n = 65536 + 1024, 384, 96
    pool_cpu = torch.randint(0, 256, (pages, bs), dtype=torch.uint8, generator=torch.Generator().manual_seed(11))
    idx_cpu = torch.randperm(pages, generator=torch.Generator().manual_seed(12))[:n]
    expect = pool_cpu[idx_cpu].reshape(-1)
    nbytes = n * bs
    fo = nbytes  # flag word right after the batch (nbytes % 256 == 0)
    pool = pool_cpu.pin_memory() if rank == 0 else None
    idx = idx_cpu.cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    budget = 10_000_000_000
    used = []
    try:
        grp = parallel.NvlsGroup(nbytes + 256)
    except RuntimeError as e:
        grp = None
        used.append(f"nvls unavailable ({e})")
    if grp is not None:
        grp.uc.zero_()
        for rep in (1, 2):
            grp.uc[:nbytes].zero_()
            torch.cuda.synchronize()
            dist.barrier()
            if rank == 0:
                ops.gather_bcast(pool.data_ptr(), pages, idx, bs, mc_ptr=grp.mc_ptr, mc_flag=grp.mc_ptr + fo,
                                 counter=ctr.data_ptr(), status_ptr=status.data_ptr())
            ops.wait_flag(grp.uc_ptr + fo, rep, budget, status_ptr=status.data_ptr())
            torch.cuda.synchronize()
            assert status.item() == 0, f"rank {rank} status {status.item()}"
            assert torch.equal(grp.uc[:nbytes].cpu(), expect), "fused NVLS broadcast mismatch"
            dist.barrier()
        used.append("nvls")
        grp.close()
    bufs = parallel.PeerBuffers(nbytes + 256)
    for rep in (1, 2):
        bufs.local.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            ops.gather_bcast(pool.data_ptr(), pages, idx, bs, dst_ptrs=bufs.ptrs,
                             flags=[p + fo for p in bufs.ptrs], flag_value=100 + rep, counter=ctr.data_ptr(),
                             status_ptr=status.data_ptr())
        ops.wait_flag(bufs.local.data_ptr() + fo, 100 + rep, budget, status_ptr=status.data_ptr())
        torch.cuda.synchronize()
        assert status.item() == 0, f"rank {rank} status {status.item()}"
        assert torch.equal(bufs.local[:nbytes].cpu(), expect), "fused P2P fan-out mismatch"
        dist.barrier()
    used.append("p2p")
    bufs.close()
    if rank == 0:
        print(f"gather_bcast case used: {used}", flush=True)


def case_peer_exit(rank, world):
    """Rank 1 leaves between steps (its MPComm shut down, nothing in flight)
    and tells rank 0 through the store. Rank 0's next PUT to it must fail
    fast on the host (peer liveness check, no launch at the dead peer's
    memory) and rank 0's engine must stay usable."""
    n = 8 << 20
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    inbox = torch.zeros(n, dtype=torch.uint8, device="cuda")
    comm = mpcomm.MPComm()
    assert comm.init(f"r{rank}") == 0 and comm.start_accept_thread() == 0
    for t in (src, inbox):
        assert comm.register_memory(t.data_ptr(), n) == 0
    assert comm.publish_buffer(inbox.data_ptr(), n) == 0
    info = [None] * world
    dist.all_gather_object(info, (comm.get_tcp_port(), os.getpid()))
    peer = rank ^ 1
    assert comm.connect("peer", "127.0.0.1", info[peer][0]) == 0
    remote = comm.query_remote_buffers("peer", "127.0.0.1", info[peer][0])["buffers"][0]["addr"]
    h = comm.put_async(src.data_ptr(), "peer", remote, n)
    assert comm.wait_transfer(h, 60000) == 0
    comm.release_transfer(h)
    torch.cuda.synchronize()
    dist.barrier()  # step 1 done on both sides
    store = dist.distributed_c10d._get_default_store()
    if rank == 1:
        comm.shutdown()
        store.set("r1_left", "1")
        return True
    store.wait(["r1_left"], datetime.timedelta(seconds=60))
    deadline = time.time() + 60
    while time.time() < deadline:
        try:
            os.kill(info[1][1], 0)
        except ProcessLookupError:
            break
        time.sleep(0.05)
    else:
        raise AssertionError("rank 1 did not exit")
    t0 = time.time()
    h = comm.put_async(src.data_ptr(), "peer", remote, n)
    rc = comm.wait_transfer(h, 20000) if h else -1
    if h:
        comm.release_transfer(h)
    assert rc != 0 and rc != int(mpcomm.MPCommError.ERR_TIMEOUT), rc
    assert time.time() - t0 < 10, "failure took too long to surface"
    # The engine is still usable: PUT into a pinned host pool of our own.
    pool = torch.zeros(n, dtype=torch.uint8, pin_memory=True)
    assert comm.register_memory(pool.data_ptr(), n) == 0 and comm.publish_buffer(pool.data_ptr(), n) == 0
    port = comm.get_tcp_port()
    assert comm.connect("self", "127.0.0.1", port) == 0 and comm.query_remote_buffers("self", "127.0.0.1", port)
    h = comm.put_async(src.data_ptr(), "self", pool.data_ptr(), n)
    assert comm.wait_transfer(h, 60000) == 0
    comm.release_transfer(h)
    assert torch.equal(pool, src.cpu())
    comm.shutdown()
    return True


def case_engine_bcast(rank, world):
    os.environ["MPCOMM_NVL_CHUNK_SIZE"] = str(16 << 20)  # several chunks per broadcast
    n = (40 << 20) + 4096
    comm = mpcomm.MPComm()
    assert comm.init(f"b{rank}") == 0 and comm.get_fabric_name() == "nvl"
    assert comm.start_accept_thread() == 0
    g = torch.Generator(device="cuda").manual_seed(77)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)  # same on every rank
    inbox = torch.zeros(n, dtype=torch.uint8, device="cuda")
    for t in (src, inbox):
        assert comm.register_memory(t.data_ptr(), n) == 0
    assert comm.publish_buffer(inbox.data_ptr(), n) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    dist.barrier()
    hosts = [f"b{r}" for r in range(1, world)]
    if rank == 0:
        for r in range(1, world):
            assert comm.connect(f"b{r}", "127.0.0.1", ports[r]) == 0

    def trace_kinds():
        return [t["kind"] for t in mpcomm._native.kernel_trace()]

    def bcast(raddrs, want_kind):
        mpcomm._native.kernel_trace_reset()
        h = comm.broadcast_async(src.data_ptr(), n, hosts, raddrs)
        assert h != mpcomm.INVALID_TRANSFER_HANDLE
        assert comm.wait_transfer(h, 60000) == 0, "broadcast failed"
        res = comm.get_transfer_result(h)
        comm.release_transfer(h)
        assert res["bytes_transferred"] == n * (world - 1), res
        kinds = trace_kinds()
        # 3 chunks of at most 16 MiB: one fused launch each, no per-destination copies.
        assert kinds.count(want_kind) == 3 and "copy_batch" not in kinds, kinds

    if rank == 0:
        raddrs = []
        for r in range(1, world):
            info = comm.query_remote_buffers(f"b{r}", "127.0.0.1", ports[r])
            raddrs.append(next(b["addr"] for b in info["buffers"] if b["length"] == n))
        bcast(raddrs, "gather_bcast_p2p")
    dist.barrier()
    if rank != 0:
        assert torch.equal(inbox, src), "fused P2P broadcast mismatch"
    used = ["p2p"]
    try:
        grp = parallel.NvlsGroup(n)
    except RuntimeError as e:
        grp = None
        used.append(f"nvls unavailable ({e})")
    if grp is not None:
        grp.uc.zero_()
        torch.cuda.synchronize()
        grp.register(comm)
        assert comm.publish_buffer(grp.uc_ptr, grp.size, 7) == 0
        ucs = [None] * world
        dist.all_gather_object(ucs, grp.uc_ptr)
        dist.barrier()
        if rank == 0:
            for r in range(1, world):  # refresh the peers' buffer lists
                assert comm.query_remote_buffers(f"b{r}", "127.0.0.1", ports[r])
            bcast(ucs[1:], "gather_bcast_nvls")
        dist.barrier()
        # Every member's copy holds the batch, the sender's own included.
        assert torch.equal(grp.uc[:n], src), "fused NVLS broadcast mismatch"
        dist.barrier()
        comm.unpublish_buffer(grp.uc_ptr)
        comm.unregister_memory(grp.uc_ptr)
        dist.barrier()
        grp.close()
        used.append("nvls")
    dist.barrier()
    comm.shutdown()
    if rank == 0:
        print(f"engine_bcast case used: {used}", flush=True)


def case_engine_pxn(rank, world):
    bs, pages, n = 65536, 2048, 200
    name = f"mpcomm-test-epxn-{os.environ.get('MASTER_PORT', '0')}"
    if rank == 0:
        pool = parallel.SharedHostPool(name, pages * bs, create=True)
        g = torch.Generator().manual_seed(21)
        pool.tensor.copy_(torch.randint(0, 256, (pages * bs,), dtype=torch.uint8, generator=g))
    dist.barrier()
    if rank != 0:
        pool = parallel.SharedHostPool(name, pages * bs, create=False)
    dist.barrier()
    requester = (rank - 1) % world
    wants = [torch.randperm(pages, generator=torch.Generator().manual_seed(30 + r))[:n] for r in range(world)]
    idx = wants[requester].cuda()
    inbox = torch.zeros(n * bs, dtype=torch.uint8, device="cuda")
    comm = mpcomm.MPComm()
    assert comm.init(f"p{rank}") == 0 and comm.start_accept_thread() == 0
    dram = comm.map_dram_to_gpu(pool.tensor.data_ptr(), pages * bs)
    assert dram
    assert comm.register_memory(inbox.data_ptr(), inbox.numel()) == 0
    assert comm.publish_buffer(inbox.data_ptr(), inbox.numel()) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    dist.barrier()
    host = f"p{requester}"
    assert comm.connect(host, "127.0.0.1", ports[requester]) == 0
    info = comm.query_remote_buffers(host, "127.0.0.1", ports[requester])
    raddr = info["buffers"][0]["addr"]
    h = comm.put_pages_async(dram, idx.data_ptr(), n, bs, host, raddr)
    assert h != mpcomm.INVALID_TRANSFER_HANDLE
    assert comm.wait_transfer(h, 60000) == 0, "paged PUT failed"
    res = comm.get_transfer_result(h)
    comm.release_transfer(h)
    assert res["bytes_transferred"] == n * bs
    dist.barrier()  # every rank's pages have landed
    assert torch.equal(inbox.view(n, bs).cpu(), pool.tensor.view(pages, bs)[wants[rank]]), "paged PUT mismatch"
    dist.barrier()
    comm.unmap_dram_from_gpu(pool.tensor.data_ptr())
    comm.shutdown()
    dist.barrier()
    pool.close(unlink=(rank == 0))


def main():
    os.environ.setdefault("MPCOMM_KERNEL_TRACE", "4096")
    p = argparse.ArgumentParser()
    p.add_argument("case", choices=["putget", "pxn", "nvls", "gather_bcast", "peer_exit", "engine_bcast", "engine_pxn",
                                      "all"])
    a = p.parse_args()
    rank, world, _ = parallel.init_from_env("gloo")
    if a.case == "peer_exit":
        # Ranks leave independently: no final collective.
        if rank < 2:
            case_peer_exit(rank, world)
        if rank == 0:
            print("case peer_exit ok", flush=True)
        os._exit(0)
    cases = (["putget", "pxn", "nvls", "gather_bcast", "engine_bcast", "engine_pxn"] if a.case == "all"
             else [a.case])
    for c in cases:
        globals()[f"case_{c}"](rank, world)
        if rank == 0:
            print(f"case {c} ok", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
