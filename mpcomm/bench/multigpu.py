"""Inter-GPU paths measured by the headline run at N >= 2 GPUs.

``bench.py`` measures HBM <-> host-DRAM PUT/GET on every rank; at two GPUs
and more it then calls :func:`run` here, which measures, on the same ranks
and in the same process group, the three paths that cross NVLink:

* ``nvlink``  zero-copy PUT/GET between GPU pairs through the MPComm engine
              (rank r <-> rank r^1 HBM over the GPU fabric, CUDA IPC), 1 GiB
              blocks, batch 4 (reference
              user_examples/scatter_test.cpp:864-1187).
* ``pxn``     fused paged gather + NVLink forward (config 4): 1,024 random
              64 KiB Llama-3-8B KV pages per rank (seed 3 + rank) from a
              shared host pool, gathered by rank (r+1) % N and stored into
              rank r's HBM by one kernel (reference PXN copy path
              src/mpcomm_pxn.cpp:638-814).
* ``bcast``   the 57.9 MB RL rollout batch (seed 4) gathered from rank 0's
              pinned host memory and delivered to every GPU by one
              gather_bcast launch: NVLS ``multimem.st`` where multicast is
              supported, bulk stores to each peer otherwise (config 5;
              reference broadcastAsync src/mpcomm.cpp:4937-4954).

Every path is timed with CUDA events on the device (max over ranks), its
result checked by CRC-32 on every rank, and reported against its roofline
measured in the same run: NVLink at 770 GB/s per direction per GPU (the
pool's measured peer copy) and PCIe host reads at the copy-engine rate of
the same bytes, all ranks at once.
"""
from __future__ import annotations

import os
from typing import Callable, Optional

import torch
import torch.distributed as dist

import mpcomm
from mpcomm import ops, parallel
from mpcomm.models import LLAMA3_8B_KV, RolloutBatch

NVLINK_GBS = 770.0  # measured peer copy per direction per B200 on this pool
PAGE = 65536
WAIT_BUDGET_NS = 5_000_000_000


def _all_max(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _all_true(ok: bool, dev) -> bool:
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


_host_barrier_seq = [0]


def _host_barrier(timeout_s: float = 300.0) -> None:
    """Barrier through the process group's TCP store: no device work, so a
    rank waiting here leaves its GPU streams free while a peer's control-plane
    handshake (connect, buffer query) reaches this process."""
    import time

    store = dist.distributed_c10d._get_default_store()
    _host_barrier_seq[0] += 1
    key = f"mpcomm-bench-barrier-{_host_barrier_seq[0]}"
    store.add(key, 1)
    deadline = time.time() + timeout_s
    while store.add(key, 0) < dist.get_world_size():
        if time.time() > deadline:
            raise TimeoutError(f"host barrier {key} timed out")
        time.sleep(0.002)


def _timed(step: Callable[[int], None], stream: torch.cuda.Stream, warmup: int, iters: int, dev,
           seq0: int = 0) -> float:
    """Mean device ms of one step on this rank's stream, max over ranks."""
    for i in range(warmup):
        step(seq0 + i)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(iters):
        step(seq0 + warmup + i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = _all_max(e0.elapsed_time(e1) / iters, dev)
    dist.barrier()
    return ms


def nvlink_putget(comm, src: torch.Tensor, dst: torch.Tensor, block: int, batch: int,
                  fstream: torch.cuda.Stream, warmup: int = 2, iters: int = 5) -> dict:
    """PUT src -> peer HBM, then GET peer HBM -> dst, through ``comm``."""
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = src.device
    total = block * batch
    target = torch.zeros(total, dtype=torch.uint8, device=dev)
    assert comm.register_memory(target.data_ptr(), total) == 0
    assert comm.publish_buffer(target.data_ptr(), total) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    _host_barrier()
    peer = rank ^ 1
    assert comm.connect("nvpeer", "127.0.0.1", ports[peer]) == 0
    info = comm.query_remote_buffers("nvpeer", "127.0.0.1", ports[peer])
    raddr = next(b["addr"] for b in info["buffers"] if b["gpu_device_id"] >= 0 and b["length"] == total)
    _host_barrier()
    sp, dp = src.data_ptr(), dst.data_ptr()

    def phase(put: bool):
        hs = []
        for i in range(batch):
            if put:
                h = comm.put_async(sp + i * block, "nvpeer", raddr + i * block, block)
            else:
                h = comm.get_async(dp + i * block, "nvpeer", raddr + i * block, block)
            assert h != mpcomm.INVALID_TRANSFER_HANDLE
            hs.append(h)
        for h in hs:
            assert comm.wait_transfer(h, 120000) == 0, "NVLink transfer failed"
            comm.release_transfer(h)

    dst.zero_()
    put_ms = _timed(lambda _s: phase(True), fstream, warmup, iters, dev)
    get_ms = _timed(lambda _s: phase(False), fstream, warmup, iters, dev)
    crc_ok = _all_true(torch.equal(ops.crc32_blocks(dst, batch), ops.crc32_blocks(src, batch)), dev)
    dist.barrier()
    assert comm.unpublish_buffer(target.data_ptr()) == 0
    comm.unregister_memory(target.data_ptr())
    del target
    per_gpu_put = total / (put_ms * 1e-3) / 1e9
    per_gpu_get = total / (get_ms * 1e-3) / 1e9
    return {
        "nvlink_put_gbs": round(world * per_gpu_put, 3),
        "nvlink_get_gbs": round(world * per_gpu_get, 3),
        "nvlink_putget_gbs": round(world * 2 * total / ((put_ms + get_ms) * 1e-3) / 1e9, 3),
        "nvlink_put_roofline_frac": round(per_gpu_put / NVLINK_GBS, 4),
        "nvlink_get_roofline_frac": round(per_gpu_get / NVLINK_GBS, 4),
        "nvlink_crc_ok": crc_ok,
        "nvlink_what": f"rank r <-> r^1 HBM through MPComm (GPU fabric, CUDA IPC), {batch} x {block >> 20} MiB; "
                       f"roofline {NVLINK_GBS:.0f} GB/s per direction per GPU",
    }


def _fill_kv_pool(view: torch.Tensor, dev, seed: int = 0) -> None:
    """Llama-3-8B KV pages (bf16 ~ N(0, 1)) generated on the GPU, copied in."""
    g = torch.Generator(device=dev).manual_seed(seed)
    rows = max(1, (256 << 20) // view.shape[1])
    for s in range(0, view.shape[0], rows):
        e = min(view.shape[0], s + rows)
        vals = torch.randn((e - s, view.shape[1] // 2), generator=g, device=dev, dtype=torch.float32)
        view[s:e].copy_(vals.to(torch.bfloat16).view(torch.uint8))
    torch.cuda.synchronize()


def pxn_forward(comm, fstream: torch.cuda.Stream, dev, pool_pages: int = 65536, request: int = 1024,
                warmup: int = 3, iters: int = 10) -> dict:
    rank, world = dist.get_rank(), dist.get_world_size()
    bs = LLAMA3_8B_KV.page_bytes
    name = f"mpcomm-bench-pxn-{os.environ.get('MASTER_PORT', '0')}"
    nbytes = pool_pages * bs
    pool = parallel.SharedHostPool(name, nbytes, create=True) if rank == 0 else None
    if rank == 0:
        _fill_kv_pool(pool.tensor.view(pool_pages, bs), dev)
    dist.barrier()
    if rank != 0:
        pool = parallel.SharedHostPool(name, nbytes, create=False)
    dist.barrier()
    requester = (rank - 1) % world  # this rank forwards for its left neighbour
    wants = LLAMA3_8B_KV.sample_pages(pool_pages, request, seed=3 + rank).to(dev)
    fwd_idx = LLAMA3_8B_KV.sample_pages(pool_pages, request, seed=3 + requester).to(dev)
    out = parallel.PeerBuffers(request * bs)
    flags = parallel.PeerBuffers(64)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    pool_view = pool.tensor.view(pool_pages, bs)

    def step(seq: int):
        ops.pxn_gather_forward(pool.dev_ptr, pool_pages, fwd_idx, out.ptrs[requester], bs,
                               done_flag=flags.ptrs[requester], flag_value=seq + 1, counter=ctr.data_ptr(),
                               stream=stream)
        ops.wait_flag(flags.local.data_ptr(), seq + 1, WAIT_BUDGET_NS, status.data_ptr(), stream=stream)

    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    ms = _timed(step, stream, warmup, iters, dev)
    launches = mpcomm.MPComm.get_kernel_launch_count() - launches0
    # Check: CRC of what arrived vs CRC of the same pages gathered by this
    # rank itself over its own PCIe link.
    ref = torch.empty(request * bs, dtype=torch.uint8, device=dev)
    ops.paged_gather(pool_view, wants, out=ref.view(request, bs))
    got = ops.crc32_blocks(out.local, request)
    exp = ops.crc32_blocks(ref, request)
    torch.cuda.synchronize()
    crc_ok = _all_true(torch.equal(got, exp) and status.item() == 0, dev)

    # The same forward through the public engine API: put_pages_async on the
    # GPU holding the indices, into the requester's published buffer (one
    # fused launch per chunk of pages, tracked by a handle). Each proxy's
    # transfer completes once its pages have landed, so the max over ranks
    # of the per-rank device time is the delivery time.
    dram = comm.map_dram_to_gpu(pool.tensor.data_ptr(), nbytes)
    assert dram
    inbox = torch.zeros(request * bs, dtype=torch.uint8, device=dev)
    assert comm.register_memory(inbox.data_ptr(), inbox.numel()) == 0
    assert comm.publish_buffer(inbox.data_ptr(), inbox.numel()) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    _host_barrier()
    assert comm.connect("pxnreq", "127.0.0.1", ports[requester]) == 0
    info = comm.query_remote_buffers("pxnreq", "127.0.0.1", ports[requester])
    raddr = next(b["addr"] for b in info["buffers"] if b["length"] == request * bs and b["gpu_device_id"] >= 0)
    _host_barrier()

    def engine_step(_seq: int):
        # `iters` requests in flight at once, as an application keeps them.
        hs = [comm.put_pages_async(dram, fwd_idx.data_ptr(), request, bs, "pxnreq", raddr) for _ in range(iters)]
        for h in hs:
            assert h != mpcomm.INVALID_TRANSFER_HANDLE
            assert comm.wait_transfer(h, 60000) == 0, "paged PUT failed"
            comm.release_transfer(h)

    engine_ms = _timed(engine_step, fstream, 1, 1, dev) / iters
    engine_ok = _all_true(torch.equal(ops.crc32_blocks(inbox, request), exp), dev)
    dist.barrier()
    comm.unpublish_buffer(inbox.data_ptr())
    comm.unregister_memory(inbox.data_ptr())
    comm.unmap_dram_from_gpu(pool.tensor.data_ptr())

    # Unfused two step (the reference's shape: gather into the proxy's own
    # HBM, then a separate peer copy into the requester's buffer; here both
    # steps are this library's kernels).
    staging = torch.empty(request * bs, dtype=torch.uint8, device=dev)

    def two_step(_seq: int):
        ops.paged_gather(pool_view, fwd_idx, out=staging.view(request, bs), stream=stream)
        ops.copy_spans([staging.data_ptr()], [out.ptrs[requester]], [request * bs], stream=stream)

    two_ms = _timed(two_step, stream, 1, max(3, iters // 2), dev)

    # Roofline: every proxy's host read at the copy-engine rate of the same
    # pool, all ranks at once (PCIe + host ceiling; NVLink is faster).
    chunk = pool.tensor[: request * bs]
    ce_dst = staging

    def ce_step(_seq: int):
        with torch.cuda.stream(stream):
            ce_dst.copy_(chunk, non_blocking=True)

    ce_ms = _timed(ce_step, stream, 1, 5, dev)
    dist.barrier()
    out.close()
    flags.close()
    pool.close(unlink=(rank == 0))
    total = world * request * bs
    gbs = total / (ms * 1e-3) / 1e9
    roof = total / (ce_ms * 1e-3) / 1e9
    return {
        "pxn_forward_gbs": round(gbs, 3),
        "pxn_forward_ms": round(ms, 4),
        "pxn_roofline_gbs": round(roof, 3),
        "pxn_roofline_frac": round(gbs / roof, 4),
        "pxn_two_step_gbs": round(total / (two_ms * 1e-3) / 1e9, 3),
        "pxn_engine_gbs": round(total / (engine_ms * 1e-3) / 1e9, 3),
        "pxn_engine_roofline_frac": round(total / (engine_ms * 1e-3) / 1e9 / roof, 4),
        "pxn_engine_crc_ok": engine_ok,
        "pxn_crc_ok": crc_ok,
        "pxn_gpu_launches": int(launches),
        "pxn_what": f"{request} x 64 KiB KV pages per rank (seed 3+rank) from a {nbytes >> 30} GiB shared host pool, "
                    f"gathered by rank (r+1)%N and stored into rank r's HBM by one kernel (pxn_*: the kernel "
                    f"with a device flag; pxn_engine_*: MPComm.put_pages_async, {iters} requests in flight, one launch "
                    f"each); "
                    f"roofline = copy-engine H2D of the same bytes on every rank at once",
    }


def gather_bcast_rollout(comm, fstream: torch.cuda.Stream, dev, warmup: int = 3, iters: int = 20) -> dict:
    rank, world = dist.get_rank(), dist.get_world_size()
    raw, ids, lens = RolloutBatch().make(seed=4)
    pad = (-raw.numel()) % PAGE
    if pad:
        raw = torch.cat([raw, torch.zeros(pad, dtype=torch.uint8)])
    nbytes = raw.numel()
    pages = nbytes // PAGE
    host = raw.pin_memory() if rank == 0 else None
    idx = torch.arange(pages, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    exp_crc = ops.crc32_blocks(raw.to(dev), pages)
    fo = nbytes  # completion flag right after the batch
    res = {"bcast_bytes": nbytes, "bcast_tokens": int(ids.shape[0]), "bcast_sequences": int(lens.numel())}
    try:
        grp: Optional[parallel.NvlsGroup] = parallel.NvlsGroup(nbytes + 256)
    except RuntimeError as e:
        grp = None
        res["bcast_nvls"] = f"unavailable: {e}"
    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    if grp is not None:
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()

        def step(seq: int):
            if rank == 0:
                ops.gather_bcast(host.data_ptr(), pages, idx, PAGE, mc_ptr=grp.mc_ptr, mc_flag=grp.mc_ptr + fo,
                                 counter=ctr.data_ptr(), stream=stream, status_ptr=status.data_ptr())
            ops.wait_flag(grp.uc_ptr + fo, seq + 1, WAIT_BUDGET_NS, status.data_ptr(), stream=stream)

        ms = _timed(step, stream, warmup, iters, dev)
        got = ops.crc32_blocks(grp.uc[:nbytes], pages)
        sink = "nvls"
    else:
        bufs = parallel.PeerBuffers(nbytes + 256)
        dist.barrier()

        def step(seq: int):
            if rank == 0:
                ops.gather_bcast(host.data_ptr(), pages, idx, PAGE, dst_ptrs=bufs.ptrs,
                                 flags=[p + fo for p in bufs.ptrs], flag_value=seq + 1, counter=ctr.data_ptr(),
                                 stream=stream, status_ptr=status.data_ptr())
            ops.wait_flag(bufs.local.data_ptr() + fo, seq + 1, WAIT_BUDGET_NS, status.data_ptr(), stream=stream)

        ms = _timed(step, stream, warmup, iters, dev)
        got = ops.crc32_blocks(bufs.local[:nbytes], pages)
        sink = "p2p"
    launches = mpcomm.MPComm.get_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    crc_ok = _all_true(torch.equal(got, exp_crc) and status.item() == 0, dev)

    # The same broadcast through the public engine API: rank 0's
    # broadcast_async from its pinned batch to every other rank's copy (the
    # NVLS group's copies, registered as its members, or plain published
    # buffers): one fused launch per chunk. Its transfer completes when the
    # bytes have landed everywhere, so rank 0's device time is the delivery.
    dest = grp.uc if grp is not None else bufs.local
    dest.zero_()
    if grp is not None:
        grp.register(comm)
    else:
        assert comm.register_memory(dest.data_ptr(), dest.numel()) == 0
    assert comm.publish_buffer(dest.data_ptr(), dest.numel(), 11) == 0
    if rank == 0:
        assert comm.register_memory(host.data_ptr(), nbytes) == 0
    ports = [None] * world
    dist.all_gather_object(ports, comm.get_tcp_port())
    dests = [None] * world
    dist.all_gather_object(dests, dest.data_ptr())
    _host_barrier()
    hosts = [f"bc{r}" for r in range(1, world)]
    if rank == 0:
        for r in range(1, world):
            assert comm.connect(f"bc{r}", "127.0.0.1", ports[r]) == 0
            assert comm.query_remote_buffers(f"bc{r}", "127.0.0.1", ports[r])
    _host_barrier()

    def engine_step(_seq: int):
        # `iters` broadcasts in flight at once, as an application keeps them.
        if rank == 0:
            hs = [comm.broadcast_async(host.data_ptr(), nbytes, hosts, dests[1:]) for _ in range(iters)]
            for h in hs:
                assert h != mpcomm.INVALID_TRANSFER_HANDLE
                assert comm.wait_transfer(h, 60000) == 0, "engine broadcast failed"
                comm.release_transfer(h)

    engine_ms = _timed(engine_step, fstream, 1, 1, dev) / iters
    engine_ok = _all_true(rank == 0 or torch.equal(ops.crc32_blocks(dest[:nbytes], pages), exp_crc), dev)
    dist.barrier()
    comm.unpublish_buffer(dest.data_ptr())
    comm.unregister_memory(dest.data_ptr())
    if rank == 0:
        comm.unregister_memory(host.data_ptr())

    # Library comparator: H2D copy of the batch into rank 0's HBM, then NCCL
    # broadcast to every rank.
    staged = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def nccl_step(_seq: int):
        with torch.cuda.stream(stream):
            if rank == 0:
                staged.copy_(host, non_blocking=True)
            dist.broadcast(staged, src=0)

    nccl_ms = _timed(nccl_step, stream, 2, max(5, iters // 2), dev)
    # Roofline: the PCIe read of the batch on rank 0 at the copy-engine rate
    # (measured now), or the NVLink side (NVLS: the bytes leave rank 0 once;
    # P2P: once per consumer), whichever is slower.
    if rank == 0:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            staged.copy_(host, non_blocking=True)
            e0.record(stream)
            for _ in range(5):
                staged.copy_(host, non_blocking=True)
            e1.record(stream)
        stream.synchronize()
        ce_ms = e0.elapsed_time(e1) / 5
    else:
        ce_ms = 0.0
    ce_ms = _all_max(ce_ms, dev)
    fanout = 1 if sink == "nvls" else max(world - 1, 1)
    roof_ms = max(ce_ms, nbytes * fanout / NVLINK_GBS / 1e6)
    dist.barrier()
    if grp is not None:
        grp.close()
    else:
        bufs.close()
    res.update({
        "gather_bcast_sink": sink,
        "gather_bcast_ms": round(ms, 4),
        "gather_bcast_delivered_gbs": round(nbytes * (world - 1) / (ms * 1e-3) / 1e9, 3),
        "gather_bcast_roofline_ms": round(roof_ms, 4),
        "gather_bcast_roofline_frac": round(roof_ms / ms, 4),
        "gather_bcast_crc_ok": crc_ok,
        "gather_bcast_engine_ms": round(engine_ms, 4),
        "gather_bcast_engine_roofline_frac": round(roof_ms / engine_ms, 4),
        "gather_bcast_engine_crc_ok": engine_ok,
        "gather_bcast_gpu_launches": int(launches),
        "bcast_nccl_ms": round(nccl_ms, 4),
        "bcast_ce_h2d_gbs": round(nbytes / (ce_ms * 1e-3) / 1e9, 3),
        "gather_bcast_what": "rollout batch (1,048,576 x 8 int32 expert IDs + 4,096 lognormal sequences, seed 4) "
                             "in rank 0's pinned DRAM, one gather_bcast launch to every GPU, device completion "
                             "flag on each (gather_bcast_engine_*: MPComm.broadcast_async from rank 0, 20 in flight, one "
                             "fused launch per 32 MiB chunk); roofline = max(copy-engine H2D of the batch, NVLink bytes / 770 GB/s); "
                             "comparator bcast_nccl_ms = copy-engine H2D + NCCL broadcast",
    })
    return res


def hbm_broadcast(dev, warmup: int = 3, iters: int = 20) -> dict:
    """Broadcast of the rollout batch already in rank 0's HBM to every rank:
    this library's all-source NVLS broadcast (every rank loads its 1/N slice
    from rank 0 over NVLink and multicasts it) and single-source NVLS
    broadcast, against NCCL's broadcast of the same buffer. Every iteration
    ends with the same one-element NCCL all-reduce as a delivery barrier
    (data is complete on every rank only once every rank's launch is done);
    kernel_us is the device duration of the broadcast launch alone (trace
    ring, slowest rank)."""
    rank, world = dist.get_rank(), dist.get_world_size()
    raw, _, _ = RolloutBatch().make(seed=4)
    nbytes = raw.numel() - raw.numel() % 4096
    src = parallel.PeerBuffers(nbytes)
    if rank == 0:
        src.local.copy_(raw[:nbytes].to(dev))
    exp = ops.crc32_blocks(raw[:nbytes].to(dev), nbytes // 4096)
    stream = torch.cuda.Stream(device=dev)
    sync = torch.zeros(1, device=dev)
    recv = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    res = {}
    try:
        grp: Optional[parallel.NvlsGroup] = parallel.NvlsGroup(nbytes)
    except RuntimeError as e:
        grp = None
        res["hbm_bcast_nvls"] = f"unavailable: {e}"

    def with_barrier(fn):
        def step(_seq):
            fn()
            with torch.cuda.stream(stream):
                dist.all_reduce(sync)
        return step

    def kernel_us():
        d = sorted(r["duration_us"] for r in mpcomm._native.kernel_trace() if r["kind"] == "nvls_broadcast")
        return _all_max(d[len(d) // 2] if d else 0.0, dev)

    barrier_ms = _timed(with_barrier(lambda: None), stream, warmup, iters, dev)
    tracing = mpcomm._native.kernel_trace_slots() > 0
    if grp is not None:
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        if tracing:
            mpcomm._native.kernel_trace_reset()
        pull_ms = _timed(with_barrier(lambda: grp.broadcast_from(src.ptrs[0], nbytes, stream=stream)), stream,
                         warmup, iters, dev)
        pull_ok = _all_true(torch.equal(ops.crc32_blocks(grp.uc[:nbytes], nbytes // 4096), exp), dev)
        res.update({"hbm_bcast_allsource_ms": round(pull_ms, 4), "hbm_bcast_allsource_crc_ok": pull_ok})
        if tracing:
            k = kernel_us()
            res["hbm_bcast_allsource_kernel_us"] = round(k, 2)
            res["hbm_bcast_allsource_kernel_frac"] = round(nbytes / (k * 1e-6) / 1e9 / NVLINK_GBS, 4)
            mpcomm._native.kernel_trace_reset()
        # The same all-source broadcast with bulk copies of the slice into
        # shared memory (gather_bcast) instead of per-thread loads.
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        bulk_ms = _timed(with_barrier(lambda: grp.broadcast_from(src.ptrs[0], nbytes, stream=stream,
                                                                 method="bulk")), stream, warmup, iters, dev)
        bulk_ok = _all_true(torch.equal(ops.crc32_blocks(grp.uc[:nbytes], nbytes // 4096), exp), dev)
        res.update({"hbm_bcast_allsource_bulk_ms": round(bulk_ms, 4), "hbm_bcast_allsource_bulk_crc_ok": bulk_ok})
        if tracing:
            d = sorted(r["duration_us"] for r in mpcomm._native.kernel_trace() if r["kind"] == "gather_bcast_nvls")
            k = _all_max(d[len(d) // 2] if d else 0.0, dev)
            res["hbm_bcast_allsource_bulk_kernel_us"] = round(k, 2)
            if k:
                res["hbm_bcast_allsource_bulk_kernel_frac"] = round(nbytes / (k * 1e-6) / 1e9 / NVLINK_GBS, 4)
            mpcomm._native.kernel_trace_reset()
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        one_ms = _timed(with_barrier(lambda: rank == 0 and ops.nvls_broadcast(src.local, grp.mc_ptr, nbytes,
                                                                               stream=stream)),
                        stream, warmup, iters, dev)
        one_ok = _all_true(torch.equal(ops.crc32_blocks(grp.uc[:nbytes], nbytes // 4096), exp), dev)
        res.update({"hbm_bcast_onesource_ms": round(one_ms, 4), "hbm_bcast_onesource_crc_ok": one_ok})
        if tracing:
            k = kernel_us()
            res["hbm_bcast_onesource_kernel_us"] = round(k, 2)
            res["hbm_bcast_onesource_kernel_frac"] = round(nbytes / (k * 1e-6) / 1e9 / NVLINK_GBS, 4)
    if rank == 0:
        recv.copy_(src.local)

    def nccl():
        with torch.cuda.stream(stream):
            dist.broadcast(recv, src=0)

    nccl_ms = _timed(with_barrier(nccl), stream, warmup, iters, dev)
    nccl_ok = _all_true(torch.equal(ops.crc32_blocks(recv, nbytes // 4096), exp), dev)
    dist.barrier()
    if grp is not None:
        grp.close()
    src.close()
    res.update({
        "hbm_bcast_bytes": nbytes,
        "hbm_bcast_barrier_ms": round(barrier_ms, 4),
        "hbm_bcast_nccl_ms": round(nccl_ms, 4),
        "hbm_bcast_nccl_crc_ok": nccl_ok,
        "hbm_bcast_what": "rollout batch in rank 0's HBM to every rank; each step = broadcast + one-element NCCL "
                          "all-reduce (hbm_bcast_barrier_ms alone); allsource = NvlsGroup.broadcast_from, "
                          "onesource = nvls_broadcast from rank 0, nccl = torch.distributed.broadcast; "
                          "kernel_frac = bytes / kernel time / 770 GB/s",
    })
    return res


def run(comm, src: torch.Tensor, dst: torch.Tensor, block: int, batch: int, fstream: torch.cuda.Stream) -> dict:
    """All inter-GPU paths; every rank calls it, rank 0 reports."""
    dev = src.device
    out = {}
    out.update(nvlink_putget(comm, src, dst, block, batch, fstream))
    out.update(pxn_forward(comm, fstream, dev))
    out.update(gather_bcast_rollout(comm, fstream, dev))
    out.update(hbm_broadcast(dev))
    return out
