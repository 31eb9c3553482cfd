#!/usr/bin/env python3
"""Headline benchmark: zero-copy PUT/GET GB/s (1 GiB blocks, batch=4).

Workload (the reference's scatter_test "batch=4" PUT/GET, user_examples/
scatter_test.cpp:864-1187, on a single B200 box): every rank owns one GPU
and one MPComm instance. Its memory-pool target is a pinned host-DRAM
buffer it publishes itself (connect-to-self over the TCP control plane, as
the reference's "both" mode), so every byte crosses that GPU's PCIe link,
the path GPUDirect RDMA uses. A step is 4 concurrent PUTs (HBM -> pool,
1 GiB each), wait, then 4 concurrent GETs (pool -> HBM), wait. The data
plane is this library's GPU-fabric rail: the sm_100a bulk-copy kernel
(cp.async.bulk pipeline), no cudaMemcpy. Per-GPU work is fixed, so scaling
is weak.

Timing: CUDA events on the fabric stream (every copy kernel runs on it),
bracketed by barrier + synchronize, K timed steps after W warm-up steps,
max over ranks. Inputs (4 GiB) exceed the 126 MB L2. `e2e` repeats the step
through the Python API with wall-clock timing, adding per step the H2D copy
of the step's request table and a D2H read of the GET result's CRC-32s
(verified against the source CRCs).

At N >= 2 the same run then measures the paths that cross NVLink
(mpcomm.bench.multigpu): GPU-pair PUT/GET through the engine, the fused PXN
gather + forward and the fused rollout-batch gather + broadcast, each
CRC-checked on every rank and reported against its roofline as extra keys.
The headline is also reported against independent ceilings: the copy
engine on one link alone (rank 0, others idle) times N, and the host's own
DRAM write/read bandwidth (CPU threads, no GPU involved).

Reference arm (--impl reference): runs the reference build installed in
baseline/_ref when there is one; otherwise it configures the reference's
source tree (baseline/_ref/src_tree) with CMake and reports the error that
stops it.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N>1 launch with torch.distributed.run (one rank per GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PUT/GET GB/s zero-copy & staging (1 GB, batch=4); gather/PXN GB/s + % roofline"
BASELINE_GBS = 195.7  # reference README.md:113 (zero-copy PUT/GET, 1 GB, batch=4, 4 NICs)
BASELINE_NOTE = ("different hardware and path: the published 195.7 GB/s is 4 x CX-7 NIC-to-NIC RDMA between two "
                 "hosts; this value is HBM <-> host DRAM over each GPU's own PCIe Gen5 x16 link (no RDMA NIC on "
                 "these boxes), so the ratio is context, not parity")
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--block-mb", type=int, default=1024)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the inter-GPU paths and the ceilings measured after the headline")
    p.add_argument("--pool-alloc", choices=["pinned", "hugepage"], default="pinned",
                   help="pinned: cudaHostAlloc via torch; hugepage: anonymous mmap with MADV_HUGEPAGE, "
                        "pinned by MPComm.register_memory (fewer IOMMU translations per byte)")
    return p.parse_args()


def alloc_pool(nbytes: int, how: str):
    import mmap

    import torch

    if how == "pinned":
        return torch.empty(nbytes, dtype=torch.uint8, pin_memory=True), None
    mm = mmap.mmap(-1, nbytes, mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
    try:
        mm.madvise(mmap.MADV_HUGEPAGE)
    except (AttributeError, OSError):
        pass
    t = torch.frombuffer(mm, dtype=torch.uint8)
    t[:: 1 << 21].zero_()  # first touch (2 MiB stride: one fault per huge page)
    return t, mm


def rank_env():
    r = int(os.environ.get("RANK", "0"))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", str(r)))
    return r, w, lr


def bind_numa_local(dev: int):
    """Pins this rank's threads to its GPU's NUMA node (first-touch pool pages land there)."""
    import torch

    try:
        props = torch.cuda.get_device_properties(dev)
        bdf = "%04x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
        node = int(open(f"/sys/bus/pci/devices/{bdf}/numa_node").read().strip())
        if node >= 0:
            cpus = open(f"/sys/devices/system/node/node{node}/cpulist").read().strip()
            cs = set()
            for part in cpus.split(","):
                a, _, b = part.partition("-")
                cs.update(range(int(a), int(b or a) + 1))
            os.sched_setaffinity(0, cs & os.sched_getaffinity(0) or os.sched_getaffinity(0))
            return node
    except Exception:
        pass
    return -1


def reference_unavailable_reason() -> str:
    """Why the reference cannot run here, found by trying: its installed
    package (pip --target baseline/_ref) and the init() it needs, else a CMake
    configure of its source tree."""
    import subprocess
    import tempfile

    pkg = os.path.join(REF_DIR, "mpcomm")
    if os.path.isdir(pkg):
        code = ("import sys; sys.path.insert(0, %r); import mpcomm; c = mpcomm.MPComm(); "
                "print('init_rc', c.init('ref-bench'))" % REF_DIR)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
        out = (r.stdout + r.stderr).strip().splitlines()
        return "installed reference did not initialise: " + " | ".join(out[-3:])
    src = os.path.join(REF_DIR, "src_tree")
    if not os.path.isfile(os.path.join(src, "CMakeLists.txt")):
        return "reference not installed in baseline/_ref and its source tree is absent"
    with tempfile.TemporaryDirectory(prefix="mpcomm-ref-") as bdir:
        r = subprocess.run(["cmake", "-S", src, "-B", bdir], capture_output=True, text=True, timeout=300)
    if r.returncode == 0:
        return "reference configured but is not installed (pip install into baseline/_ref failed earlier)"
    lines = [ln.strip() for ln in (r.stdout + r.stderr).splitlines() if ln.strip()]
    err = [ln for i, ln in enumerate(lines) if "Error" in ln or (i and "Error" in lines[i - 1])]
    return ("reference build fails offline (CMake configure rc=%d): %s; the boxes have no rdma-core and no "
            "RDMA NIC, which its init() also requires" % (r.returncode, " ".join(err[:3]) or lines[-1]))


def main():
    args = parse()
    rank, world, local = rank_env()
    if world > 1 and not args.no_extras:
        # Device start/end of the broadcast launches measured after the
        # headline (kernel trace ring; read once, outside every timed loop).
        os.environ.setdefault("MPCOMM_KERNEL_TRACE", "4096")
    if args.impl == "reference":
        # Every rank reaches the same conclusion; rank 0 reports it.
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reference_unavailable_reason()}), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    import mpcomm
    from mpcomm.ops import crc32_blocks
    from mpcomm.utils import ClockSampler

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa = bind_numa_local(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    block = args.block_mb << 20
    batch = args.batch
    total = block * batch

    # Host DRAM ceiling, measured by CPU threads alone (rank 0; GPUs idle).
    host_bw = {}
    if rank == 0 and not args.no_extras:
        host_bw = mpcomm._native.host_bandwidth(2 << 30, 0, numa, 3)
    barrier()

    gen = torch.Generator(device=dev)
    gen.manual_seed(2 + rank)
    src = torch.randint(0, 256, (total,), dtype=torch.uint8, device=dev, generator=gen)
    dst = torch.empty(total, dtype=torch.uint8, device=dev)
    pool, pool_map = alloc_pool(total, args.pool_alloc)

    comm = mpcomm.MPComm()
    assert comm.init(f"rank{rank}") == 0
    assert comm.get_fabric_name() == "nvl", "GPU fabric expected"
    assert comm.start_accept_thread() == 0
    for t in (src, dst, pool):
        assert comm.register_memory(t.data_ptr(), t.numel()) == 0
    assert comm.publish_buffer(pool.data_ptr(), total) == 0
    port = comm.get_tcp_port()
    assert comm.connect("pool", "127.0.0.1", port) == 0
    assert comm.query_remote_buffers("pool", "127.0.0.1", port)
    fstream = torch.cuda.Stream(device=dev)
    comm.set_fabric_stream(fstream.cuda_stream)

    sp, pp, dp = src.data_ptr(), pool.data_ptr(), dst.data_ptr()

    def run_phase(put: bool, s_ptr: int = 0, d_ptr: int = 0):
        s_ptr, d_ptr = s_ptr or sp, d_ptr or dp
        hs = []
        for i in range(batch):
            if put:
                h = comm.put_async(s_ptr + i * block, "pool", pp + i * block, block)
            else:
                h = comm.get_async(d_ptr + i * block, "pool", pp + i * block, block)
            assert h != mpcomm.INVALID_TRANSFER_HANDLE
            hs.append(h)
        for h in hs:
            rc = comm.wait_transfer(h, 120000)
            assert rc == 0, f"transfer failed rc={rc}"
            comm.release_transfer(h)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def step(times=None):
        if times is not None:
            ev[0].record(fstream)
        run_phase(True)
        if times is not None:
            ev[1].record(fstream)
        run_phase(False)
        if times is not None:
            ev[2].record(fstream)
            fstream.synchronize()
            times.append((ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])))

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    # correctness of the round trip (outside the timed region)
    torch.cuda.synchronize()
    crc_src = crc32_blocks(src, batch)
    crc_dst = crc32_blocks(dst, batch)
    torch.cuda.synchronize()
    assert torch.equal(crc_src, crc_dst), "PUT/GET round trip corrupted data"

    # Copy-engine roofline of the same path (cudaMemcpyAsync; timing only),
    # run on every rank at once so it includes the host-memory ceiling the
    # ranks share; aggregate = world * bytes / max-over-ranks time.
    ce = []
    s_ce = torch.cuda.Stream(device=dev)
    for d2h in (True, False):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s_ce):
            (pool.copy_(src, non_blocking=True) if d2h else dst.copy_(pool, non_blocking=True))
        s_ce.synchronize()
        barrier()
        with torch.cuda.stream(s_ce):
            a.record(s_ce)
            for _ in range(2):
                if d2h:
                    pool.copy_(src, non_blocking=True)
                else:
                    dst.copy_(pool, non_blocking=True)
            b.record(s_ce)
        s_ce.synchronize()
        t = torch.tensor([a.elapsed_time(b) / 2], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ce.append(world * total / (t.item() * 1e-3) / 1e9)

    # ---- device-timed region ----
    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    barrier()
    torch.cuda.synchronize()
    times = []
    with ClockSampler(local) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(fstream)
        for _ in range(args.steps):
            step(times)
        t_end.record(fstream)
        torch.cuda.synchronize()
    barrier()
    launches = mpcomm.MPComm.get_kernel_launch_count() - launches0
    ms = t_start.elapsed_time(t_end) / args.steps
    put_ms = sum(t[0] for t in times) / len(times)
    get_ms = sum(t[1] for t in times) / len(times)
    stats = torch.tensor([ms, put_ms, get_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, put_ms, get_ms = stats.tolist()

    # ---- end-to-end through the public API (wall clock) ----
    e2e = None
    if not args.no_e2e:
        req_host = torch.tensor([[pp + i * block, block] for i in range(batch)], dtype=torch.int64).pin_memory()
        req_dev = torch.empty_like(req_host, device=dev)
        crc_host = torch.empty(batch, dtype=torch.int32).pin_memory()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            req_dev.copy_(req_host, non_blocking=True)   # step's request table H2D
            torch.cuda.current_stream().synchronize()
            step()
            crc32_blocks(dst, batch, out=crc_dst)
            crc_host.copy_(crc_dst, non_blocking=True)    # step's result D2H
            torch.cuda.current_stream().synchronize()
            assert torch.equal(crc_host, crc_src.cpu())
        wall = torch.tensor([(time.perf_counter() - t0) / args.steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(wall, op=dist.ReduceOp.MAX)
        e2e = {"value": round(world * 2 * total / wall.item() / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": req_host.numel() * 8, "d2h_bytes_per_step": batch * 4}

    # Paged KV gather / scatter on every rank at once:
    # the 4 GiB host pool is 65,536 Llama-3-8B KV pages of 64 KiB; 4,096 of
    # them (seed 1) are gathered into HBM with tmaGather and scattered back
    # with tmaScatter (the same bytes, so the pool is unchanged), checked
    # against torch indexing of the pool.
    kv = {}
    if not args.no_extras:
        from mpcomm.models import LLAMA3_8B_KV

        pbytes = LLAMA3_8B_KV.page_bytes
        npages, nreq = total // pbytes, 4096
        kv_idx_cpu = LLAMA3_8B_KV.sample_pages(npages, nreq, seed=1)
        kv_idx = kv_idx_cpu.to(dev)
        kv_out = torch.empty(nreq * pbytes, dtype=torch.uint8, device=dev)
        dram = comm.map_dram_to_gpu(pp, total)
        assert dram, "map_dram_to_gpu failed"
        fs = fstream.cuda_stream
        kv_ms = []
        for gather in (True, False):
            def one():
                if gather:
                    rc = comm.tma_gather(dram, kv_idx.data_ptr(), kv_out.data_ptr(), nreq, pbytes, 0, 0, fs)
                else:
                    rc = comm.tma_scatter(kv_out.data_ptr(), kv_idx.data_ptr(), dram, nreq, pbytes, 0, 0, fs)
                assert rc == 0
            for _ in range(2):
                one()
            torch.cuda.synchronize()
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(fstream)
            for _ in range(5):
                one()
            b.record(fstream)
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b) / 5], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            kv_ms.append(t.item())
        ok = torch.equal(kv_out.view(nreq, pbytes).cpu(), pool.view(npages, pbytes)[kv_idx_cpu])
        okt = torch.tensor([1 if ok else 0], device=dev)
        if world > 1:
            dist.all_reduce(okt, op=dist.ReduceOp.MIN)
        comm.unmap_dram_from_gpu(pp)
        kv_bytes = world * nreq * pbytes
        kv = {"kv_gather_gbs": round(kv_bytes / (kv_ms[0] * 1e-3) / 1e9, 3),
              "kv_scatter_gbs": round(kv_bytes / (kv_ms[1] * 1e-3) / 1e9, 3),
              "kv_gather_roofline_frac": round(kv_bytes / (kv_ms[0] * 1e-3) / 1e9 / ce[1], 4),
              "kv_scatter_roofline_frac": round(kv_bytes / (kv_ms[1] * 1e-3) / 1e9 / ce[0], 4),
              "kv_bitexact": bool(okt.item()),
              "kv_what": "4,096 x 64 KiB Llama-3-8B KV pages (seed 1) of a 65,536-page pinned pool per rank, "
                         "tmaGather into HBM / tmaScatter back, all ranks at once; roofline = concurrent "
                         "copy-engine H2D / D2H of the pool"}
        del kv_out

    # Staging (non-zero-copy) PUT/GET: the same 4 x 1 GiB from and into HBM
    # that was never registered; the library stages it through slabs in the
    # same GPU's HBM (device-to-device stage copies, then the zero-copy
    # engine). Every kernel of it runs on the fabric stream, so CUDA events
    # there bracket the whole transfer.
    staging = {}
    if not args.no_extras:
        ssrc = src.clone()
        sdst = torch.zeros_like(dst)
        torch.cuda.synchronize()
        st_ms = []
        for put in (True, False):
            for _ in range(2):
                run_phase(put, ssrc.data_ptr(), sdst.data_ptr())
            torch.cuda.synchronize()
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(fstream)
            for _ in range(3):
                run_phase(put, ssrc.data_ptr(), sdst.data_ptr())
            b.record(fstream)
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b) / 3], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            st_ms.append(t.item())
        ok = torch.equal(crc32_blocks(sdst, batch), crc_src)
        okt = torch.tensor([1 if ok else 0], device=dev)
        if world > 1:
            dist.all_reduce(okt, op=dist.ReduceOp.MIN)
        staging = {"staging_put_gbs": round(world * total / (st_ms[0] * 1e-3) / 1e9, 3),
                   "staging_get_gbs": round(world * total / (st_ms[1] * 1e-3) / 1e9, 3),
                   "staging_crc_ok": bool(okt.item()),
                   "staging_what": "PUT/GET of 4 x 1 GiB from/into unregistered HBM through the staging pool "
                                   "(HBM slabs, device stage copies, then the zero-copy engine); published "
                                   "reference bcopy 91.9 / 84.5 GB/s is NIC-to-NIC on other hardware"}
        del ssrc, sdst

    # Copy engine on one link alone (rank 0; the others wait): the per-link
    # ceiling, N times which the headline could reach if nothing were shared.
    solo = [0.0, 0.0]
    if not args.no_extras:
        barrier()
        if rank == 0:
            for k, d2h in enumerate((True, False)):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(s_ce):
                    a.record(s_ce)
                    for _ in range(2):
                        (pool.copy_(src, non_blocking=True) if d2h else dst.copy_(pool, non_blocking=True))
                    b.record(s_ce)
                s_ce.synchronize()
                solo[k] = 2 * total / (a.elapsed_time(b) * 1e-3) / 1e9
        barrier()

    # The host pool is not used past this point.
    comm.unpublish_buffer(pp)
    comm.unregister_memory(pp)
    del pool
    extras = {}
    if world > 1 and not args.no_extras:
        from mpcomm.bench import multigpu

        torch.cuda.synchronize()
        extras = multigpu.run(comm, src, dst, block, batch, fstream)

    value = world * 2 * total / (ms * 1e-3) / 1e9
    if rank == 0:
        cs = clocks.summary()
        out = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / BASELINE_GBS, 4),
            "vs_baseline_note": BASELINE_NOTE,
            "dtype": "uint8",
            "data": "synthetic (uint8 uniform, seed 2+rank, torch generator on device)",
            "config": {
                "model": "mpcomm zero-copy PUT/GET, HBM <-> pinned host-DRAM pool, GPU-fabric rail "
                         "(sm_100a cp.async.bulk copy kernel)",
                "global_batch": batch * world,
                "seq_len": block,
                "block_bytes": block,
                "batch_per_gpu": batch,
                "parallelism": f"rail-per-gpu x{world}",
                "l2": f"inputs {total >> 20} MiB per GPU > 126 MB L2 (no flush needed)",
                "numa_node": numa,
                "pool_alloc": args.pool_alloc,
            },
            "put_gbs": round(world * total / (put_ms * 1e-3) / 1e9, 3),
            "get_gbs": round(world * total / (get_ms * 1e-3) / 1e9, 3),
            "roofline": {
                "what": "copy-engine cudaMemcpyAsync on the same pinned buffers, all ranks at once "
                        "(aggregate GB/s)",
                "ce_d2h_gbs": round(ce[0], 3),
                "ce_h2d_gbs": round(ce[1], 3),
                "put_frac": round(world * total / (put_ms * 1e-3) / 1e9 / ce[0], 4),
                "get_frac": round(world * total / (get_ms * 1e-3) / 1e9 / ce[1], 4),
                "step_frac": round(2 * world * total / (ms * 1e-3) / 1e9 /
                                   (2 / (1 / ce[0] + 1 / ce[1])), 4),
            },
            "clocks": {"sm_mhz": cs["sm_mhz"], "sm_max_mhz": cs["sm_max_mhz"], "reasons": cs["reasons"]},
            "gpu_launches": int(launches),
            "impl": "ours",
        }
        if e2e:
            out["e2e"] = e2e
        if solo[0] and host_bw:
            put_gbs, get_gbs = out["put_gbs"], out["get_gbs"]
            out["ceilings"] = {
                "what": "N x the copy engine on one link alone (rank 0, others idle), and the host DRAM "
                        "bandwidth of CPU threads alone (memset / read; no GPU involved)",
                "solo_ce_d2h_gbs": round(solo[0], 3), "solo_ce_h2d_gbs": round(solo[1], 3),
                "links_put_gbs": round(world * solo[0], 3), "links_get_gbs": round(world * solo[1], 3),
                "put_frac_of_links": round(put_gbs / (world * solo[0]), 4),
                "get_frac_of_links": round(get_gbs / (world * solo[1]), 4),
                "host_cpu_write_gbs": round(host_bw["write_gbs"], 3),
                "host_cpu_read_gbs": round(host_bw["read_gbs"], 3),
                "host_cpu_threads": host_bw["threads"],
                "put_frac_of_host_cpu_write": round(put_gbs / host_bw["write_gbs"], 4),
                "get_frac_of_host_cpu_read": round(get_gbs / host_bw["read_gbs"], 4),
            }
        out.update(kv)
        out.update(staging)
        out.update(extras)
        print(json.dumps(out), flush=True)
    comm.shutdown()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
