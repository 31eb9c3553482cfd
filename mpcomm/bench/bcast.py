"""RL rollout / R3 expert-ID broadcast under H2D-aware QoS (one process per GPU).

Batch (seed 4): 1,048,576 tokens x top_k=8 int32 expert IDs in [0, 256) plus
4,096 int32 token sequences with lognormal(7, 0.8) lengths clipped to
[16, 32768], packed in pinned host memory of rank 0. Rank 0 H2D-gathers it
(64 KiB pages, tmaGather) into HBM and broadcasts it to every GPU:
  nvls    multimem.st into an NVLS multicast object bound on all GPUs
  fanout  the same bytes stored to each peer's IPC-mapped buffer
  nccl    torch.distributed.broadcast (library baseline)
  fused_nvls / fused_p2p  ONE kernel (gather_bcast) that reads the pages from
          host DRAM into shared memory and stores each tile straight to the
          multicast address (multimem.st) or to every GPU's buffer (bulk
          stores): no staging in HBM, PCIe read and NVLink fan-out overlap.
Times: CUDA events on rank 0's stream for gather+broadcast, then a device
barrier (NCCL all-reduce) so the max over ranks covers delivery.

QoS part (rank 0 only, one GPU): background GETs (pinned host pool -> HBM,
the same PCIe direction as the H2D gather; 2 MiB chunks) run through MPComm
while the gather repeats; the gather latency and the background bandwidth
are measured with QoS off, and with enable_h2d_qos(rate) (0 = pause READ
posts while the gather kernel's window is open).

    torchrun --nproc-per-node 8 -m mpcomm.bench.bcast
"""
from __future__ import annotations

import argparse
import json
import os
import threading
import time

import torch
import torch.distributed as dist

import mpcomm
from mpcomm import ops, parallel
from mpcomm.models import RolloutBatch

PAGE = 65536


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--qos-rate", type=float, default=0.0, help="bytes/s during H2D windows (0 = pause)")
    ap.add_argument("--bg-mb", type=int, default=1024)
    ap.add_argument("--no-qos", action="store_true")
    ap.add_argument("--sweep-ctas", default="", help="comma list: time the broadcast alone per grid size")
    ap.add_argument("--variants", default="", help="comma list of NVLS store variants (0-3) to time alone")
    ap.add_argument("--pull", action="store_true",
                    help="also time the all-source broadcast: every rank reads its 1/world slice of rank 0's "
                         "buffer over NVLink and multicasts it")
    a = ap.parse_args(argv)
    # Device start/end of every broadcast launch (kernel trace ring).
    os.environ.setdefault("MPCOMM_KERNEL_TRACE", "4096")
    rank, world, local = parallel.init_from_env("nccl")
    dev = torch.device("cuda", local)
    raw, ids, lens = RolloutBatch().make(seed=4)
    pad = (-raw.numel()) % PAGE
    if pad:
        raw = torch.cat([raw, torch.zeros(pad, dtype=torch.uint8)])
    nbytes = raw.numel()
    pages = nbytes // PAGE
    host = raw.pin_memory() if rank == 0 else None
    idx = torch.arange(pages, dtype=torch.int64, device=dev)
    staged = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    comm = mpcomm.MPComm()
    dram = comm.map_dram_to_gpu(host.data_ptr(), nbytes) if rank == 0 else 0
    sptr = stream.cuda_stream

    def gather():
        if rank == 0:
            rc = comm.tma_gather(dram, idx.data_ptr(), staged.data_ptr(), pages, PAGE, 0, 0, sptr)
            assert rc == 0

    try:
        grp = parallel.NvlsGroup(nbytes)
    except RuntimeError as e:
        grp = None
        nvls_err = str(e)
    peers = parallel.PeerBuffers(nbytes)
    recv = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    sync = torch.zeros(1, device=dev)

    def timed(step):
        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.iters):
            step()
            with torch.cuda.stream(stream):
                dist.all_reduce(sync)  # delivery barrier on the device
        e1.record(stream)
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item()

    def step_nvls():
        gather()
        if rank == 0:
            ops.nvls_broadcast(staged, grp.mc_ptr, nbytes, stream=stream)

    def step_fanout():
        gather()
        if rank == 0:
            ops.p2p_fanout(staged, [peers.ptrs[r] for r in range(1, world)], nbytes, stream=stream)

    def step_fused_nvls():
        if rank == 0:
            ops.gather_bcast(dram, pages, idx, PAGE, mc_ptr=grp.mc_ptr, stream=stream)

    def step_fused_p2p():
        if rank == 0:
            ops.gather_bcast(dram, pages, idx, PAGE, dst_ptrs=peers.ptrs, stream=stream)

    def step_nccl():
        gather()
        with torch.cuda.stream(stream):
            dist.broadcast(staged if rank == 0 else recv, src=0)

    def kernel_us(kind):
        """Median device duration of the `kind` launches since the last reset (rank 0)."""
        if rank != 0:
            return None
        d = sorted(r["duration_us"] for r in mpcomm._native.kernel_trace() if r["kind"] == kind)
        return round(d[len(d) // 2], 2) if d else None

    res = {"metric": "rollout batch H2D gather + broadcast", "n_gpus": world, "bytes": nbytes,
           "tokens": ids.shape[0], "top_k": ids.shape[1], "sequences": int(lens.numel()),
           "seq_tokens": int(lens.sum())}
    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    g_ms = timed(gather)
    res["gather_ms"] = round(g_ms, 4)
    # Copy-engine H2D of the same bytes (contiguous pinned -> HBM) on rank 0:
    # the PCIe side of every path's roofline.
    if rank == 0:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(2):
                staged.copy_(host, non_blocking=True)
            e0.record(stream)
            for _ in range(5):
                staged.copy_(host, non_blocking=True)
            e1.record(stream)
        stream.synchronize()
        ce_ms = e0.elapsed_time(e1) / 5
    else:
        ce_ms = 0.0
    t = torch.tensor([ce_ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ce_ms = t.item()
    res["ce_h2d_ms"] = round(ce_ms, 4)
    res["ce_h2d_gbs"] = round(nbytes / (ce_ms * 1e-3) / 1e9, 3)
    # Roofline of gather + broadcast: the slower of the PCIe read (copy-engine
    # rate) and the NVLink side (NVLS: the bytes leave rank 0 once; P2P:
    # world-1 times) at 770 GB/s per direction.
    nvl_gbs = 770.0
    res["roofline_ms"] = {"nvls": round(max(ce_ms, nbytes / nvl_gbs / 1e6), 4),
                          "p2p": round(max(ce_ms, nbytes * max(world - 1, 1) / nvl_gbs / 1e6), 4)}
    if grp is not None and world > 1:
        res["nvls_ms"] = round(timed(step_nvls), 4)
        ok = torch.equal(grp.uc[:nbytes].cpu(), raw)
    else:
        res["nvls"] = f"unavailable: {nvls_err}" if grp is None else "single GPU"
        ok = True
    if world > 1:
        res["fanout_ms"] = round(timed(step_fanout), 4)
        if rank != 0:
            ok = ok and torch.equal(peers.local.cpu(), raw)
        res["nccl_ms"] = round(timed(step_nccl), 4)
        if grp is not None:
            grp.uc.zero_()
            torch.cuda.synchronize()
            if rank == 0:
                mpcomm._native.kernel_trace_reset()
            res["fused_nvls_ms"] = round(timed(step_fused_nvls), 4)
            ok = ok and torch.equal(grp.uc[:nbytes].cpu(), raw)
            res["fused_nvls_kernel_us"] = kernel_us("gather_bcast_nvls")
        peers.local.zero_()
        torch.cuda.synchronize()
        if rank == 0:
            mpcomm._native.kernel_trace_reset()
        res["fused_p2p_ms"] = round(timed(step_fused_p2p), 4)
        ok = ok and torch.equal(peers.local.cpu(), raw)
        res["fused_p2p_kernel_us"] = kernel_us("gather_bcast_p2p")
        for k, roof in (("fused_nvls", "nvls"), ("fused_p2p", "p2p"), ("nvls", "nvls"), ("fanout", "p2p")):
            if f"{k}_ms" in res:
                res[f"{k}_roofline_frac"] = round(res["roofline_ms"][roof] / res[f"{k}_ms"], 4)
    okt = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    res["bitexact"] = bool(okt.item())
    res["gpu_launches"] = int(mpcomm.MPComm.get_kernel_launch_count() - launches0)
    for k in ("nvls", "fanout", "nccl", "fused_nvls", "fused_p2p"):
        if f"{k}_ms" in res:
            res[f"{k}_delivered_gbs"] = round(nbytes * (world - 1) / (res[f"{k}_ms"] * 1e-3) / 1e9, 3)
    # NVLink roofline of the broadcast (after the gather): NVLS sends the
    # bytes once through the switch; fan-out sends them world-1 times.
    res["roofline_note"] = "NVLink 770 GB/s per direction per GPU (measured peer copy)"

    if a.sweep_ctas and world > 1:
        rows = []
        for ctas in [int(x) for x in a.sweep_ctas.split(",")]:
            row = {"ctas": ctas}
            if grp is not None:
                row["nvls_ms"] = round(timed(lambda: rank == 0 and ops.nvls_broadcast(
                    staged, grp.mc_ptr, nbytes, max_ctas=ctas, stream=stream)), 4)
            row["fanout_ms"] = round(timed(lambda: rank == 0 and ops.p2p_fanout(
                staged, [peers.ptrs[r] for r in range(1, world)], nbytes, max_ctas=ctas, stream=stream)), 4)
            rows.append(row)
        res["broadcast_only_sweep"] = rows

    if a.variants and world > 1 and grp is not None:
        rows = []
        for v in [int(x) for x in a.variants.split(",")]:
            mpcomm._native._set_nvls_variant(v)
            if rank == 0:
                mpcomm._native.kernel_trace_reset()
            ms = timed(lambda: rank == 0 and ops.nvls_broadcast(staged, grp.mc_ptr, nbytes, stream=stream))
            ok_v = torch.tensor([1 if rank == 0 or torch.equal(grp.uc[:nbytes].cpu(), raw) else 0], device=dev)
            dist.all_reduce(ok_v, op=dist.ReduceOp.MIN)
            ok_v = bool(ok_v.item())
            k = kernel_us("nvls_broadcast")
            rows.append({"variant": v, "with_barrier_ms": round(ms, 4), "kernel_us": k,
                         "kernel_gbs": round(nbytes / (k * 1e-6) / 1e9, 1) if k else None, "ok": ok_v})
        mpcomm._native._set_nvls_variant(0)
        # The same broadcast from HBM through gather_bcast: bulk (TMA) loads of
        # 16 KiB tiles into shared memory, multimem.st from there.
        if rank == 0:
            mpcomm._native.kernel_trace_reset()
        grp.uc.zero_()
        torch.cuda.synchronize()
        ms = timed(lambda: rank == 0 and ops.gather_bcast(staged.data_ptr(), pages, idx, PAGE, mc_ptr=grp.mc_ptr,
                                                          stream=stream))
        ok_v = torch.tensor([1 if rank == 0 or torch.equal(grp.uc[:nbytes].cpu(), raw) else 0], device=dev)
        dist.all_reduce(ok_v, op=dist.ReduceOp.MIN)
        k = kernel_us("gather_bcast_nvls")
        rows.append({"variant": "tma_smem", "with_barrier_ms": round(ms, 4), "kernel_us": k,
                     "kernel_gbs": round(nbytes / (k * 1e-6) / 1e9, 1) if k else None, "ok": bool(ok_v.item())})
        res["nvls_variants"] = rows

    if a.pull and world > 1 and grp is not None:
        # All-source broadcast of a batch already in rank 0's HBM: rank r
        # pulls slice r from rank 0 (plain loads over NVLink) and multimem-
        # stores it, so 8 GPUs share the multicast work instead of one.
        src = parallel.PeerBuffers(nbytes)
        if rank == 0:
            src.local.copy_(staged)
        grp.uc.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        mpcomm._native.kernel_trace_reset()

        def step_pull():
            grp.broadcast_from(src.ptrs[0], nbytes, stream=stream)

        ms = timed(step_pull)
        ok_v = torch.tensor([1 if torch.equal(grp.uc[:nbytes].cpu(), raw) else 0], device=dev)
        dist.all_reduce(ok_v, op=dist.ReduceOp.MIN)
        d = sorted(r["duration_us"] for r in mpcomm._native.kernel_trace() if r["kind"] == "nvls_broadcast")
        k = torch.tensor([d[len(d) // 2] if d else 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(k, op=dist.ReduceOp.MAX)
        res["nvls_pull"] = {"with_barrier_ms": round(ms, 4), "kernel_us_max_rank": round(k.item(), 2),
                            "kernel_gbs": round(nbytes / (k.item() * 1e-6) / 1e9, 1) if k.item() else None,
                            "ok": bool(ok_v.item())}
        dist.barrier()
        src.close()
    if rank == 0 and not a.no_qos:
        res["qos"] = qos_experiment(comm, host, dram, idx, staged, pages, stream, a)
    dist.barrier()
    if grp is not None:
        grp.close()
    peers.close()
    if rank == 0:
        comm.unmap_dram_from_gpu(host.data_ptr())
        print(json.dumps(res), flush=True)
    comm.shutdown()
    dist.barrier()
    dist.destroy_process_group()


def qos_experiment(comm0, host, dram, idx, staged, pages, stream, a):
    """Gather latency with background GET traffic on the same PCIe link."""
    # Small chunks and a shallow queue bound the bytes already in flight when
    # a window opens (a launched chunk cannot be recalled): 2 QPs x 2 x 2 MiB.
    os.environ["MPCOMM_NVL_CHUNK_SIZE"] = str(2 << 20)
    os.environ["MPCOMM_NVL_OUTSTANDING_PER_QP"] = "2"
    os.environ["MPCOMM_QPS_PER_CONNECTION"] = "2"
    bg = mpcomm.MPComm()
    assert bg.init("qos-bg") == 0 and bg.start_accept_thread() == 0
    n = a.bg_mb << 20
    pool = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(n, dtype=torch.uint8, device="cuda")
    for t in (pool, dst):
        assert bg.register_memory(t.data_ptr(), n) == 0
    assert bg.publish_buffer(pool.data_ptr(), n) == 0
    port = bg.get_tcp_port()
    assert bg.connect("pool", "127.0.0.1", port) == 0 and bg.query_remote_buffers("pool", "127.0.0.1", port)
    sptr = stream.cuda_stream
    nbytes = pages * PAGE
    out = {}

    def gather_latency(comm):
        lat = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(a.iters):
            e0.record(stream)
            assert comm.tma_gather(dram, idx.data_ptr(), staged.data_ptr(), pages, PAGE, 0, 0, sptr) == 0
            e1.record(stream)
            stream.synchronize()
            lat.append(e0.elapsed_time(e1))
            time.sleep(0.002)
        lat.sort()
        return lat[len(lat) // 2]

    def with_background(fn):
        stop = threading.Event()

        def loop():
            while not stop.is_set():
                h = bg.get_async(dst.data_ptr(), "pool", pool.data_ptr(), n)
                assert bg.wait_transfer(h, 60000) == 0
                bg.release_transfer(h)
        t = threading.Thread(target=loop)
        t.start()
        time.sleep(0.05)
        b0, t0 = bg.get_nic_completed_bytes(), time.perf_counter()  # chunk-exact byte counter
        r = fn()
        b1, dt = bg.get_nic_completed_bytes(), time.perf_counter() - t0
        stop.set()
        t.join()
        return r, (b1 - b0) / dt / 1e9

    out["gather_ms_idle"] = round(gather_latency(comm0), 4)
    lat, bw = with_background(lambda: gather_latency(comm0))
    out["gather_ms_bg_qos_off"], out["bg_gbs_qos_off"] = round(lat, 4), round(bw, 3)
    bg.enable_h2d_qos(int(a.qos_rate), 0)
    # The window is opened by kernels launched through the MPComm that owns
    # the QoS state: gather through `bg`, which both paces and is paced.
    dram_bg = bg.map_dram_to_gpu(host.data_ptr(), nbytes)
    lat, bw = with_background(lambda: gather_latency_via(bg, dram_bg, idx, staged, pages, stream, a))
    out["gather_ms_bg_qos_on"], out["bg_gbs_qos_on"] = round(lat, 4), round(bw, 3)
    out["qos_rate_bps"] = a.qos_rate
    out["gather_bytes"] = nbytes
    bg.disable_h2d_qos()
    bg.unmap_dram_from_gpu(host.data_ptr())
    bg.shutdown()
    return out


def gather_latency_via(comm, dram, idx, staged, pages, stream, a):
    lat = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(a.iters):
        e0.record(stream)
        assert comm.tma_gather(dram, idx.data_ptr(), staged.data_ptr(), pages, PAGE, 0, 0, stream.cuda_stream) == 0
        e1.record(stream)
        stream.synchronize()
        lat.append(e0.elapsed_time(e1))
        time.sleep(0.002)
    lat.sort()
    return lat[len(lat) // 2]


if __name__ == "__main__":
    main()
