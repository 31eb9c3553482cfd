"""Sparse H2D movers and fabric GET/PUT into GPU or CPU memory.

    python -m mpcomm.bench.h2d_nic2gpu --path h2d [--op gather|scatter|both]
        [--num-blocks 2048 --block-size 272 --pool-multiplier 4] [--h2d-mode tma]
        [--cuda-copy-baseline] [--single] [--report-every N] [--csv out.csv]
    python -m mpcomm.bench.h2d_nic2gpu --path nic2gpu [--op get|put|both]
        [--sizes 512K,...,1G] [--dest gpu|cpu] [--target host:ip:port]

--path h2d: tmaGather / tmaScatter of --num-blocks random blocks of
--block-size bytes between a pinned pool (--pool-multiplier x larger) and
HBM; per iteration the CUDA-event latency (start event queued behind a short
device sleep so host launch time is excluded) gives avg / p50 / p99 / peak
GB/s; --cuda-copy-baseline adds a contiguous cudaMemcpyAsync of the same
byte count (the copy-engine ceiling for that size).
--path nic2gpu: GET (remote -> local) and PUT (local -> remote) of each size
into a local HBM (--dest gpu) or pinned DRAM (--dest cpu) buffer; the remote
is --target (a running target, host_id:ip:port) or, by default, this
process's own pinned pool (connect-to-self: the PCIe path of this GPU).
Wall-clock GB/s over --iterations after --warmup, as the reference's tool.
Rows print as a table and, with --csv, to a CSV file; one JSON line last.

Parity: reference user_examples/qos_bench/bench_h2d_nic2gpu.py:155-376.
"""
from __future__ import annotations

import argparse
import csv
import json
import statistics
import time

import torch

import mpcomm
from mpcomm.harness.common import parse_size

MODES = {"auto": 0, "sm": 1, "tma": 2}


def _pct(v, q):
    s = sorted(v)
    return s[min(len(s) - 1, int(round(q * (len(s) - 1))))]


def run_h2d(comm, a):
    if a.num_blocks <= 0 or a.block_size <= 0 or a.block_size % 16:
        raise ValueError("num-blocks > 0 and block-size a positive multiple of 16")
    mode = MODES[a.h2d_mode]
    payload = a.num_blocks * a.block_size
    pool_blocks = max(a.num_blocks * a.pool_multiplier, a.num_blocks)
    ops = ["gather", "scatter"] if a.op == "both" else ["gather" if a.op in ("gather", "get") else "scatter"]
    stream = torch.cuda.Stream()
    rows = []
    for op in ops:
        pool = torch.empty(pool_blocks * a.block_size, dtype=torch.uint8).pin_memory()
        if op == "gather":
            pool.random_(0, 255)
        else:
            pool.zero_()
        dram = comm.map_dram_to_gpu(pool.data_ptr(), pool.numel())
        assert dram, "map_dram_to_gpu failed"
        idx = torch.randperm(pool_blocks, generator=torch.Generator().manual_seed(5))[:a.num_blocks].cuda()
        buf = (torch.empty(payload, dtype=torch.uint8, device="cuda") if op == "gather"
               else torch.randint(0, 255, (payload,), dtype=torch.uint8, device="cuda"))

        def submit():
            if op == "gather":
                return comm.tma_gather(dram, idx.data_ptr(), buf.data_ptr(), a.num_blocks, a.block_size,
                                       a.max_sm_count, mode, stream.cuda_stream)
            return comm.tma_scatter(buf.data_ptr(), idx.data_ptr(), dram, a.num_blocks, a.block_size,
                                    a.max_sm_count, mode, stream.cuda_stream)

        for _ in range(a.warmup):
            assert submit() == 0
        stream.synchronize()
        lat = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(a.iterations):
            with torch.cuda.stream(stream):
                torch.cuda._sleep(40000)
            e0.record(stream)
            assert submit() == 0, f"{op} submission failed"
            e1.record(stream)
            e1.synchronize()
            lat.append(e0.elapsed_time(e1) * 1e3)
            if a.report_every and (i + 1) % a.report_every == 0:
                w = lat[-a.report_every:]
                print(f"[H2D-LIVE] op={op} iters {i + 2 - a.report_every}-{i + 1}: avg {statistics.mean(w):.2f} us "
                      f"({payload / (statistics.mean(w) * 1e-6) / 1e9:.2f} GB/s)", flush=True)
        torch.cuda.synchronize()
        if op == "gather":
            ok = torch.equal(buf.view(a.num_blocks, a.block_size).cpu(), pool.view(-1, a.block_size)[idx.cpu()])
        else:
            ok = torch.equal(pool.view(-1, a.block_size)[idx.cpu()], buf.view(a.num_blocks, a.block_size).cpu())
        gbs = lambda us: payload / (us * 1e-6) / 1e9  # noqa: E731
        row = {"path": "h2d", "op": op, "mode": a.h2d_mode, "blocks": a.num_blocks, "block_size": a.block_size,
               "bytes": payload, "iters": a.iterations, "avg_us": round(statistics.mean(lat), 2),
               "p50_us": round(_pct(lat, 0.5), 2), "p99_us": round(_pct(lat, 0.99), 2),
               "avg_gbs": round(gbs(statistics.mean(lat)), 3), "p50_gbs": round(gbs(_pct(lat, 0.5)), 3),
               "p99_gbs": round(gbs(_pct(lat, 0.99)), 3), "peak_gbs": round(gbs(min(lat)), 3), "verified": ok}
        if a.cuda_copy_baseline:
            src = pool[:payload] if op == "gather" else buf
            dst = buf if op == "gather" else pool[:payload]
            for _ in range(max(a.warmup, 1)):
                dst.copy_(src, non_blocking=True)
            ce = []
            for _ in range(a.iterations):
                with torch.cuda.stream(stream):
                    torch.cuda._sleep(40000)
                    e0.record(stream)
                    dst.copy_(src, non_blocking=True)
                    e1.record(stream)
                e1.synchronize()
                ce.append(e0.elapsed_time(e1) * 1e3)
            row["copy_engine_avg_gbs"] = round(gbs(statistics.mean(ce)), 3)
            row["copy_engine_peak_gbs"] = round(gbs(min(ce)), 3)
        rows.append(row)
        comm.unmap_dram_from_gpu(pool.data_ptr())
    return rows


def run_nic2gpu(comm, a):
    sizes = [parse_size(x) for x in a.sizes.split(",") if x.strip()]
    big = max(sizes)
    dev = "cuda" if a.dest == "gpu" else "cpu"
    local = torch.empty(big, dtype=torch.uint8, device=dev, pin_memory=(dev == "cpu"))
    assert comm.register_memory(local.data_ptr(), big) == 0
    if a.target:
        hid, ip, port = a.target.split(":")
        port = int(port)
    else:
        pool = torch.empty(big, dtype=torch.uint8, pin_memory=True)
        assert comm.register_memory(pool.data_ptr(), big) == 0 and comm.publish_buffer(pool.data_ptr(), big) == 0
        assert comm.start_accept_thread() == 0
        hid, ip, port = "pool", "127.0.0.1", comm.get_tcp_port()
    assert comm.connect(hid, ip, port) == 0, f"connect {hid}@{ip}:{port} failed"
    bufs = comm.query_remote_buffers(hid, ip, port)["buffers"]
    remote = max(bufs, key=lambda b: b["length"])
    ops = ["get", "put"] if a.op == "both" else ["get" if a.op in ("get", "gather") else "put"]
    rows = []
    for op in ops:
        for size in sizes:
            if size > remote["length"]:
                print(f"[nic2gpu] skip {size} B: remote buffer is {remote['length']} B", flush=True)
                continue
            fn = comm.get_async if op == "get" else comm.put_async

            def one():
                h = fn(local.data_ptr(), hid, remote["addr"], size)
                assert h and comm.wait_transfer(h, 120000) == 0, f"{op} of {size} B failed"
                comm.release_transfer(h)

            for _ in range(a.warmup):
                one()
            t = []
            for _ in range(a.iterations):
                t0 = time.perf_counter()
                one()
                t.append(time.perf_counter() - t0)
            rows.append({"path": "nic2gpu", "op": op, "dest": a.dest, "size": size, "iters": a.iterations,
                         "avg_us": round(statistics.mean(t) * 1e6, 2), "p50_us": round(_pct(t, 0.5) * 1e6, 2),
                         "avg_gbs": round(size / statistics.mean(t) / 1e9, 3),
                         "peak_gbs": round(size / min(t) / 1e9, 3)})
            print(f"[NIC-LIVE] op={op} size={size} avg {rows[-1]['avg_gbs']:.2f} GB/s", flush=True)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--path", required=True, choices=("h2d", "nic2gpu"))
    ap.add_argument("--gpu", type=int, default=0)
    ap.add_argument("--op", default="both")
    ap.add_argument("--iterations", "--iters", dest="iterations", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--single", action="store_true", help="one cold call: warmup 0, iterations 1")
    ap.add_argument("--report-every", type=int, default=0)
    ap.add_argument("--csv", default="")
    ap.add_argument("--h2d-mode", choices=tuple(MODES), default="tma")
    ap.add_argument("--num-blocks", type=int, default=2048)
    ap.add_argument("--block-size", type=int, default=272)
    ap.add_argument("--pool-multiplier", type=int, default=4)
    ap.add_argument("--max-sm-count", type=int, default=0)
    ap.add_argument("--cuda-copy-baseline", action="store_true")
    ap.add_argument("--sizes", default="512K,1M,4M,16M,64M,256M,1G")
    ap.add_argument("--target", default="", help="host_id:ip:port of a running target (default: own pinned pool)")
    ap.add_argument("--host-id", default="initiator:0")
    ap.add_argument("--device", default="")
    ap.add_argument("--dest", choices=("gpu", "cpu"), default="gpu")
    a = ap.parse_args(argv)
    if a.single:
        a.warmup, a.iterations = 0, 1
    if a.iterations <= 0 or a.warmup < 0 or a.report_every < 0:
        ap.error("iterations > 0, warmup >= 0, report-every >= 0")
    torch.cuda.set_device(a.gpu)
    comm = mpcomm.MPComm()
    assert comm.init(a.host_id, a.device) == 0
    try:
        rows = run_h2d(comm, a) if a.path == "h2d" else run_nic2gpu(comm, a)
    finally:
        comm.shutdown()
    keys = list(dict.fromkeys(k for r in rows for k in r))
    print(" | ".join(keys))
    for r in rows:
        print(" | ".join(str(r.get(k, "")) for k in keys))
    if a.csv:
        with open(a.csv, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=keys)
            w.writeheader()
            w.writerows(rows)
    print(json.dumps({"bench": f"h2d_nic2gpu/{a.path}", "rows": rows}), flush=True)


if __name__ == "__main__":
    main()
