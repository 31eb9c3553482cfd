"""Zero-copy PUT/GET block-size sweep (the reference's scatter_test sweep,
user_examples/scatter_test.cpp:864-1187, README chart 512 KB -> 1 GB).

Each rank owns one GPU and one MPComm per QP setting (MPCOMM_QPS_PER_CONNECTION
is read at construction). Pools:
  --pool dram  the rank's own pinned host-DRAM pool (PCIe), connect-to-self
  --pool peer  the HBM of rank r^1, over NVLink through CUDA IPC (needs an
               even world size; with one GPU the "peer" is a second buffer on
               the same GPU)
For every (qps, block) the step is `batch` concurrent PUTs, wait, `batch`
concurrent GETs, wait; PUT and GET are timed separately with CUDA events on
the fabric stream, max over ranks, summed over ranks (weak scaling).
Payload uint8 uniform (seed 2). Prints one JSON line.

    torchrun --nproc-per-node N -m mpcomm.bench.putget --pool peer
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

import mpcomm
from mpcomm import parallel


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--pool", choices=["dram", "peer"], default="dram")
    p.add_argument("--min-kb", type=int, default=512)
    p.add_argument("--max-mb", type=int, default=1024)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--qps", default="1,2,4")
    p.add_argument("--budget-mb", type=int, default=8192, help="bytes per measurement (per direction)")
    a = p.parse_args(argv)
    rank, world, local = parallel.init_from_env("nccl")
    dev = torch.device("cuda", local)
    maxb = a.max_mb << 20
    total = maxb * a.batch
    g = torch.Generator(device=dev).manual_seed(2 + rank)
    src = torch.randint(0, 256, (total,), dtype=torch.uint8, device=dev, generator=g)
    dst = torch.empty(total, dtype=torch.uint8, device=dev)
    if a.pool == "dram":
        pool = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    else:
        pool = torch.empty(total, dtype=torch.uint8, device=dev)
    peer = rank ^ 1 if (a.pool == "peer" and world > 1) else rank
    fstream = torch.cuda.Stream(device=dev)
    sizes = []
    s = a.min_kb << 10
    while s <= maxb:
        sizes.append(s)
        s *= 2
    results = []
    for qps in [int(x) for x in a.qps.split(",")]:
        os.environ["MPCOMM_QPS_PER_CONNECTION"] = str(qps)
        comm = mpcomm.MPComm()
        assert comm.init(f"r{rank}q{qps}") == 0
        assert comm.start_accept_thread() == 0
        for t in (src, dst, pool):
            assert comm.register_memory(t.data_ptr(), t.numel()) == 0
        assert comm.publish_buffer(pool.data_ptr(), total) == 0
        ports = [comm.get_tcp_port()]
        if world > 1:
            ports = [None] * world
            dist.all_gather_object(ports, comm.get_tcp_port())
            dist.barrier()
        port = ports[peer] if world > 1 else ports[0]
        assert comm.connect("pool", "127.0.0.1", port) == 0
        info = comm.query_remote_buffers("pool", "127.0.0.1", port)
        raddr = info["buffers"][0]["addr"]
        comm.set_fabric_stream(fstream.cuda_stream)

        def phase(put: bool, bs: int):
            hs = []
            for i in range(a.batch):
                if put:
                    h = comm.put_async(src.data_ptr() + i * bs, "pool", raddr + i * bs, bs)
                else:
                    h = comm.get_async(dst.data_ptr() + i * bs, "pool", raddr + i * bs, bs)
                assert h
                hs.append(h)
            for h in hs:
                assert comm.wait_transfer(h, 120000) == 0
                comm.release_transfer(h)

        for bs in sizes:
            iters = max(3, min(50, (a.budget_mb << 20) // (bs * a.batch)))
            row = {"qps": qps, "block": bs}
            for put in (True, False):
                phase(put, bs)  # warm-up
                if world > 1:
                    dist.barrier()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(fstream)
                for _ in range(iters):
                    phase(put, bs)
                e1.record(fstream)
                torch.cuda.synchronize()
                ms = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64, device=dev)
                if world > 1:
                    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
                gbs = world * a.batch * bs / (ms.item() * 1e-3) / 1e9
                row["put_gbs" if put else "get_gbs"] = round(gbs, 3)
            results.append(row)
        if world > 1:
            dist.barrier()
        comm.shutdown()
    torch.cuda.synchronize()
    ok = torch.equal(dst[: a.batch * sizes[-1]], src[: a.batch * sizes[-1]])
    if rank == 0:
        print(json.dumps({"metric": "zero-copy PUT/GET GB/s sweep", "pool": a.pool, "n_gpus": world,
                          "batch": a.batch, "verified_last_get": bool(ok), "rows": results}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
