"""Paged KV-cache H2D gather / D2H scatter benchmark (single GPU).

Workload: Llama-3-8B KV pool (64 KiB pages, bf16 ~ N(0,1)) of 65,536 pinned
host pages (4 GiB); gather 4,096 page indices drawn uniformly without
replacement (seed 1) into contiguous HBM through ``MPComm.tma_gather``, then
scatter them back with ``tma_scatter``; bit-exact check. Timed with CUDA
events on the launching stream after warm-up; the pool (4 GiB) exceeds L2.
Roofline: copy-engine cudaMemcpyAsync of the same byte count between the
pinned pool and HBM (contiguous, the best case for PCIe).

    python -m mpcomm.bench.h2d [--pages 65536] [--gather 4096] [--iters 10]
                               [--modes 0,1,2] [--max-sm 0]
Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json

import torch

import mpcomm
from mpcomm.models import LLAMA3_8B_KV


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--pages", type=int, default=65536)
    p.add_argument("--gather", type=int, default=4096)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--modes", default="0,1,2")
    p.add_argument("--max-sm", type=int, default=0)
    a = p.parse_args(argv)

    spec = LLAMA3_8B_KV
    bs = spec.page_bytes
    pool = spec.make_pool(a.pages, seed=0)
    idx_cpu = spec.sample_pages(a.pages, a.gather, seed=1)
    idx = idx_cpu.cuda()
    out = torch.empty((a.gather, bs), dtype=torch.uint8, device="cuda")
    comm = mpcomm.MPComm()
    dram = comm.map_dram_to_gpu(pool.data_ptr(), pool.numel())
    assert dram, "map_dram_to_gpu failed"
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    nbytes = a.gather * bs
    ref = pool[idx_cpu]
    res = {"metric": "paged KV H2D gather / D2H scatter GB/s", "page_bytes": bs, "pages": a.pages,
           "gather": a.gather, "bytes": nbytes, "modes": {}}

    # copy-engine roofline (contiguous)
    src_c = pool[: a.gather].reshape(-1)
    dst_c = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        dst_c.copy_(src_c, non_blocking=True)
    e0.record(stream)
    for _ in range(a.iters):
        dst_c.copy_(src_c, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ce_h2d = nbytes * a.iters / (e0.elapsed_time(e1) * 1e-3) / 1e9
    e0.record(stream)
    for _ in range(a.iters):
        src_c.copy_(dst_c, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ce_d2h = nbytes * a.iters / (e0.elapsed_time(e1) * 1e-3) / 1e9
    res["ce_h2d_gbs"], res["ce_d2h_gbs"] = round(ce_h2d, 3), round(ce_d2h, 3)

    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    for mode in [int(m) for m in a.modes.split(",")]:
        out.zero_()
        for _ in range(a.warmup):
            assert comm.tma_gather(dram, idx.data_ptr(), out.data_ptr(), a.gather, bs, a.max_sm, mode, sptr) == 0
        torch.cuda.synchronize()
        ok_g = torch.equal(out.cpu(), ref)
        e0.record(stream)
        for _ in range(a.iters):
            comm.tma_gather(dram, idx.data_ptr(), out.data_ptr(), a.gather, bs, a.max_sm, mode, sptr)
        e1.record(stream)
        torch.cuda.synchronize()
        g_ms = e0.elapsed_time(e1) / a.iters
        # scatter back (same bytes -> pool unchanged), then verify the pool pages
        for _ in range(a.warmup):
            assert comm.tma_scatter(out.data_ptr(), idx.data_ptr(), dram, a.gather, bs, a.max_sm, mode, sptr) == 0
        e0.record(stream)
        for _ in range(a.iters):
            comm.tma_scatter(out.data_ptr(), idx.data_ptr(), dram, a.gather, bs, a.max_sm, mode, sptr)
        e1.record(stream)
        torch.cuda.synchronize()
        s_ms = e0.elapsed_time(e1) / a.iters
        ok_s = torch.equal(pool[idx_cpu], ref)
        g_gbs, s_gbs = nbytes / (g_ms * 1e-3) / 1e9, nbytes / (s_ms * 1e-3) / 1e9
        res["modes"][{0: "auto", 1: "sm", 2: "tma"}[mode]] = {
            "gather_ms": round(g_ms, 4), "gather_gbs": round(g_gbs, 3), "gather_frac_ce": round(g_gbs / ce_h2d, 4),
            "scatter_ms": round(s_ms, 4), "scatter_gbs": round(s_gbs, 3),
            "scatter_frac_ce": round(s_gbs / ce_d2h, 4), "bitexact": bool(ok_g and ok_s)}
    res["gpu_launches"] = int(mpcomm.MPComm.get_kernel_launch_count() - launches0)
    comm.unmap_dram_from_gpu(pool.data_ptr())
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
