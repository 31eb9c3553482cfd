"""Runs every mpcomm kernel once on a small case, for profiling and quick
per-kernel timing (single GPU, a few hundred MB at most).

    python -m mpcomm.bench.kernels [--cases all|gather_tma,...] [--time]

Cases (inputs larger than the 126 MB L2 where DRAM/PCIe traffic matters):
  gather_tma / gather_sm   1,024 x 64 KiB pages from a 2,048-page pinned pool
  gather_1k                10,240 x 1 KiB blocks from a 40,960-block pinned pool
                           (the packed small-block gather kernel)
  scatter_1k               the reverse (the packed small-block scatter kernel)
  scatter_tma              the reverse
  copy_d2d                 GPU-fabric WR batch, 4 x 40 MiB HBM -> HBM
  copy_h2d                 GPU-fabric WR batch, 2 x 32 MiB pinned DRAM -> HBM
  crc32 / crc32_noalloc    4 x 40 MiB blocks
  pxn_local                fused gather + forward (destination on this GPU)
  fanout_local             P2P fan-out store path to 2 local buffers
  gather_bcast_p2p         fused host gather + delivery (bulk stores) to 2
                           local buffers, 512 x 64 KiB pages
  nvls                     multimem broadcast through a 1-GPU multicast object
  wait_flag                bounded flag wait on a flag that is already set
With --time each case is also timed with CUDA events (after 2 warm-ups) and
its GB/s printed as one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os

import torch

import mpcomm
from mpcomm import ops

PAGE = 65536
ALL = ["gather_tma", "gather_sm", "gather_1k", "scatter_1k", "scatter_tma", "copy_d2d", "copy_h2d", "crc32", "crc32_noalloc",
       "pxn_local", "fanout_local", "gather_bcast_p2p", "nvls", "wait_flag"]


def build_cases():
    g = torch.Generator().manual_seed(0)
    pool = torch.randint(0, 256, (2048, PAGE), dtype=torch.uint8, generator=g).pin_memory()
    idx = torch.randperm(2048, generator=g)[:1024].cuda()
    out = torch.empty((1024, PAGE), dtype=torch.uint8, device="cuda")
    big = torch.randint(0, 256, (160 << 20,), dtype=torch.uint8, device="cuda")
    big2 = torch.empty_like(big)
    host = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, generator=g).pin_memory()
    crc_out = torch.empty(4, dtype=torch.int32, device="cuda")
    pool1k = torch.randint(0, 256, (40960, 1024), dtype=torch.uint8, generator=g).pin_memory()
    idx1k = torch.randperm(40960, generator=g)[:10240].cuda()
    out1k = torch.empty((10240, 1024), dtype=torch.uint8, device="cuda")
    flag = torch.ones(1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = ctypes.CDLL(mpcomm.native_library_path())
    noalloc = lib.mpcomm_crc32_blocks_noalloc
    noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    nb = 1024 * PAGE
    q = 40 << 20
    cases = {
        "gather_tma": (lambda: ops.paged_gather(pool, idx, out=out, mode=ops.MODE_TMA), nb),
        "gather_sm": (lambda: ops.paged_gather(pool, idx, out=out, mode=ops.MODE_SM), nb),
        "gather_1k": (lambda: ops.paged_gather(pool1k, idx1k, out=out1k), 10240 * 1024),
        "scatter_1k": (lambda: ops.paged_scatter(out1k, idx1k, pool1k), 10240 * 1024),
        "scatter_tma": (lambda: ops.paged_scatter(out, idx, pool, mode=ops.MODE_TMA), nb),
        "copy_d2d": (lambda: ops.copy_spans([big.data_ptr() + i * q for i in range(4)],
                                            [big2.data_ptr() + i * q for i in range(4)], [q] * 4), 4 * q),
        "copy_h2d": (lambda: ops.copy_spans([host.data_ptr(), host.data_ptr() + (32 << 20)],
                                            [big2.data_ptr(), big2.data_ptr() + (32 << 20)], [32 << 20] * 2), 64 << 20),
        "crc32": (lambda: ops.crc32_blocks(big, 4, out=crc_out), big.numel()),
        "crc32_noalloc": (lambda: noalloc(big.data_ptr(), 4, big.numel() // 4, crc_out.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream), big.numel()),
        "pxn_local": (lambda: ops.pxn_gather_forward(pool.data_ptr(), 2048, idx, out.data_ptr(), PAGE,
                                                     done_flag=flag.data_ptr(), flag_value=1,
                                                     counter=ctr.data_ptr()), nb),
        "fanout_local": (lambda: ops.p2p_fanout(big[:q], [big2.data_ptr(), big2.data_ptr() + q], q), 2 * q),
        "gather_bcast_p2p": (lambda: ops.gather_bcast(pool.data_ptr(), 2048, idx[:512], PAGE,
                                                      dst_ptrs=[out.data_ptr(), out.data_ptr() + 512 * PAGE]),
                             512 * PAGE),
        "wait_flag": (lambda: ops.wait_flag(flag.data_ptr(), 1, 1_000_000, status.data_ptr()), 8),
    }
    keep = (pool, idx, out, big, big2, host, crc_out, flag, status, ctr, pool1k, idx1k, out1k)
    return cases, keep


def nvls_case():
    import torch.distributed as dist

    from mpcomm import parallel

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29599")
        dist.init_process_group("gloo", rank=0, world_size=1)
    src = torch.randint(0, 256, (160 << 20,), dtype=torch.uint8, device="cuda")
    grp = parallel.NvlsGroup(src.numel())
    return (lambda: ops.nvls_broadcast(src, grp.mc_ptr, src.numel())), src.numel(), (grp, src)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", default="all")
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    names = ALL if a.cases == "all" else a.cases.split(",")
    cases, keep = build_cases()
    if "nvls" in names:
        try:
            fn, nbytes, grp = nvls_case()
            cases["nvls"] = (fn, nbytes)
            keep = keep + (grp,)
        except Exception as e:  # multicast unavailable on this box
            print(json.dumps({"case": "nvls", "skipped": str(e)}), flush=True)
    torch.cuda.synchronize()
    for name in names:
        if name not in cases:
            continue
        fn, nbytes = cases[name]
        fn()
        torch.cuda.synchronize()
        if a.time:
            fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.iters
            print(json.dumps({"case": name, "ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 2)}),
                  flush=True)
    if "nvls" in cases:
        keep[-1][0].close()
    print(json.dumps({"kernels_launched": mpcomm.MPComm.get_kernel_launch_count()}), flush=True)


if __name__ == "__main__":
    main()
