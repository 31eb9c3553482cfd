"""This library's H2D movers against the reference's own kernels, same box.

The reference's tmaGather / tmaScatter kernels (src/mpcomm_tma_kernels.cu,
launchers :319-463) depend only on CUDA, so they build on their own. This
bench compiles that file UNMODIFIED, with the reference's own architecture
pin (compute_90: sm_90 code plus PTX, which the driver JIT-compiles for the
B200), into baseline/_ref/libref_tma.so (outside the product), and calls
its launch_tma_gather_kernel / launch_tma_scatter_kernel through ctypes.

Workloads (one GPU, pinned host pool, seeded indices, bit-exact checks of
both implementations against torch indexing):
  kv64k   4,096 x 64 KiB Llama-3-8B KV pages of a 65,536-page pool (seed 1):
          the reference in SM mode (its TMA mode cannot launch at 64 KiB:
          128 x (64 KiB + 8) B of shared memory per CTA, :371)
  b272    2,048 x 272 B blocks (the reference tool's default,
          user_examples/qos_bench/run-bench-h2d.sh:13-17), reference TMA mode
  b1k     10,240 x 1 KiB blocks (its QoS bench's gather), reference TMA mode
Ours: MPComm.tma_gather / tma_scatter (AUTO mode unless --ours-mode) on the
same stream.

Timing: per launch, CUDA events on the legacy default stream (where the
reference launches), the start event queued behind a short device sleep so
host launch time (the reference prints a line per launch) is excluded;
median of --iters launches after --warmup.

    python -m mpcomm.bench.h2d_vs_reference [--iters 20] [--warmup 3]
Prints one JSON line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import subprocess
import sys

import torch

import mpcomm
from mpcomm.models import LLAMA3_8B_KV

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_SRC = os.path.join(REF_DIR, "src_tree", "src", "mpcomm_tma_kernels.cu")
REF_LIB = os.path.join(REF_DIR, "libref_tma.so")
# Itanium-mangled names of mpcomm::launch_tma_{gather,scatter}_kernel(
#     const char*, const int64_t*, char*, int, int, int, int).
GATHER_SYM = "_ZN6mpcomm24launch_tma_gather_kernelEPKcPKlPciiii"
SCATTER_SYM = "_ZN6mpcomm25launch_tma_scatter_kernelEPKcPKlPciiii"
REF_SM, REF_TMA = 1, 2


def build_reference() -> str:
    """Compiles the reference kernel file as shipped; returns the library path."""
    if os.path.isfile(REF_LIB) and (not os.path.isfile(REF_SRC) or
                                    os.path.getmtime(REF_LIB) >= os.path.getmtime(REF_SRC)):
        return REF_LIB
    if not os.path.isfile(REF_SRC):
        raise FileNotFoundError("reference source tree not found under baseline/_ref/src_tree")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-gencode", "arch=compute_90,code=sm_90", "-gencode", "arch=compute_90,code=compute_90",
           REF_SRC, "-o", REF_LIB]
    subprocess.run(cmd, check=True)
    return REF_LIB


class RefKernels:
    def __init__(self, path: str):
        self.lib = ctypes.CDLL(path)
        args = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                ctypes.c_int]
        self.gather = getattr(self.lib, GATHER_SYM)
        self.scatter = getattr(self.lib, SCATTER_SYM)
        for f in (self.gather, self.scatter):
            f.argtypes = args
            f.restype = None


def _device_ms(launch, iters: int, warmup: int) -> float:
    stream = torch.cuda.default_stream()
    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    times = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(iters):
        torch.cuda._sleep(200_000)  # the GPU is busy while the launch is queued
        e0.record(stream)
        launch()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    return times[len(times) // 2]


def run_case(name, comm, ref, pool_blocks, n, bs, ref_mode, seed, iters, warmup, kv=False, ours_mode=0):
    if kv:
        pool = LLAMA3_8B_KV.make_pool(pool_blocks, seed=0)
        idx_cpu = LLAMA3_8B_KV.sample_pages(pool_blocks, n, seed=seed)
    else:
        g = torch.Generator().manual_seed(seed)
        pool = torch.randint(0, 256, (pool_blocks, bs), dtype=torch.uint8, generator=g).pin_memory()
        idx_cpu = torch.randperm(pool_blocks, generator=g)[:n].to(torch.int64)
    dram = comm.map_dram_to_gpu(pool.data_ptr(), pool.numel())
    assert dram, "map_dram_to_gpu failed"
    idx = idx_cpu.cuda()
    expect = pool[idx_cpu].reshape(-1).clone()
    out = torch.empty(n * bs, dtype=torch.uint8, device="cuda")
    nbytes = n * bs
    row = {"blocks": n, "block_bytes": bs, "pool_blocks": pool_blocks,
           "reference_mode": {REF_SM: "sm", REF_TMA: "tma"}[ref_mode]}

    def ours_gather():
        assert comm.tma_gather(dram, idx.data_ptr(), out.data_ptr(), n, bs, 0, ours_mode, 0) == 0

    def ours_scatter():
        assert comm.tma_scatter(out.data_ptr(), idx.data_ptr(), dram, n, bs, 0, ours_mode, 0) == 0

    def ref_gather():
        ref.gather(dram, idx.data_ptr(), out.data_ptr(), bs, n, 0, ref_mode)

    def ref_scatter():
        ref.scatter(out.data_ptr(), idx.data_ptr(), dram, bs, n, 0, ref_mode)

    for impl, g_fn, s_fn in (("ours", ours_gather, ours_scatter), ("reference", ref_gather, ref_scatter)):
        out.zero_()
        torch.cuda.synchronize()
        g_ms = _device_ms(g_fn, iters, warmup)
        ok_g = torch.equal(out.cpu(), expect)
        # Scatter writes the same bytes back: the pool must be unchanged.
        s_ms = _device_ms(s_fn, iters, warmup)
        ok_s = torch.equal(pool[idx_cpu].reshape(-1), expect)
        row[impl] = {"gather_us": round(g_ms * 1e3, 2), "gather_gbs": round(nbytes / (g_ms * 1e-3) / 1e9, 3),
                     "scatter_us": round(s_ms * 1e3, 2), "scatter_gbs": round(nbytes / (s_ms * 1e-3) / 1e9, 3),
                     "bitexact": bool(ok_g and ok_s)}
    row["gather_speedup"] = round(row["reference"]["gather_us"] / row["ours"]["gather_us"], 3)
    row["scatter_speedup"] = round(row["reference"]["scatter_us"] / row["ours"]["scatter_us"], 3)
    comm.unmap_dram_from_gpu(pool.data_ptr())
    del pool
    return name, row


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cases", default="kv64k,b272,b1k")
    ap.add_argument("--ours-mode", choices=["auto", "sm", "tma"], default="auto",
                    help="this library's H2D mode (the reference's is fixed per case)")
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    ref = RefKernels(build_reference())
    comm = mpcomm.MPComm()
    res = {"metric": "H2D gather / D2H scatter: this library vs the reference's own kernels (same GPU, same data)",
           "device": torch.cuda.get_device_name(0),
           "reference_build": "src/mpcomm_tma_kernels.cu unmodified, nvcc -gencode compute_90 (sm_90 + PTX, "
                              "JIT-compiled for sm_100 by the driver)",
           "timing": "median per-launch CUDA-event time, host launch excluded", "ours_mode": a.ours_mode,
           "cases": {}}
    specs = {
        "kv64k": dict(pool_blocks=65536, n=4096, bs=LLAMA3_8B_KV.page_bytes, ref_mode=REF_SM, seed=1, kv=True),
        "b272": dict(pool_blocks=8192, n=2048, bs=272, ref_mode=REF_TMA, seed=5),
        "b1k": dict(pool_blocks=40960, n=10240, bs=1024, ref_mode=REF_TMA, seed=6),
    }
    for c in a.cases.split(","):
        name, row = run_case(c, comm, ref, iters=a.iters, warmup=a.warmup,
                             ours_mode={"auto": 0, "sm": 1, "tma": 2}[a.ours_mode], **specs[c])
        res["cases"][name] = row
    # The reference prints a line per launch through C stdio: flush it first
    # so the JSON line is the last one.
    ctypes.CDLL(None).fflush(None)
    sys.stdout.flush()
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
