"""NVLink-forwarded (PXN) paged gather benchmark (one process per GPU).

A host-DRAM pool of Llama-3-8B KV pages (64 KiB, bf16 ~ N(0,1)) lives in
POSIX shared memory placed on one NUMA node (by default not the node of
rank 0's GPU when the host has more than one). Every rank requests 1,024
pages drawn uniformly without replacement (seed 3 + rank). A proxy GPU —
NUMA-local to the pool — gathers them and forwards them into the requester's
HBM with one fused kernel (cp.async.bulk loads from the host pool, bulk
stores into the peer's IPC-mapped HBM, last CTA publishes a done flag in the
requester's memory). The requester's stream waits on that flag with a
bounded device wait. Proxy of requester r: the r-th NUMA-local GPU round
robin, or (r+1)%N when every GPU is NUMA-local, so bytes always cross
NVLink.

Timing: CUDA events per rank around [forward launches for its requesters,
wait for its own flag]; max over ranks. Baselines in the same run:
  direct     each requester gathers its pages itself (tma path, own PCIe)
  two_step   reference-style PXN: proxy gathers into its own HBM, then a
             peer copy (cudaMemcpyPeerAsync) to the requester
Roofline: each proxy's forward is bounded by its PCIe H2D rate (measured
copy-engine rate of the same pool) since NVLink (770 GB/s) is faster.

    torchrun --nproc-per-node 8 -m mpcomm.bench.pxn
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

import mpcomm
from mpcomm import ops, parallel
from mpcomm.models import LLAMA3_8B_KV


def gpu_numa(dev: int) -> int:
    p = torch.cuda.get_device_properties(dev)
    bdf = "%04x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
    try:
        return int(open(f"/sys/bus/pci/devices/{bdf}/numa_node").read().strip())
    except (OSError, ValueError):
        return -1


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--pages", type=int, default=65536)
    ap.add_argument("--request", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    rank, world, local = parallel.init_from_env("nccl")
    dev = torch.device("cuda", local)
    bs = LLAMA3_8B_KV.page_bytes
    numas = [None] * world
    dist.all_gather_object(numas, gpu_numa(local))
    nodes = sorted({n for n in numas if n >= 0}) or [0]
    pool_node = nodes[(nodes.index(numas[0]) + 1) % len(nodes)] if numas[0] in nodes and len(nodes) > 1 else nodes[0]
    name = f"mpcomm-pxn-{os.environ.get('MASTER_PORT', '0')}"
    nbytes = a.pages * bs
    if rank == 0:
        pool = parallel.SharedHostPool(name, nbytes, create=True, numa_node=pool_node)
        src = LLAMA3_8B_KV.make_pool(min(a.pages, 4096), seed=0, pinned=False).reshape(-1)
        view = pool.tensor.view(a.pages, bs)
        for s in range(0, a.pages, 4096):
            e = min(a.pages, s + 4096)
            view[s:e].copy_(src.view(-1, bs)[: e - s])
    dist.barrier()
    if rank != 0:
        pool = parallel.SharedHostPool(name, nbytes, create=False)
    dist.barrier()

    local_proxies = [r for r in range(world) if numas[r] == pool_node]
    if not local_proxies or len(local_proxies) == world:
        proxy_of = [(r + 1) % world for r in range(world)]
    else:
        proxy_of = [local_proxies[r % len(local_proxies)] for r in range(world)]
    my_requesters = [r for r in range(world) if proxy_of[r] == rank]

    wants = [LLAMA3_8B_KV.sample_pages(a.pages, a.request, seed=3 + r) for r in range(world)]
    idx_for = {r: wants[r].to(dev) for r in my_requesters}
    my_idx = wants[rank].to(dev)
    dst = parallel.PeerBuffers(a.request * bs)
    flags = parallel.PeerBuffers(64)
    ctrs = torch.zeros(max(1, len(my_requesters)), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    budget = 2_000_000_000

    def pxn_step(seq: int):
        for k, r in enumerate(my_requesters):
            ops.pxn_gather_forward(pool.dev_ptr, a.pages, idx_for[r], dst.ptrs[r], bs,
                                   done_flag=flags.ptrs[r], flag_value=seq,
                                   counter=ctrs.data_ptr() + 4 * k, stream=stream)
        ops.wait_flag(flags.local.data_ptr(), seq, budget, status.data_ptr(), stream=stream)

    comm = mpcomm.MPComm()
    direct_out = torch.empty(a.request * bs, dtype=torch.uint8, device=dev)
    staging = torch.empty(a.request * bs, dtype=torch.uint8, device=dev)

    def direct_step(_seq: int):
        ops.paged_gather(pool.tensor.view(a.pages, bs), my_idx, out=direct_out.view(a.request, bs), stream=stream)

    peer_out = dst  # two-step writes into the same destination buffers

    def two_step(_seq: int):
        for r in my_requesters:
            ops.paged_gather(pool.tensor.view(a.pages, bs), idx_for[r], out=staging.view(a.request, bs),
                             stream=stream)
            with torch.cuda.stream(stream):
                parallel.device_view(peer_out.ptrs[r], a.request * bs).copy_(staging, non_blocking=True)

    def run(fn, seq0):
        for i in range(a.warmup):
            fn(seq0 + i)
        stream.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(a.iters):
            fn(seq0 + a.warmup + i)
        e1.record(stream)
        stream.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        return ms.item()

    launches0 = mpcomm.MPComm.get_kernel_launch_count()
    pxn_ms = run(pxn_step, 1)
    launches = mpcomm.MPComm.get_kernel_launch_count() - launches0
    ok = torch.equal(dst.local.view(a.request, bs).cpu(), pool.tensor.view(a.pages, bs)[wants[rank]])
    ok_t = torch.tensor([1 if ok and status.item() == 0 else 0], device=dev)
    dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
    direct_ms = run(direct_step, 0)
    two_ms = run(two_step, 0)
    # copy-engine H2D rate of the pool (per GPU, contiguous): the roofline
    ce = torch.empty(a.request * bs, dtype=torch.uint8, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    chunk = pool.tensor[: a.request * bs]
    ce.copy_(chunk, non_blocking=True)
    e0.record()
    for _ in range(5):
        ce.copy_(chunk, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ce_gbs = a.request * bs * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e9
    ce_t = torch.tensor([ce_gbs], dtype=torch.float64, device=dev)
    dist.all_reduce(ce_t, op=dist.ReduceOp.MIN)
    total = world * a.request * bs
    busy_proxies = len(set(proxy_of))
    roof_gbs = busy_proxies * ce_t.item()
    if rank == 0:
        gbs = total / (pxn_ms * 1e-3) / 1e9
        print(json.dumps({
            "metric": "PXN fused gather+forward GB/s (aggregate)", "n_gpus": world, "page_bytes": bs,
            "pages_per_rank": a.request, "pool_pages": a.pages, "pool_numa": pool_node, "gpu_numa": numas,
            "proxy_of": proxy_of, "pxn_ms": round(pxn_ms, 4), "pxn_gbs": round(gbs, 3),
            "direct_ms": round(direct_ms, 4), "direct_gbs": round(total / (direct_ms * 1e-3) / 1e9, 3),
            "two_step_ms": round(two_ms, 4), "two_step_gbs": round(total / (two_ms * 1e-3) / 1e9, 3),
            "roofline_gbs": round(roof_gbs, 3), "roofline_what": f"{busy_proxies} proxies x copy-engine H2D",
            "frac_of_roofline": round(gbs / roof_gbs, 4), "bitexact": bool(ok_t.item()),
            "gpu_launches": int(launches)}), flush=True)
    dist.barrier()
    dst.close()
    flags.close()
    pool.close(unlink=(rank == 0))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
