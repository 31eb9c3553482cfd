"""NVLink peer-copy microbenchmark, one process driving two GPUs.

The kernel runs on GPU 0 and either writes into GPU 1's HBM (PUT direction)
or reads from it (GET direction), with the bulk (TMA) pipeline or the vector
SM kernel, over a range of grid sizes; the copy engine (torch peer copy)
is the reference. 256 MiB per copy, CUDA events, 10 iterations. "bidir":
both GPUs copy at once (the GPU-pair exchange pattern), copy engine vs the
bulk kernel.

    python -m mpcomm.bench.peer        (needs >= 2 visible GPUs)
"""
from __future__ import annotations

import json

import torch

from mpcomm import _native, ops


def main():
    assert torch.cuda.device_count() >= 2, "needs two GPUs"
    n = 256 << 20
    a = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda:0")
    b = torch.zeros(n, dtype=torch.uint8, device="cuda:1")
    assert _native.enable_peer_access(0, 1) == 0 and _native.enable_peer_access(1, 0) == 0
    torch.cuda.set_device(0)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def t(fn, iters=10):
        fn()
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        e0.record(s)
        for _ in range(iters):
            fn()
        e1.record(s)
        torch.cuda.synchronize(0)
        return round(n / (e0.elapsed_time(e1) / iters * 1e-3) / 1e9, 2)

    q = n // 4
    res = {"bytes": n, "ce_put_gbs": t(lambda: b.copy_(a, non_blocking=True)),
           "ce_get_gbs": t(lambda: a.copy_(b, non_blocking=True)), "rows": []}
    for mode in (ops.MODE_TMA, ops.MODE_SM):
        for ctas in (37, 74, 148, 296):
            if mode == ops.MODE_TMA and ctas > 148:
                continue
            put = t(lambda: ops.copy_spans([a.data_ptr() + i * q for i in range(4)],
                                           [b.data_ptr() + i * q for i in range(4)], [q] * 4, ctas, mode=mode))
            get = t(lambda: ops.copy_spans([b.data_ptr() + i * q for i in range(4)],
                                           [a.data_ptr() + i * q for i in range(4)], [q] * 4, ctas, mode=mode))
            res["rows"].append({"path": "bulk" if mode == ops.MODE_TMA else "vector", "ctas": ctas,
                                "put_gbs": put, "get_gbs": get})
    torch.cuda.synchronize()
    res["verified"] = bool(torch.equal(a.cpu(), b.cpu()))
    res["bidir"] = bidirectional(n)
    print(json.dumps(res), flush=True)


def bidirectional(n: int, iters: int = 10) -> dict:
    """Both GPUs copy at once, each in the same direction relative to itself
    (both pull = GET, both push = PUT): the pattern of a GPU-pair exchange,
    where every link direction carries one GPU's data and the other's
    requests. Per-GPU GB/s of the slower GPU, copy engine vs the bulk and
    vector kernels at several grid sizes per GPU."""
    x = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=f"cuda:{d}") for d in (0, 1)]
    y = [torch.zeros(n, dtype=torch.uint8, device=f"cuda:{d}") for d in (0, 1)]
    streams = [torch.cuda.Stream(device=d) for d in (0, 1)]
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in (0, 1)]
    q = n // 4

    def issue(d, get, engine):
        peer = 1 - d
        src = x[peer] if get else x[d]   # GET: pull the peer's bytes here; PUT: push ours there
        dst = y[d] if get else y[peer]
        with torch.cuda.device(d), torch.cuda.stream(streams[d]):
            if engine == "ce":  # on this GPU's stream (torch would copy on the source's)
                assert _native.copy_engine_async(dst.data_ptr(), src.data_ptr(), n, streams[d].cuda_stream) == 0
            else:
                path, ctas = engine.split("_")
                ops.copy_spans([src.data_ptr() + i * q for i in range(4)], [dst.data_ptr() + i * q for i in range(4)],
                               [q] * 4, int(ctas), mode=ops.MODE_TMA if path == "bulk" else ops.MODE_SM)

    def run(get, engine):
        for d in (0, 1):
            issue(d, get, engine)
        for d in (0, 1):
            torch.cuda.synchronize(d)
        for d in (0, 1):
            ev[d][0].record(streams[d])
        for _ in range(iters):
            for d in (0, 1):
                issue(d, get, engine)
        for d in (0, 1):
            ev[d][1].record(streams[d])
        for d in (0, 1):
            torch.cuda.synchronize(d)
        ms = max(ev[d][0].elapsed_time(ev[d][1]) for d in (0, 1)) / iters
        return round(n / (ms * 1e-3) / 1e9, 2)

    out = {}
    for get in (True, False):
        for engine in ("ce", "bulk_74", "bulk_148", "vector_148", "vector_296", "vector_592"):
            out[f"{engine}_{'get' if get else 'put'}_gbs_per_gpu"] = run(get, engine)
    out["verified"] = bool(torch.equal(y[0].cpu(), x[1].cpu()) and torch.equal(y[1].cpu(), x[0].cpu()))
    return out


if __name__ == "__main__":
    main()
