"""NVLink peer-copy microbenchmark, one process driving two GPUs.

The kernel runs on GPU 0 and either writes into GPU 1's HBM (PUT direction)
or reads from it (GET direction), with the bulk (TMA) pipeline or the vector
SM kernel, over a range of grid sizes; the copy engine (torch peer copy)
is the reference. 256 MiB per copy, CUDA events, 10 iterations.

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
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
