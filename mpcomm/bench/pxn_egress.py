"""PXN egress/ingress: one GPU's PUT/GET to the host-DRAM pool, striped over
every GPU's PCIe link (MPCOMM_PXN_ENABLE=1) versus only its own.

One process, all visible GPUs. The buffers live on GPU 0 (HBM) and in pinned
host memory (pool); with PXN the GPU fabric opens a rail per GPU and each
peer GPU moves its share of the chunks: it reads GPU 0's HBM over NVLink and
writes the pool over its own PCIe link (PUT), or the reverse (GET). Blocks
of 1 GiB, batch 4 (the headline shape). Because the kernels of one transfer
run on several GPUs, each phase is timed on the host from submission to
completion (every kernel's completion event observed), after warm-up.

    python -m mpcomm.bench.pxn_egress      (needs >= 2 visible GPUs)
"""
from __future__ import annotations

import json
import os
import time

import torch

import mpcomm


def run(pxn: bool, src, dst, pool, block, batch, iters):
    os.environ["MPCOMM_PXN_ENABLE"] = "1" if pxn else "0"
    c = mpcomm.MPComm()
    assert c.init("pxn" if pxn else "direct") == 0 and c.start_accept_thread() == 0
    total = block * batch
    for t in (src, dst, pool):
        assert c.register_memory(t.data_ptr(), total) == 0
    assert c.publish_buffer(pool.data_ptr(), total) == 0
    port = c.get_tcp_port()
    assert c.connect("pool", "127.0.0.1", port) == 0 and c.query_remote_buffers("pool", "127.0.0.1", port)
    rails = c.get_active_devices()

    def phase(put):
        hs = [(c.put_async if put else c.get_async)((src if put else dst).data_ptr() + i * block, "pool",
                                                    pool.data_ptr() + i * block, block) for i in range(batch)]
        for h in hs:
            assert c.wait_transfer(h, 120000) == 0
            c.release_transfer(h)

    out = {"rails": rails}
    for put in (True, False):
        phase(put)
        t0 = time.perf_counter()
        for _ in range(iters):
            phase(put)
        dt = (time.perf_counter() - t0) / iters
        out["put_gbs" if put else "get_gbs"] = round(total / dt / 1e9, 3)
    c.shutdown()
    return out


def main():
    n = torch.cuda.device_count()
    assert n >= 2, "needs >= 2 GPUs"
    torch.cuda.set_device(0)
    block, batch, iters = 1 << 30, 4, 3
    total = block * batch
    src = torch.randint(0, 256, (total,), dtype=torch.uint8, device="cuda:0")
    dst = torch.empty(total, dtype=torch.uint8, device="cuda:0")
    pool = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    res = {"metric": "single-GPU PUT/GET to host pool, own link vs PXN over all GPUs", "gpus_visible": n,
           "block": block, "batch": batch, "timing": "host wall clock per phase (multi-device kernels)"}
    res["direct"] = run(False, src, dst, pool, block, batch, iters)
    res["pxn"] = run(True, src, dst, pool, block, batch, iters)
    torch.cuda.synchronize()
    res["verified"] = bool(torch.equal(dst, src))
    res["speedup_put"] = round(res["pxn"]["put_gbs"] / res["direct"]["put_gbs"], 3)
    res["speedup_get"] = round(res["pxn"]["get_gbs"] / res["direct"]["get_gbs"], 3)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
