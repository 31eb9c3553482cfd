"""Staging-pool (non-zero-copy) PUT/GET, CPU only.

Config 1: one process, host-DRAM -> host-DRAM PUT then GET of 64 blocks x
1 MiB over an in-process transport (``--fabric lo``, default) or the socket
fabric (``--fabric sock``), through the staging pool: the local buffers are
NOT registered, so every block is copied into / out of pre-registered slabs
by the copy threads while other slabs are on the wire. Payload uint8
uniform from seed 0; every block is verified by CRC-32 after the GET. The
same transfers from a registered buffer (zero-copy) run as the comparison.

    python -m mpcomm.bench.staging [--blocks 64] [--block-size 1M] [--iters 5]
                                   [--fabric lo|sock] [--rails 4] [--sweep]

--sweep adds the reference chart's block sweep (512 KiB -> 1 GiB, batch 4).
Wall-clock GB/s = bytes / seconds (as the reference's scatter_test).
Parity: reference README.md:105-116 (bcopy numbers; the reference ships no
staging code).
"""
from __future__ import annotations

import argparse
import json
import mmap
import os
import time
import zlib

import numpy as np

import mpcomm
from mpcomm.harness.common import parse_size


def _buf(n):
    mm = mmap.mmap(-1, max(n, 1), mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS, mmap.PROT_READ | mmap.PROT_WRITE)
    arr = np.frombuffer(mm, dtype=np.uint8, count=n)
    arr[::4096] = 0  # fault the pages in
    return mm, arr


def _run(comm, op, local_ptr, remote_ptr, nblocks, bs, batch):
    fn = comm.put_async if op == "put" else comm.get_async
    t0 = time.perf_counter()
    pending = []
    for i in range(nblocks):
        pending.append(fn(local_ptr + i * bs, "pool", remote_ptr + i * bs, bs))
        if len(pending) >= batch:
            h = pending.pop(0)
            assert h and comm.wait_transfer(h, 120000) == 0, f"{op} failed"
            comm.release_transfer(h)
    for h in pending:
        assert h and comm.wait_transfer(h, 120000) == 0, f"{op} failed"
        comm.release_transfer(h)
    return time.perf_counter() - t0


def measure(nblocks, bs, iters, batch, zero_copy, seed=0, warmup=1):
    n = nblocks * bs
    a, b = mpcomm.MPComm(), mpcomm.MPComm()
    assert a.init("initiator") == 0 and b.init("pool-host") == 0 and b.start_accept_thread() == 0
    try:
        pool_mm, pool = _buf(n)
        src_mm, src = _buf(n)
        back_mm, back = _buf(n)
        src[:] = np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)
        ptr = lambda arr: arr.ctypes.data  # noqa: E731
        assert b.register_memory(ptr(pool), n) == 0 and b.publish_buffer(ptr(pool), n) == 0
        port = b.get_tcp_port()
        assert a.connect("pool", "127.0.0.1", port) == 0 and a.query_remote_buffers("pool", "127.0.0.1", port)
        if zero_copy:
            assert a.register_memory(ptr(src), n) == 0 and a.register_memory(ptr(back), n) == 0
        for _ in range(warmup):
            _run(a, "put", ptr(src), ptr(pool), nblocks, bs, batch)
            _run(a, "get", ptr(back), ptr(pool), nblocks, bs, batch)
        tp = sum(_run(a, "put", ptr(src), ptr(pool), nblocks, bs, batch) for _ in range(iters))
        back[:] = 0
        tg = sum(_run(a, "get", ptr(back), ptr(pool), nblocks, bs, batch) for _ in range(iters))
        want = [zlib.crc32(src[i * bs:(i + 1) * bs]) for i in range(nblocks)]
        got = [mpcomm.ops.crc32_host(back[i * bs:(i + 1) * bs].tobytes()) for i in range(nblocks)]
        ok = want == got
        return {"blocks": nblocks, "block_bytes": bs, "batch": batch, "iters": iters,
                "put_gbs": round(n * iters / tp / 1e9, 3), "get_gbs": round(n * iters / tg / 1e9, 3),
                "crc32_verified": ok}
    finally:
        a.shutdown()
        b.shutdown()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--blocks", type=int, default=64)
    ap.add_argument("--block-size", default="1M")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--batch", type=int, default=64, help="transfers in flight (config 1 submits all 64)")
    ap.add_argument("--fabric", default="lo", choices=["lo", "sock"])
    ap.add_argument("--rails", type=int, default=4, help="loopback rails (one copy engine thread each; the "
                    "reference's numbers use 4 NICs)")
    ap.add_argument("--staging-threads", type=int, default=0, help="copy threads of the staging pool (0 = default)")
    ap.add_argument("--sweep", action="store_true")
    a = ap.parse_args(argv)
    os.environ["MPCOMM_FABRIC"] = a.fabric
    os.environ["MPCOMM_LOOPBACK_NICS"] = str(a.rails)
    if a.staging_threads:
        os.environ["MPCOMM_STAGING_THREADS"] = str(a.staging_threads)
    os.environ.setdefault("MPCOMM_LOG_LEVEL", "1")
    bs = parse_size(a.block_size)
    res = {"metric": "staging-pool PUT/GET GB/s (CPU, host DRAM -> host DRAM)", "fabric": a.fabric, "rails": a.rails,
           "cpus": len(os.sched_getaffinity(0)),
           "staging": measure(a.blocks, bs, a.iters, a.batch, zero_copy=False),
           "zero_copy": measure(a.blocks, bs, a.iters, a.batch, zero_copy=True)}
    if a.sweep:
        rows = []
        for size in [512 << 10, 1 << 20, 4 << 20, 16 << 20, 64 << 20, 256 << 20, 1 << 30]:
            # Enough rounds of 4 blocks to move ~1 GiB (at least --iters, at most 256).
            rounds = max(a.iters, min(256, (1 << 30) // (4 * size)))
            r = measure(4, size, rounds, 4, zero_copy=False, warmup=3)
            rows.append({"block": size, "put_gbs": r["put_gbs"], "get_gbs": r["get_gbs"], "ok": r["crc32_verified"]})
            print(json.dumps(rows[-1]), flush=True)
        res["sweep_batch4"] = rows
    print(json.dumps(res), flush=True)
    if not (res["staging"]["crc32_verified"] and res["zero_copy"]["crc32_verified"]):
        raise SystemExit("CRC-32 mismatch")


if __name__ == "__main__":
    main()
