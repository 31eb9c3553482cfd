"""Small-transfer latency: PUT/GET round trips through the public API.

Measures wall-clock time from put_async/get_async to the return of
wait_transfer for small blocks, back to back and after an idle gap (when the
engine's worker and the caller have gone to sleep), and prints p50/p90/p99
per case as one JSON line. The target buffer is published by a second
MPComm in the same process (connect-to-self over the TCP control plane).

    python -m mpcomm.bench.latency [--fabric lo|sock|nvl] [--sizes 4K,64K,1M]
                                   [--gaps-ms 0,2] [--iters 300] [--device cuda]

--device cuda places the source in HBM and the target in pinned host
memory (the GPU fabric's HBM <-> DRAM-pool path); the default uses host
memory on both sides. On the GPU fabric the line also carries
"kernel_floor": the same copy kernel launched bare and timed to its
host-visible done word, i.e. what is left without the engine. The
reference publishes no latency numbers.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import time

from mpcomm.harness.common import parse_size


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--fabric", default=os.environ.get("MPCOMM_FABRIC", "lo"))
    ap.add_argument("--sizes", default="4K,64K,1M")
    ap.add_argument("--gaps-ms", default="0,2")
    ap.add_argument("--iters", type=int, default=300)
    ap.add_argument("--device", choices=["host", "cuda"], default="host")
    a = ap.parse_args(argv)
    os.environ["MPCOMM_FABRIC"] = a.fabric
    import mpcomm

    sizes = [parse_size(x) for x in a.sizes.split(",")]
    n = max(sizes)
    keep = []
    if a.device == "cuda":
        import torch

        src_t = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
        dst_t = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        keep += [src_t, dst_t]
        src, dst = src_t.data_ptr(), dst_t.data_ptr()
    else:
        s = ctypes.create_string_buffer(os.urandom(n), n)
        t = ctypes.create_string_buffer(n)
        keep += [s, t]
        src, dst = ctypes.addressof(s), ctypes.addressof(t)
    ini, tgt = mpcomm.MPComm(), mpcomm.MPComm()
    assert ini.init("lat-initiator") == 0 and tgt.init("lat-target") == 0
    assert tgt.start_accept_thread() == 0
    assert tgt.register_memory(dst, n) == 0 and tgt.publish_buffer(dst, n) == 0
    assert ini.register_memory(src, n) == 0
    port = tgt.get_tcp_port()
    assert ini.connect("T", "127.0.0.1", port) == 0 and ini.query_remote_buffers("T", "127.0.0.1", port)
    rows = []
    for size in sizes:
        for gap_ms in [float(x) for x in a.gaps_ms.split(",")]:
            for op in ("put", "get"):
                lat = []
                for i in range(a.iters + 10):
                    if gap_ms:
                        time.sleep(gap_ms * 1e-3)
                    t0 = time.perf_counter()
                    h = (ini.put_async(src, "T", dst, size) if op == "put" else ini.get_async(src, "T", dst, size))
                    rc = ini.wait_transfer(h, 10000)
                    dt = time.perf_counter() - t0
                    ini.release_transfer(h)
                    assert rc == 0, f"{op} failed rc={rc}"
                    if i >= 10:  # warm-up
                        lat.append(dt * 1e6)
                lat.sort()
                q = lambda f: round(lat[min(len(lat) - 1, int(f * len(lat)))], 1)
                rows.append({"op": op, "bytes": size, "gap_ms": gap_ms, "p50_us": q(0.5), "p90_us": q(0.9),
                             "p99_us": q(0.99)})
    floor = []
    if a.device == "cuda" and a.fabric == "nvl":
        # What the engine adds: the same copy kernel launched bare, timed to
        # its host-visible done word (no queue, worker, handle or Python).
        from mpcomm import _native
        for size in sizes:
            lat = sorted(_native.copy_roundtrip_us(src, dst, size, a.iters + 10)[10:])
            if lat:
                q = lambda f: round(lat[min(len(lat) - 1, int(f * len(lat)))], 1)
                floor.append({"op": "put (bare kernel round trip)", "bytes": size, "p50_us": q(0.5),
                              "p90_us": q(0.9), "p99_us": q(0.99)})
    ini.shutdown()
    tgt.shutdown()
    out = {"metric": "small-transfer latency (submit -> wait_transfer returns)", "fabric": a.fabric,
           "device": a.device, "iters": a.iters, "rows": rows}
    if floor:
        out["kernel_floor"] = floor
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
