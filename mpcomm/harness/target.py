"""Target server: allocates, registers and publishes one buffer per NUMA
node (host DRAM) or one HBM buffer (--gpu), seeds the first MiB of each with
the IPv4 pattern of its host id, and serves buffer queries and one-sided
traffic until SIGINT/SIGTERM (or --duration seconds).

    python -m mpcomm.harness.target --host-id 10.0.0.2:5000 --tcp-port 5000 \\
        --buffer-size 10G [--num-numas 0,1 | --gpu 0] [--ready-file PATH]

Prints one line "[target] ready host=<id> port=<p> buffers=<n>" when it
accepts connections (orchestration waits for it). Behavioural parity:
reference user_examples/mpcomm_target.py (single and multi-NUMA targets).
"""
from __future__ import annotations

import argparse
import os
import signal
import sys
import time

import mpcomm
from mpcomm.harness.common import SEED_BYTES, LocalBuffer, ipv4_bytes, ipv4_pattern, parse_size


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--host-id", default=os.getenv("MPCOMM_HOST_ID", "127.0.0.1:12345"))
    p.add_argument("--tcp-port", type=int, default=int(os.getenv("MPCOMM_TCP_PORT", "12345")),
                   help="control-plane port (0 = ephemeral; the ready line prints it)")
    p.add_argument("--device", default=os.getenv("MPCOMM_DEVICE", ""), help="rail names (CSV); empty = auto")
    p.add_argument("--buffer-size", default=os.getenv("MPCOMM_BUFFER_SIZE", "10G"), help="per buffer, K/M/G/T")
    p.add_argument("--gpu", type=int, default=-1, help="publish HBM of this GPU instead of host DRAM")
    p.add_argument("--num-numas", default="0", help="NUMA nodes of the host buffers, e.g. '0' or '0,1'")
    p.add_argument("--ready-file", default="", help="write the TCP port here once ready")
    p.add_argument("--duration", type=float, default=0.0, help="exit after this many seconds (0 = until signal)")
    p.add_argument("--verbose", "-v", action="store_true", help="print buffer status periodically")
    return p.parse_args(argv)


class Target:
    def __init__(self, host_id: str, device: str, tcp_port: int, size: int, gpu: int, numas):
        self.comm = mpcomm.MPComm()
        if gpu >= 0:
            import torch
            torch.cuda.set_device(gpu)
        if self.comm.init(host_id, device, tcp_port) != 0:
            raise RuntimeError("MPComm init failed")
        self.host_id = host_id
        self.buffers = []
        pattern = ipv4_pattern(ipv4_bytes(host_id), min(size, SEED_BYTES))
        for numa in ([-1] if gpu >= 0 else numas):
            b = LocalBuffer(size, numa=numa, gpu=gpu)
            if self.comm.register_memory(b.ptr, size) != 0:
                raise RuntimeError(f"register_memory failed ({size} bytes, numa {numa}, gpu {gpu})")
            b.write(0, pattern)
            if self.comm.publish_buffer(b.ptr, size, numa) != 0:
                raise RuntimeError("publish_buffer failed")
            self.buffers.append(b)
        if self.comm.start_accept_thread() != 0:
            raise RuntimeError("start_accept_thread failed")
        self.port = self.comm.get_tcp_port()

    def close(self):
        self.comm.unpublish_all_buffers()
        for b in self.buffers:
            self.comm.unregister_memory(b.ptr)
        self.comm.shutdown()
        for b in self.buffers:
            b.close()
        self.buffers = []


def main(argv=None) -> int:
    args = parse_args(argv)
    numas = [int(x) for x in args.num_numas.split(",") if x.strip()] or [0]
    size = parse_size(args.buffer_size)
    stop = {"flag": False}

    def on_signal(signum, frame):
        stop["flag"] = True

    signal.signal(signal.SIGINT, on_signal)
    signal.signal(signal.SIGTERM, on_signal)
    t = Target(args.host_id, args.device, args.tcp_port, size, args.gpu, numas)
    where = f"gpu {args.gpu}" if args.gpu >= 0 else f"numa {numas}"
    print(f"[target] fabric={t.comm.get_fabric_name()} rails={t.comm.get_active_devices()} "
          f"buffers={len(t.buffers)} x {size} bytes ({where})", flush=True)
    if args.ready_file:
        with open(args.ready_file + ".tmp", "w") as f:
            f.write(str(t.port))
        os.replace(args.ready_file + ".tmp", args.ready_file)
    print(f"[target] ready host={args.host_id} port={t.port} buffers={len(t.buffers)}", flush=True)
    t0 = time.monotonic()
    last = t0
    while not stop["flag"] and (args.duration <= 0 or time.monotonic() - t0 < args.duration):
        time.sleep(0.1)
        if args.verbose and time.monotonic() - last >= 5:
            last = time.monotonic()
            print(f"[target] published={t.comm.get_published_buffer_count()} "
                  f"completed_bytes={t.comm.get_nic_completed_bytes()}", flush=True)
    t.close()
    print("[target] stopped", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
