"""Initiator harness: correctness and performance runs of SCATTER, GATHER,
BROADCAST, PUT and GET against one or more running targets
(`python -m mpcomm.harness.target`).

    python -m mpcomm.harness.initiator --targets 10.0.0.2:10.0.0.2:5000 \\
        --mode all --test-mode correctness
    python -m mpcomm.harness.initiator --targets t1:10.0.0.2:5000,t2:10.0.0.3:5000 \\
        --mode both --test-mode performance --iterations 20 --batch-size 4 --gpu 0 --json

Plans are drawn from seeded RNGs (iteration i of a mode uses seed + i):
SCATTER/GATHER move a random length in [--min-chunk-size, --max-chunk-size]
per target, laid out back to back in the local buffer; BROADCAST one random
length to every target; PUT/GET one random length to one random target.
Correctness mode writes seeded random payloads, reads every write back with
a GATHER/GET and compares, checks GATHER/GET data against the pattern each
target seeded (IPv4 bytes of its host id), and writes that pattern back after
every write so the modes can run in any order. Performance mode skips data
preparation and checks and reports GB/s = bytes / wall seconds.

With --num-numas 0,1 there is one local buffer per NUMA node (and the
target's buffer on the same node is used when it published one per node);
--gpu N uses one HBM buffer of GPU N instead. --batch-size B submits B
requests per buffer per iteration before waiting for all of them.

Behavioural parity: reference user_examples/test_mpcomm.py (CLI at
:1421-1608, plans at :539-592, verification at :942-1347).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
import time
from dataclasses import dataclass
from typing import Dict, List

import mpcomm
from mpcomm.harness.common import (DEFAULT_SEEDS, SEED_BYTES, LocalBuffer, TargetSpec, fmt_rate, ipv4_bytes,
                                   ipv4_pattern, parse_seed, parse_targets, preview)

MODES = ("scatter", "gather", "broadcast", "put", "get")
MODE_SETS = {"both": ("scatter", "gather"), "all": MODES}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--mode", choices=list(MODES) + ["both", "all"], default="both")
    p.add_argument("--host-id", default=os.getenv("MPCOMM_HOST_ID", "initiator:0"))
    p.add_argument("--device", default=os.getenv("MPCOMM_DEVICE", ""), help="rail names (CSV); empty = auto")
    p.add_argument("--targets", action="append", required=True,
                   help="host_id:tcp_addr:tcp_port[:remote_addr:rkey,rkey] (repeat or comma-separate)")
    p.add_argument("--min-chunk-size", type=int, default=32 * 1024)
    p.add_argument("--max-chunk-size", type=int, default=128 * 1024)
    p.add_argument("--num-threads", type=int, default=1,
                   help="accepted for CLI compatibility; the engine's workers move the data")
    p.add_argument("--num-numas", default="", help="NUMA nodes of the local buffers, e.g. '0,1'")
    p.add_argument("--gpu", type=int, default=-1, help="local buffer in HBM of this GPU")
    for m in MODES:
        p.add_argument(f"--{m}-seed", default=None, help=f"seed of the {m} plans (int, 0x.., base-36)")
    p.add_argument("--test-mode", choices=["correctness", "performance"], default="correctness")
    p.add_argument("--iterations", type=int, default=1)
    p.add_argument("--warmup", type=int, default=0, help="untimed iterations before the timed ones")
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--async-mode", choices=["wait", "polling"], default="wait")
    p.add_argument("--async-timeout-ms", type=int, default=-1)
    p.add_argument("--poll-interval-us", type=int, default=100)
    p.add_argument("--connect-retries", type=int, default=20, help="connect attempts, 0.5 s apart")
    p.add_argument("--json", action="store_true", help="print one JSON summary line at the end")
    return p.parse_args(argv)


@dataclass
class Plan:
    targets: List[int]        # index into the target list, per segment
    lengths: List[int]
    offsets: List[int]        # local offsets
    payload: bytes = b""      # local bytes [0, sum(lengths)) in correctness mode


class Harness:
    def __init__(self, args):
        self.args = args
        self.perf = args.test_mode == "performance"
        self.targets: List[TargetSpec] = parse_targets(args.targets)
        if args.gpu >= 0:
            import torch
            torch.cuda.set_device(args.gpu)
            self.numas = [-1]
        else:
            self.numas = [int(x) for x in args.num_numas.split(",") if x.strip()] or [-1]
        if args.min_chunk_size <= 0 or args.max_chunk_size < args.min_chunk_size:
            raise ValueError("need 0 < --min-chunk-size <= --max-chunk-size")
        self.comm = mpcomm.MPComm()
        if self.comm.init(args.host_id, args.device, 0) != 0:
            raise RuntimeError("MPComm init failed")
        for t in self.targets:
            self._connect(t)
        self.capacity = args.max_chunk_size * max(1, len(self.targets))
        self.bufs = []
        for numa in self.numas:
            b = LocalBuffer(self.capacity, numa=numa, gpu=args.gpu)
            if self.comm.register_memory(b.ptr, self.capacity) != 0:
                raise RuntimeError("register_memory failed for the local buffer")
            self.bufs.append(b)
        self.patterns = [ipv4_bytes(t.host_id) for t in self.targets]

    def _connect(self, t: TargetSpec):
        rc = -1
        for _ in range(max(1, self.args.connect_retries)):
            rc = self.comm.connect(t.host_id, t.addr, t.port)
            if rc == 0:
                break
            time.sleep(0.5)
        if rc != 0:
            raise RuntimeError(f"connect to {t.host_id} @ {t.addr}:{t.port} failed ({rc})")
        if t.rkeys:
            if self.comm.update_remote_memory_info(t.host_id, t.rkeys) != 0:
                raise RuntimeError(f"update_remote_memory_info({t.host_id}) failed")
            t.buffers = [{"addr": t.remote_addr, "length": 0, "numa_node": -1}]
        else:
            info = self.comm.query_remote_buffers(t.host_id, t.addr, t.port)
            t.buffers = list(info.get("buffers", [])) if isinstance(info, dict) else []
            if not t.buffers:
                raise RuntimeError(f"{t.host_id} publishes no buffer")
            small = [b for b in t.buffers if b["length"] < self.args.max_chunk_size]
            if small:
                raise RuntimeError(f"{t.host_id}: buffer of {small[0]['length']} bytes < --max-chunk-size")

    def remote(self, ti: int, numa: int) -> int:
        return self.targets[ti].buffer_for_numa(numa)["addr"]

    # -- plans ---------------------------------------------------------------
    def plan(self, mode: str, seed: int) -> Plan:
        rng = random.Random(seed)
        lo, hi = self.args.min_chunk_size, self.args.max_chunk_size
        n = len(self.targets)
        if mode in ("scatter", "gather"):
            tix, lengths = list(range(n)), [rng.randint(lo, hi) for _ in range(n)]
        elif mode == "broadcast":
            tix, lengths = list(range(n)), [rng.randint(lo, hi)] * n
        else:
            length = rng.randint(lo, hi)
            tix, lengths = [rng.randrange(n)], [length]
        offsets, cur = [], 0
        for ln in lengths:
            offsets.append(cur)
            cur += ln if mode != "broadcast" else 0
        p = Plan(tix, lengths, offsets)
        if not self.perf and mode in ("scatter", "broadcast", "put"):
            p.payload = random.Random(seed ^ 0x5EED).randbytes(max(offsets[-1] + lengths[-1], 1))
        return p

    # -- submission ----------------------------------------------------------
    def submit(self, mode: str, p: Plan, bi: int) -> int:
        c, lp, numa = self.comm, self.bufs[bi].ptr, self.numas[bi]
        hosts = [self.targets[i].host_id for i in p.targets]
        raddrs = [self.remote(i, numa) for i in p.targets]
        if mode == "scatter":
            return c.scatter_async(lp, hosts, raddrs, p.lengths)
        if mode == "gather":
            return c.gather_async(lp, hosts, raddrs, p.lengths)
        if mode == "broadcast":
            return c.broadcast_async(lp, p.lengths[0], hosts, raddrs)
        if mode == "put":
            return c.put_async(lp, hosts[0], raddrs[0], p.lengths[0])
        return c.get_async(lp, hosts[0], raddrs[0], p.lengths[0])

    def wait_all(self, handles: List[int]) -> int:
        polls = 0
        try:
            if self.args.async_mode == "polling":
                pending = set(handles)
                deadline = (time.monotonic() + self.args.async_timeout_ms / 1e3
                            if self.args.async_timeout_ms >= 0 else None)
                while pending:
                    polls += len(pending)
                    pending = {h for h in pending if not self.comm.is_transfer_complete(h)}
                    if pending:
                        if deadline is not None and time.monotonic() > deadline:
                            raise RuntimeError(f"{len(pending)} transfers still pending after "
                                               f"{self.args.async_timeout_ms} ms")
                        time.sleep(self.args.poll_interval_us / 1e6)
            for h in handles:
                rc = self.comm.wait_transfer(h, self.args.async_timeout_ms)
                if rc != 0:
                    raise RuntimeError(f"wait_transfer failed ({rc})")
                r = self.comm.get_transfer_result(h)
                if r["error_code"] != 0:
                    raise RuntimeError(f"transfer error {r['error_code']}")
        finally:
            for h in handles:
                self.comm.release_transfer(h)
        return polls

    def run_once(self, mode: str, p: Plan):
        if not self.perf:
            for b in self.bufs:
                if p.payload:
                    b.write(0, p.payload)
                else:
                    b.clear(0, self.capacity)
        handles = []
        t0 = time.perf_counter()
        for _ in range(self.args.batch_size):
            for bi in range(len(self.bufs)):
                h = self.submit(mode, p, bi)
                if h == mpcomm.INVALID_TRANSFER_HANDLE:
                    for x in handles:
                        self.comm.release_transfer(x)
                    raise RuntimeError(f"{mode}_async was rejected")
                handles.append(h)
        polls = self.wait_all(handles)
        dt = time.perf_counter() - t0
        nbytes = sum(p.lengths) * len(self.bufs) * self.args.batch_size
        if not self.perf:
            self.verify(mode, p)
        return dt, nbytes, polls

    # -- verification ----------------------------------------------------------
    def _read_back(self, p: Plan, bi: int, offsets: List[int]):
        b = self.bufs[bi]
        b.clear(0, self.capacity)
        hosts = [self.targets[i].host_id for i in p.targets]
        raddrs = [self.remote(i, self.numas[bi]) for i in p.targets]
        h = self.comm.gather_async(b.ptr, hosts, raddrs, p.lengths) if len(hosts) > 1 else \
            self.comm.get_async(b.ptr, hosts[0], raddrs[0], p.lengths[0])
        if h == mpcomm.INVALID_TRANSFER_HANDLE:
            raise RuntimeError("read-back submit failed")
        self.wait_all([h])
        return [b.read(off, ln) for off, ln in zip(offsets, p.lengths)]

    def _restore(self, p: Plan):
        """Write the seeded pattern back into every remote region the plan
        wrote (once per distinct target buffer, after all checks)."""
        b, done = self.bufs[0], set()
        for bi in range(len(self.bufs)):
            for ti, ln in zip(p.targets, p.lengths):
                raddr = self.remote(ti, self.numas[bi])
                n = min(ln, SEED_BYTES)
                if (ti, raddr) in done:
                    continue
                done.add((ti, raddr))
                b.write(0, ipv4_pattern(self.patterns[ti], n))
                self.wait_all([self.comm.put_async(b.ptr, self.targets[ti].host_id, raddr, n)])

    def verify(self, mode: str, p: Plan):
        for bi, numa in enumerate(self.numas):
            if mode in ("scatter", "broadcast", "put"):
                offs = [sum(p.lengths[:k]) for k in range(len(p.lengths))]
                got = self._read_back(p, bi, offs)
                for k, (ti, ln) in enumerate(zip(p.targets, p.lengths)):
                    want = p.payload[p.offsets[k]:p.offsets[k] + ln]
                    self._check(mode, numa, ti, want, got[k])
            else:
                for k, (ti, ln) in enumerate(zip(p.targets, p.lengths)):
                    n = min(ln, SEED_BYTES)
                    got = self.bufs[bi].read(p.offsets[k], n)
                    self._check(mode, numa, ti, ipv4_pattern(self.patterns[ti], n), got)
        if mode in ("scatter", "broadcast", "put"):
            self._restore(p)

    def _check(self, mode, numa, ti, want: bytes, got: bytes):
        tag = f"[{mode} verify numa {numa}] target={self.targets[ti].host_id} len={len(want)}B"
        if want != got:
            bad = next(i for i in range(min(len(want), len(got))) if want[i] != got[i]) \
                if len(want) == len(got) else min(len(want), len(got))
            print(f"{tag} MISMATCH at byte {bad}: expected={preview(want[bad:])} actual={preview(got[bad:])}",
                  flush=True)
            raise AssertionError(f"{mode} verification failed (target {self.targets[ti].host_id})")
        print(f"{tag} OK", flush=True)

    def close(self):
        for b in self.bufs:
            self.comm.unregister_memory(b.ptr)
        self.comm.shutdown()
        for b in self.bufs:
            b.close()


def main(argv=None) -> int:
    args = parse_args(argv)
    modes = MODE_SETS.get(args.mode, (args.mode,))
    h = Harness(args)
    where = f"gpu {args.gpu}" if args.gpu >= 0 else f"numa {h.numas}"
    print(f"[initiator] fabric={h.comm.get_fabric_name()} rails={h.comm.get_active_devices()} targets="
          f"{[t.host_id for t in h.targets]} local={where} batch={args.batch_size} mode={args.test_mode}",
          flush=True)
    summary: Dict[str, dict] = {}
    try:
        for mode in modes:
            seed0 = parse_seed(getattr(args, f"{mode}_seed"), DEFAULT_SEEDS[mode])
            for w in range(args.warmup):
                h.run_once(mode, h.plan(mode, seed0 - 1 - w))
            tot_s = tot_b = 0.0
            for i in range(args.iterations):
                dt, nb, polls = h.run_once(mode, h.plan(mode, seed0 + i))
                tot_s += dt
                tot_b += nb
                extra = f" polls={polls}" if args.async_mode == "polling" else ""
                print(f"[{mode}] iter {i + 1}/{args.iterations}: {nb} B in {dt * 1e6:.1f} us "
                      f"({fmt_rate(nb / dt if dt else 0.0)}){extra}", flush=True)
            rate = tot_b / tot_s if tot_s else 0.0
            summary[mode] = {"gbps": round(rate / 1e9, 4), "bytes": int(tot_b), "seconds": round(tot_s, 6),
                             "iterations": args.iterations}
            print(f"=== {mode}: {int(tot_b)} B over {args.iterations} iterations, {fmt_rate(rate)}", flush=True)
    finally:
        h.close()
    print("[initiator] all tests passed" if not h.perf else "[initiator] done", flush=True)
    if args.json:
        print(json.dumps({"harness": "initiator", "test_mode": args.test_mode, "batch": args.batch_size,
                          "targets": len(h.targets), "results": summary}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
