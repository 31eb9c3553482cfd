"""QoS benchmarks on one GPU: a background GET stream (pinned host pool ->
HBM through the GPU fabric, i.e. the same PCIe link) against a foreground
H2D gather, and the runtime throttle's reaction time.

    python -m mpcomm.bench.qos h2d       single-shot H2D QoS (10,240 x 1 KiB tmaGather)
    python -m mpcomm.bench.qos throttle  set_nic_throttle latency and bandwidth
    python -m mpcomm.bench.qos repro     H2D latency alone vs under background GETs

h2d (parity: reference user_examples/qos_bench/bench_h2d_qos.py): isolated
H2D latency (CUDA events, --h2d-iters), isolated background bandwidth
(--measure-seconds), then --repeat single-shot gathers with the background
running, QoS disabled and enabled (enable_h2d_qos(rate, burst)). For every
trial: H2D latency and bandwidth, and the background bandwidth inside the
H2D window (completed-byte counter read at the two host-side boundaries).

throttle (parity: bench_throttle_latency.py): background bandwidth before,
then per cycle set_nic_throttle(outstanding, chunk) and the engine's own
timestamps: worker_us (published -> worker applied), drain_us (applied ->
WRs posted before it completed), effective_us (published -> drained), and
the bandwidth while throttled and after clear_nic_throttle.

repro (parity: _repro_h2d.py): --repeat gathers alone, then with the
background stream, no QoS; prints per-trial latencies and the median ratio.

The background queue is kept shallow (--bg-chunk, --bg-qps,
--bg-outstanding) so that a QoS window bounds the bytes still in flight:
a launched chunk cannot be recalled. Every command prints one JSON line last.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import threading
import time

import torch

import mpcomm
from mpcomm.harness.common import parse_size


class Background:
    """Back-to-back GETs of `size` bytes from the pinned pool into HBM."""

    def __init__(self, comm, size):
        self.comm, self.size = comm, size
        self.pool = torch.empty(size, dtype=torch.uint8, pin_memory=True)
        self.dst = torch.empty(size, dtype=torch.uint8, device="cuda")
        for t in (self.pool, self.dst):
            assert comm.register_memory(t.data_ptr(), size) == 0
        assert comm.publish_buffer(self.pool.data_ptr(), size) == 0
        port = comm.get_tcp_port()
        assert comm.connect("pool", "127.0.0.1", port) == 0
        assert comm.query_remote_buffers("pool", "127.0.0.1", port)
        self.ops, self.error = 0, None
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        try:
            while not self._stop.is_set():
                h = self.comm.get_async(self.dst.data_ptr(), "pool", self.pool.data_ptr(), self.size)
                if h == mpcomm.INVALID_TRANSFER_HANDLE:
                    raise RuntimeError("get_async rejected")
                rc = self.comm.wait_transfer(h, 120000)
                self.comm.release_transfer(h)
                if rc != 0:
                    raise RuntimeError(f"background GET failed ({rc})")
                self.ops += 1
        except Exception as e:  # reported by healthy()
            self.error = e

    def start(self):
        self._stop.clear()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join(timeout=180)

    def healthy(self):
        if self.error:
            raise RuntimeError(f"background stream died: {self.error}")

    def bandwidth(self, seconds):
        """GB/s from the chunk-exact completed-byte counter over `seconds`."""
        b0, o0, t0 = self.comm.get_nic_completed_bytes(), self.ops, time.perf_counter()
        time.sleep(seconds)
        b1, o1, dt = self.comm.get_nic_completed_bytes(), self.ops, time.perf_counter() - t0
        self.healthy()
        if b1 == b0:
            raise RuntimeError("background stream moved no bytes")
        return (b1 - b0) / dt / 1e9


class Gather:
    """One H2D paged gather: num_blocks x block_size from a pinned pool
    (pool_mult x larger, random block indices) into HBM."""

    def __init__(self, comm, block, num_blocks, pool_mult, mode, seed=7, max_sm=0):
        self.comm, self.block, self.n, self.mode, self.max_sm = comm, block, num_blocks, mode, max_sm
        pool_blocks = num_blocks * pool_mult
        self.host = torch.randint(0, 256, (pool_blocks * block,), dtype=torch.uint8).pin_memory()
        self.dram = comm.map_dram_to_gpu(self.host.data_ptr(), self.host.numel())
        assert self.dram, "map_dram_to_gpu failed"
        g = torch.Generator().manual_seed(seed)
        self.idx = torch.randperm(pool_blocks, generator=g)[:num_blocks].to(torch.int64).cuda()
        self.out = torch.empty(num_blocks * block, dtype=torch.uint8, device="cuda")
        self.stream = torch.cuda.Stream()
        self.bytes = num_blocks * block

    def once(self):
        """(latency_us, background bytes completed in the window, window s).
        A short device sleep is queued ahead of the start event so the start
        event, the gather and the end event are all enqueued before the
        stream runs them: host launch time stays out of the interval."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.stream.synchronize()
        t0 = time.perf_counter()
        b0 = self.comm.get_nic_completed_bytes()
        with torch.cuda.stream(self.stream):
            torch.cuda._sleep(40000)
        e0.record(self.stream)
        rc = self.comm.tma_gather(self.dram, self.idx.data_ptr(), self.out.data_ptr(), self.n, self.block,
                                  self.max_sm, self.mode, self.stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"tma_gather failed ({rc})")
        e1.record(self.stream)
        e1.synchronize()
        dt = time.perf_counter() - t0
        b1 = self.comm.get_nic_completed_bytes()
        w = self.comm.get_last_h2d_window(torch.cuda.current_device())
        self.kernel_us = w["duration_us"] if w else float("nan")
        return e0.elapsed_time(e1) * 1e3, b1 - b0, dt

    def check(self):
        want = self.host.view(-1, self.block)[self.idx.cpu()].reshape(-1)
        return bool(torch.equal(self.out.cpu(), want))

    def close(self):
        self.comm.unmap_dram_from_gpu(self.host.data_ptr())


def _stats(v):
    s = sorted(v)
    return {"mean": round(statistics.mean(s), 3), "p50": round(s[len(s) // 2], 3),
            "p99": round(s[min(len(s) - 1, int(round(0.99 * (len(s) - 1))))], 3), "min": round(s[0], 3),
            "max": round(s[-1], 3)}


def _comm(a):
    os.environ["MPCOMM_NVL_CHUNK_SIZE"] = str(parse_size(a.bg_chunk))
    os.environ["MPCOMM_NVL_OUTSTANDING_PER_QP"] = str(a.bg_outstanding)
    os.environ["MPCOMM_QPS_PER_CONNECTION"] = str(a.bg_qps)
    os.environ.setdefault("MPCOMM_PCIE_STAT_ENABLE", "1")  # defer counts in the JSON
    c = mpcomm.MPComm()
    assert c.init("qos-bench") == 0 and c.start_accept_thread() == 0
    return c


def trials(g, bg, label, repeat, gap):
    lat, h2d_bw, nic_bw, kern = [], [], [], []
    for i in range(repeat):
        bg.healthy()
        us, nb, win = g.once()
        lat.append(us)
        kern.append(g.kernel_us)
        h2d_bw.append(g.bytes / (us * 1e-6) / 1e9)
        nic_bw.append(nb / win / 1e9 if win > 0 else 0.0)
        print(f"[{label}] trial {i + 1:3d}: h2d {us:9.2f} us (kernel {kern[-1]:9.2f} us) {h2d_bw[-1]:6.2f} GB/s"
              f"  background in window {nic_bw[-1]:6.2f} GB/s", flush=True)
        if gap > 0:
            time.sleep(gap)
    return lat, h2d_bw, nic_bw, kern


UNLIMITED = 1 << 62  # a QoS rate that never defers: windows are armed, nothing is gated


def cmd_h2d(a):
    c = _comm(a)
    g = Gather(c, a.block_size, a.num_blocks, a.pool_multiplier, a.mode, max_sm=a.max_sm)
    # QoS "off" runs with an unlimited rate: H2D windows still record the
    # gather kernel's device start/end (first CTA / last CTA), nothing waits.
    c.enable_h2d_qos(UNLIMITED, UNLIMITED)
    for _ in range(a.h2d_warmup):
        g.once()
    iso, iso_k = [], []
    for _ in range(a.h2d_iters):
        iso.append(g.once()[0])
        iso_k.append(g.kernel_us)
    ok = g.check()
    bg = Background(c, parse_size(a.size)).start()
    time.sleep(a.warmup_seconds)
    nic_only = bg.bandwidth(a.measure_seconds)
    d = trials(g, bg, "qos off", a.repeat, a.gap_seconds)
    c.enable_h2d_qos(a.qos_rate_bps, a.qos_burst_bytes)
    time.sleep(a.gap_seconds)
    e = trials(g, bg, "qos on", a.repeat, a.gap_seconds)
    c.disable_h2d_qos()
    bg.stop()
    bg.healthy()
    stats = c.get_pcie_domain_stats()
    g.close()
    c.shutdown()
    avg_bw = lambda lat: g.bytes / (statistics.mean(lat) * 1e-6) / 1e9  # noqa: E731
    res = {"bench": "h2d_qos", "h2d_bytes": g.bytes, "block": a.block_size, "blocks": a.num_blocks,
           "mode": a.mode, "verified": ok, "qos_rate_bps": a.qos_rate_bps,
           "h2d_only_us": _stats(iso), "h2d_only_kernel_us": _stats(iso_k), "h2d_only_gbs": round(avg_bw(iso), 3),
           "nic_only_gbs": round(nic_only, 3),
           "qos_off": {"h2d_us": _stats(d[0]), "kernel_us": _stats(d[3]), "h2d_gbs": round(avg_bw(d[0]), 3),
                       "nic_in_window_gbs": _stats(d[2])},
           "qos_on": {"h2d_us": _stats(e[0]), "kernel_us": _stats(e[3]), "h2d_gbs": round(avg_bw(e[0]), 3),
                      "nic_in_window_gbs": _stats(e[2])},
           "defer_count": sum(s.get("defer_count", 0) for s in stats)}
    print(f"\nsingle H2D {g.bytes / 2**20:.2f} MiB | H2D only {res['h2d_only_gbs']:.2f} GB/s "
          f"(p50 {res['h2d_only_us']['p50']:.1f} us, kernel {res['h2d_only_kernel_us']['p50']:.1f} us) | "
          f"background only {nic_only:.2f} GB/s")
    for k in ("qos_off", "qos_on"):
        r = res[k]
        print(f"  concurrent, {k:7s}: H2D {r['h2d_gbs']:6.2f} GB/s (p50 {r['h2d_us']['p50']:.1f} us, "
              f"p99 {r['h2d_us']['p99']:.1f} us, kernel p50 {r['kernel_us']['p50']:.1f} us), "
              f"background in window {r['nic_in_window_gbs']['mean']:.2f} GB/s")
    print(json.dumps(res), flush=True)


def cmd_throttle(a):
    c = _comm(a)
    bg = Background(c, parse_size(a.size)).start()
    time.sleep(a.warmup_seconds)
    base = bg.bandwidth(a.measure_seconds)
    print(f"[throttle] baseline {base:.2f} GB/s", flush=True)
    rows = []
    for cycle in range(a.repeat):
        c.set_nic_throttle(a.throttle_outstanding, parse_size(a.throttle_chunk))
        deadline = time.monotonic() + a.poll_timeout
        st = c.get_throttle_latency()
        while not st["drained"] and time.monotonic() < deadline:
            time.sleep(0.0005)
            st = c.get_throttle_latency()
        if not st["drained"]:
            print(f"[throttle] cycle {cycle}: not drained within {a.poll_timeout} s", flush=True)
            c.clear_nic_throttle()
            continue
        thr = bg.bandwidth(a.measure_seconds)
        c.clear_nic_throttle()
        rest = bg.bandwidth(a.measure_seconds)
        row = {"worker_us": st["worker_us"], "drain_us": st["drain_us"], "effective_us": st["effective_us"],
               "snapshot_wqes": st["snapshot_outstanding_wqes"], "throttled_gbs": round(thr, 3),
               "restored_gbs": round(rest, 3)}
        rows.append(row)
        print(f"[throttle] cycle {cycle}: " + " ".join(f"{k}={v}" for k, v in row.items()), flush=True)
    bg.stop()
    bg.healthy()
    c.shutdown()
    summ = {k: _stats([r[k] for r in rows]) for k in ("worker_us", "drain_us", "effective_us", "snapshot_wqes",
                                                      "throttled_gbs", "restored_gbs")} if rows else {}
    print(json.dumps({"bench": "throttle_latency", "baseline_gbs": round(base, 3), "cycles": len(rows),
                      "throttle_outstanding": a.throttle_outstanding, "throttle_chunk": a.throttle_chunk,
                      "summary": summ}), flush=True)


def cmd_repro(a):
    c = _comm(a)
    g = Gather(c, a.block_size, a.num_blocks, a.pool_multiplier, a.mode, max_sm=a.max_sm)
    for _ in range(5):
        g.once()
    alone = [g.once()[0] for _ in range(a.repeat)]
    bg = Background(c, parse_size(a.size)).start()
    time.sleep(a.warmup_seconds)
    busy = [g.once()[0] for _ in range(a.repeat)]
    bg.stop()
    bg.healthy()
    g.close()
    c.shutdown()
    for i, (x, y) in enumerate(zip(alone, busy)):
        print(f"trial {i + 1:3d}: alone {x:9.2f} us   with background {y:9.2f} us", flush=True)
    ratio = statistics.median(busy) / statistics.median(alone)
    print(json.dumps({"bench": "h2d_repro", "alone_us": _stats(alone), "with_background_us": _stats(busy),
                      "median_ratio": round(ratio, 3)}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("cmd", choices=["h2d", "throttle", "repro"])
    ap.add_argument("--gpu", type=int, default=0)
    ap.add_argument("--size", default="1G", help="bytes per background GET")
    ap.add_argument("--block-size", type=int, default=1024)
    ap.add_argument("--num-blocks", type=int, default=10240)
    ap.add_argument("--pool-multiplier", type=int, default=4)
    ap.add_argument("--mode", type=int, default=2, help="H2D mode: 0 auto, 1 SM, 2 TMA bulk")
    ap.add_argument("--max-sm", type=int, default=0, help="CTA cap of the gather (0 = library default)")
    ap.add_argument("--qos-rate-bps", type=int, default=0, help="0 = pause READ posts in H2D windows")
    ap.add_argument("--qos-burst-bytes", type=int, default=0)
    ap.add_argument("--warmup-seconds", type=float, default=1.0)
    ap.add_argument("--measure-seconds", type=float, default=1.0)
    ap.add_argument("--repeat", type=int, default=30)
    ap.add_argument("--h2d-warmup", type=int, default=100)
    ap.add_argument("--h2d-iters", type=int, default=1000)
    ap.add_argument("--gap-seconds", type=float, default=0.05)
    ap.add_argument("--throttle-outstanding", type=int, default=1)
    ap.add_argument("--throttle-chunk", default="0", help="chunk while throttled (0 = unchanged)")
    ap.add_argument("--poll-timeout", type=float, default=5.0)
    ap.add_argument("--bg-chunk", default="2M")
    ap.add_argument("--bg-qps", type=int, default=2)
    ap.add_argument("--bg-outstanding", type=int, default=2)
    a = ap.parse_args(argv)
    torch.cuda.set_device(a.gpu)
    {"h2d": cmd_h2d, "throttle": cmd_throttle, "repro": cmd_repro}[a.cmd](a)


if __name__ == "__main__":
    main()
