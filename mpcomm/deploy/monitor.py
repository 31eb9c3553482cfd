"""Live link throughput monitor.

RDMA ports: ``/sys/class/infiniband/<dev>/ports/<p>/counters/port_rcv_data``
and ``port_xmit_data`` count 32-bit words; the monitor prints GB/s per
interval from their deltas (parity: reference
user_examples/qos_bench/monitor_rdma_rx_bw.sh). GPUs: PCIe RX/TX throughput
from NVML (``nvmlDeviceGetPcieThroughput``, KB/s over the driver's sampling
window) when the NVML bindings are importable — on RDMA-less GPU boxes this
is the link the GPU fabric's host traffic crosses. Read-only: nothing is
configured on the devices.
"""
from __future__ import annotations

import glob
import os
import time
from typing import Callable, Dict, List, Optional


def rdma_counters(sysfs_root: str = "/", devices: Optional[List[str]] = None) -> Dict[str, Dict[str, int]]:
    """{"<dev>/<port>": {"rx": bytes, "tx": bytes}} from the port counters."""
    out = {}
    base = os.path.join(sysfs_root, "sys/class/infiniband")
    for port_dir in sorted(glob.glob(os.path.join(base, "*", "ports", "*"))):
        dev = port_dir.split(os.sep)[-3]
        if devices and dev not in devices:
            continue
        vals = {}
        for key, name in (("rx", "port_rcv_data"), ("tx", "port_xmit_data")):
            try:
                with open(os.path.join(port_dir, "counters", name)) as f:
                    vals[key] = int(f.read().strip()) * 4  # 32-bit words -> bytes
            except (OSError, ValueError):
                pass
        if vals:
            out[f"{dev}/{os.path.basename(port_dir)}"] = vals
    return out


def nvml_pcie(nvml=None) -> Dict[str, Dict[str, float]]:
    """{"gpu<i>": {"rx_gbs", "tx_gbs"}} from NVML; {} without NVML."""
    if nvml is None:
        try:
            import pynvml as nvml  # nvidia-ml-py
        except ImportError:
            return {}
    try:
        nvml.nvmlInit()
    except Exception:
        return {}
    out = {}
    try:
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            rx = nvml.nvmlDeviceGetPcieThroughput(h, nvml.NVML_PCIE_UTIL_RX_BYTES)
            tx = nvml.nvmlDeviceGetPcieThroughput(h, nvml.NVML_PCIE_UTIL_TX_BYTES)
            out[f"gpu{i}"] = {"rx_gbs": rx * 1024 / 1e9, "tx_gbs": tx * 1024 / 1e9}
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    return out


def monitor(interval: float = 1.0, count: int = 0, sysfs_root: str = "/", devices: Optional[List[str]] = None,
            gpus: bool = True, nvml=None, emit: Callable[[dict], None] = print,
            sleep: Callable[[float], None] = time.sleep, clock: Callable[[], float] = time.monotonic) -> int:
    """Emits one record per interval ({"t", "rdma": {port: {rx_gbs, tx_gbs}},
    "gpu": {...}}); `count` 0 = until interrupted. Returns records emitted."""
    if interval <= 0:
        raise ValueError("interval must be > 0")
    prev, t_prev = rdma_counters(sysfs_root, devices), clock()
    n = 0
    try:
        while count <= 0 or n < count:
            sleep(interval)
            cur, t = rdma_counters(sysfs_root, devices), clock()
            dt = max(t - t_prev, 1e-9)
            rec = {"t": round(t, 3), "rdma": {}}
            for port, v in cur.items():
                p = prev.get(port, {})
                rec["rdma"][port] = {f"{k}_gbs": round((v[k] - p.get(k, v[k])) / dt / 1e9, 3) for k in v}
            if gpus:
                rec["gpu"] = {k: {a: round(b, 3) for a, b in v.items()} for k, v in nvml_pcie(nvml).items()}
            emit(rec)
            prev, t_prev = cur, t
            n += 1
    except KeyboardInterrupt:
        pass
    return n
