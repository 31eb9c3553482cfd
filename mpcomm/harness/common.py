"""Shared pieces of the target/initiator harness: size parsing, the IPv4 byte
pattern, target specs and local buffers (host DRAM on a NUMA node, or HBM).

Behavioural parity: reference user_examples/test_mpcomm.py:117-136 and
mpcomm_target.py:61-81 (the pattern a target seeds and an initiator checks).
"""
from __future__ import annotations

import ctypes
import hashlib
import ipaddress
import mmap
import os
import socket
from dataclasses import dataclass, field
from typing import List, Optional

_SUFFIX = {"": 1, "B": 1, "K": 1 << 10, "KB": 1 << 10, "KIB": 1 << 10, "M": 1 << 20, "MB": 1 << 20,
           "MIB": 1 << 20, "G": 1 << 30, "GB": 1 << 30, "GIB": 1 << 30, "T": 1 << 40, "TB": 1 << 40,
           "TIB": 1 << 40}

# Seed of the first iteration of each mode (base-36 words, as the reference's
# CLI defaults, so a plan can be named by the same --*-seed value).
DEFAULT_SEEDS = {"scatter": int("5CATT3R", 36), "gather": int("6A7H3R", 36), "broadcast": int("BR0ADCA", 36),
                 "put": int("PU7S33D", 36), "get": int("G37S33D", 36)}

# The target seeds this many leading bytes of every buffer with its pattern.
SEED_BYTES = 1 << 20


def parse_size(text: str) -> int:
    """'10GB', '512M', '4096', '1.5G' -> bytes (binary multiples)."""
    s = str(text).strip().upper()
    i = len(s)
    while i and s[i - 1].isalpha():
        i -= 1
    num, suf = s[:i].strip(), s[i:]
    if suf not in _SUFFIX or not num:
        raise ValueError(f"bad size '{text}' (use e.g. 4096, 64K, 512M, 10G)")
    return int(float(num) * _SUFFIX[suf])


def parse_seed(value: Optional[str], fallback: int) -> int:
    """Seed from '0x..', decimal or base-36 text; fallback when absent."""
    if value is None:
        return fallback
    for base in (0, 36):
        try:
            return int(value, base)
        except ValueError:
            pass
    raise ValueError(f"bad seed '{value}'")


def ipv4_bytes(host_id: str) -> List[int]:
    """Pattern bytes of a host id: the IPv4 address of its host part
    ('10.0.0.2:5000' -> 10.0.0.2, as the reference harness), or, when that
    part does not resolve ('t1:5000'), the first four bytes of its SHA-1 so
    two targets with unresolvable names still hold distinct, non-zero
    content (the reference falls back to zeros, which a cleared buffer
    would pass)."""
    host = host_id.split(":", 1)[0]
    try:
        return list(ipaddress.ip_address(socket.gethostbyname(host)).packed)
    except (OSError, ValueError, UnicodeError):
        return list(hashlib.sha1(host.encode()).digest()[:4])


def ipv4_pattern(ip: List[int], n: int) -> bytes:
    """n bytes repeating the four address bytes: the content a target seeds
    and a GATHER/GET checks."""
    if n <= 0:
        return b""
    four = bytes(ip or [0, 0, 0, 0])
    return (four * (n // 4 + 1))[:n]


@dataclass
class TargetSpec:
    """host_id:tcp_addr:tcp_port[:remote_addr:rkey,rkey,...]"""
    host_id: str
    addr: str
    port: int
    remote_addr: int = 0
    rkeys: List[int] = field(default_factory=list)
    buffers: List[dict] = field(default_factory=list)  # from the buffer query

    @staticmethod
    def parse(text: str) -> "TargetSpec":
        parts = text.strip().split(":")
        if len(parts) < 3:
            raise ValueError(f"bad target '{text}': want host_id:tcp_addr:tcp_port[:remote_addr:rkeys]")
        t = TargetSpec(parts[0], parts[1], int(parts[2]))
        if len(parts) >= 5:
            t.remote_addr = int(parts[3], 0)
            t.rkeys = [int(r, 0) for r in parts[4].split(",") if r]
        return t

    def buffer_for_numa(self, numa: int) -> dict:
        """The published buffer on `numa` (else the first one)."""
        for b in self.buffers:
            if b.get("numa_node") == numa:
                return b
        if self.buffers:
            return self.buffers[0]
        return {"addr": self.remote_addr, "length": 0, "numa_node": -1}


def parse_targets(items: List[str]) -> List[TargetSpec]:
    out = []
    for item in items:
        out += [TargetSpec.parse(t) for t in item.split(",") if t.strip()]
    return out


def node_cpus(node: int) -> Optional[set]:
    try:
        txt = open(f"/sys/devices/system/node/node{node}/cpulist").read().strip()
    except OSError:
        return None
    cpus = set()
    for part in txt.split(","):
        a, _, b = part.partition("-")
        if a:
            cpus.update(range(int(a), int(b or a) + 1))
    return (cpus & os.sched_getaffinity(0)) or None


class LocalBuffer:
    """A registered-ready byte buffer: host DRAM placed on `numa` by first
    touch from that node's CPUs, or HBM of `gpu` (torch allocation).

    Host buffers are shared file mappings under /dev/shm (removed on close),
    so the GPU fabric of another process on this host can map and reach
    them; private anonymous memory is the fallback where /dev/shm is absent.
    """

    _count = 0

    def __init__(self, nbytes: int, numa: int = -1, gpu: int = -1):
        self.nbytes, self.numa, self.gpu = nbytes, numa, gpu
        self.path = None
        if gpu >= 0:
            import torch
            self.tensor = torch.zeros(nbytes, dtype=torch.uint8, device=f"cuda:{gpu}")
            self.ptr = self.tensor.data_ptr()
            self._mm = None
            return
        LocalBuffer._count += 1
        path = f"/dev/shm/mpcomm-harness.{os.getpid()}.{LocalBuffer._count}"
        try:
            fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_EXCL, 0o600)
        except OSError:
            fd = -1
        if fd >= 0:
            try:
                os.ftruncate(fd, max(nbytes, 1))
                self._mm = mmap.mmap(fd, max(nbytes, 1), mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
                self.path = path
            finally:
                os.close(fd)
        else:
            self._mm = mmap.mmap(-1, max(nbytes, 1), mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS,
                                 mmap.PROT_READ | mmap.PROT_WRITE)
        self._cbuf = (ctypes.c_char * max(nbytes, 1)).from_buffer(self._mm)
        self.ptr = ctypes.addressof(self._cbuf)
        saved = os.sched_getaffinity(0)
        try:
            cpus = node_cpus(numa) if numa >= 0 else None
            if cpus:
                os.sched_setaffinity(0, cpus)
            ctypes.memset(self.ptr, 0, nbytes)  # first touch on the chosen node
        finally:
            os.sched_setaffinity(0, saved)

    def write(self, off: int, data: bytes) -> None:
        if self.gpu >= 0:
            import torch
            src = torch.frombuffer(bytearray(data), dtype=torch.uint8)
            self.tensor[off:off + len(data)].copy_(src)
            torch.cuda.synchronize(self.gpu)
        else:
            ctypes.memmove(self.ptr + off, data, len(data))

    def clear(self, off: int, n: int) -> None:
        if self.gpu >= 0:
            self.tensor[off:off + n].zero_()
            import torch
            torch.cuda.synchronize(self.gpu)
        else:
            ctypes.memset(self.ptr + off, 0, n)

    def read(self, off: int, n: int) -> bytes:
        if self.gpu >= 0:
            import torch
            torch.cuda.synchronize(self.gpu)
            return self.tensor[off:off + n].cpu().numpy().tobytes()
        return ctypes.string_at(self.ptr + off, n)

    def close(self) -> None:
        if self._mm is not None:
            del self._cbuf
            self._mm.close()
            self._mm = None
        if self.path:
            try:
                os.unlink(self.path)
            except OSError:
                pass
            self.path = None
        self.tensor = None


def preview(b: bytes, n: int = 16) -> str:
    return " ".join(str(x) for x in b[:n]) + (" ..." if len(b) > n else "")


def fmt_rate(bps: float) -> str:
    return f"{bps / 1e9:.3f} GB/s"
