"""Multi-process plumbing on one NVSwitch box (one process per GPU).

torch.distributed carries the small control messages (handles, ports,
barriers); the bytes move through this package's own kernels:

* ``init_from_env``   — rank/world/local rank from torchrun's environment,
                        CUDA device selection, process group with a timeout.
* ``PeerBuffers``     — a device buffer per rank, CUDA-IPC-mapped into every
                        other rank, so kernels can store straight into a
                        peer's HBM over NVLink (PXN forward, P2P fan-out).
* ``SharedHostPool``  — one host-DRAM pool shared by all local ranks
                        (POSIX shared memory, optionally bound to a NUMA
                        node), pinned and mapped into every rank's GPU.
* ``NvlsGroup``       — an NVLS multicast buffer: one allocation per GPU
                        bound to a multicast object; ``multimem.st`` to the
                        multicast address lands on every GPU
                        (``broadcast_from``: all-source broadcast of a
                        buffer in the root's HBM).
"""
from __future__ import annotations

import mmap
import os
import socket
import uuid
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist

from .. import _native

__all__ = ["init_from_env", "device_view", "PeerBuffers", "SharedHostPool", "NvlsGroup"]


def init_from_env(backend: str = "nccl", timeout_s: int = 120):
    """Initialises torch.distributed from torchrun's env; returns (rank, world, local_rank)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        kw = {"timeout": timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return rank, world, local


class _CudaArray:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, nbytes: int) -> torch.Tensor:
    """uint8 CUDA tensor aliasing ``nbytes`` of device memory at ``ptr`` (no copy)."""
    return torch.as_tensor(_CudaArray(ptr, nbytes), device="cuda")


def _all_gather_object(obj):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


class PeerBuffers:
    """``nbytes`` of HBM per rank, addressable by every rank's kernels.

    The buffers are shared with CUDA IPC; when the allocator hands out VMM
    memory that CUDA IPC cannot export (``PYTORCH_CUDA_ALLOC_CONF=
    expandable_segments:True``), through each rank's descriptor server
    instead (``vmm_offer`` / ``vmm_open``: the allocations' POSIX handles,
    mapped back to back by the peer)."""

    def __init__(self, nbytes: int, dtype=torch.uint8):
        self.nbytes = nbytes
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.local = torch.zeros(nbytes // torch.empty((), dtype=dtype).element_size(), dtype=dtype,
                                 device="cuda")
        ptr = self.local.data_ptr()
        self._vmm_key = 0
        err, handle, off = _native.ipc_export(ptr)
        if err:
            verr, key, base, _ = _native.vmm_offer(ptr, self.local.numel() * self.local.element_size())
            if verr:
                raise RuntimeError(f"neither CUDA IPC ({err}) nor a VMM offer ({verr}) can share this buffer")
            self._vmm_key = key
            info = ("vmm", os.getpid(), key, ptr - base)
        else:
            info = ("ipc", handle, off)
        infos = _all_gather_object(info)
        self._imported = []  # (kind, address, sizes)
        self.ptrs = []
        dev = torch.cuda.current_device()
        for r, inf in enumerate(infos):
            if r == self.rank:
                self.ptrs.append(ptr)
                continue
            if inf[0] == "vmm":
                err, va, sizes = _native.vmm_open(inf[1], inf[2], dev)
                if err:
                    raise RuntimeError(f"vmm_open of rank {r} failed ({err})")
                self._imported.append(("vmm", va, sizes))
                self.ptrs.append(va + inf[3])
            else:
                err, base = _native.ipc_import(inf[1])
                if err:
                    raise RuntimeError(f"ipc_import of rank {r} failed ({err})")
                self._imported.append(("ipc", base, None))
                self.ptrs.append(base + inf[2])

    def peer_view(self, r: int) -> torch.Tensor:
        return device_view(self.ptrs[r], self.nbytes)

    def close(self):
        for kind, b, sizes in self._imported:
            if kind == "vmm":
                _native.vmm_unmap(b, sizes)
            else:
                _native.ipc_release(b)
        self._imported = []
        if self._vmm_key:
            _native.vmm_withdraw(self._vmm_key)
            self._vmm_key = 0


class SharedHostPool:
    """Host pool in POSIX shared memory, pinned + device-mapped in this process.

    The creating rank (``create=True``) sizes and fills the segment; the
    others attach by ``name``. ``numa_node`` >= 0 binds the pages there
    (mbind through the native library's allocator is not needed: the
    creator first-touches the pages while pinned to that node's CPUs).
    """

    def __init__(self, name: str, nbytes: int, create: bool, numa_node: int = -1):
        self.name, self.nbytes = name, nbytes
        self.path = f"/dev/shm/{name}"
        flags = os.O_RDWR | (os.O_CREAT if create else 0)
        fd = os.open(self.path, flags, 0o600)
        try:
            if create:
                os.ftruncate(fd, nbytes)
            self._mm = mmap.mmap(fd, nbytes, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        finally:
            os.close(fd)
        self.tensor = torch.frombuffer(self._mm, dtype=torch.uint8)
        if create:
            saved = os.sched_getaffinity(0)
            try:
                if numa_node >= 0:
                    cpus = _node_cpus(numa_node)
                    if cpus:
                        os.sched_setaffinity(0, cpus)
                self.tensor.view(-1)[:: 4096].zero_()  # first touch on the chosen node
            finally:
                os.sched_setaffinity(0, saved)
        err, dptr, pinned = _native.host_register(self.tensor.data_ptr(), nbytes)
        if err:
            raise RuntimeError(f"host_register failed ({err})")
        self.dev_ptr, self._pinned = dptr, pinned

    def close(self, unlink: bool = False):
        if self._pinned:
            _native.host_unregister(self.tensor.data_ptr())
            self._pinned = False
        del self.tensor
        self._mm.close()
        if unlink and os.path.exists(self.path):
            os.unlink(self.path)


def _node_cpus(node: int):
    try:
        txt = open(f"/sys/devices/system/node/node{node}/cpulist").read().strip()
    except OSError:
        return None
    cpus = set()
    for part in txt.split(","):
        a, _, b = part.partition("-")
        if a:
            cpus.update(range(int(a), int(b or a) + 1))
    return cpus & os.sched_getaffinity(0) or None


class NvlsGroup:
    """Multicast buffer of ``nbytes`` on every rank (NVLS through NVSwitch).

    ``uc`` is this rank's own copy (a uint8 CUDA tensor); ``mc_ptr`` is the
    multicast address a kernel stores to (``mpcomm.ops.nvls_broadcast``).
    Raises RuntimeError where multicast is unsupported (callers fall back to
    ``mpcomm.ops.p2p_fanout`` over PeerBuffers).
    """

    def __init__(self, nbytes: int, root: int = 0):
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.dev = torch.cuda.current_device()
        ok = _all_gather_object(int(_native.multicast_supported(self.dev)))
        if not all(ok):
            raise RuntimeError("NVLS multicast not supported on every GPU")
        err, gran = _native.multicast_granularity(nbytes, self.world)
        if err:
            raise RuntimeError(f"multicast granularity query failed ({err})")
        self.size = (nbytes + gran - 1) // gran * gran
        self.mc = self.mem = self.uc_ptr = self.mc_ptr = 0
        name = None
        token = 0
        srv = None
        fd = -1
        if self.rank == root:
            token = uuid.uuid4().int & ((1 << 63) - 1) | 1
            err, self.mc, fd = _native.multicast_create(self.size, self.world)
            if err:
                raise RuntimeError(f"cuMulticastCreate failed ({err})")
            name = "\0mpcomm-nvls-" + uuid.uuid4().hex
            srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            srv.bind(name)
            srv.listen(self.world)
        holder = [name, token]
        dist.broadcast_object_list(holder, src=root)
        name, self.token = holder
        try:
            if self.rank == root:
                for _ in range(self.world - 1):
                    conn, _ = srv.accept()
                    with conn:
                        socket.send_fds(conn, [b"F"], [fd])
            else:
                with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as s:
                    s.connect(name)
                    _, fds, _, _ = socket.recv_fds(s, 1, 1)
                    err, self.mc = _native.multicast_import(fds[0])
                    os.close(fds[0])
                    if err:
                        raise RuntimeError(f"multicast import failed ({err})")
        finally:
            if srv is not None:
                srv.close()
            if fd >= 0:
                os.close(fd)
        if _native.multicast_add_device(self.mc, self.dev):
            raise RuntimeError("cuMulticastAddDevice failed")
        dist.barrier()
        err, self.mem, self.uc_ptr = _native.multicast_bind_local(self.mc, self.size, self.dev)
        if err:
            raise RuntimeError(f"multicast bind failed ({err})")
        dist.barrier()
        err, self.mc_ptr = _native.multicast_map(self.mc, self.size, self.dev)
        if err:
            raise RuntimeError(f"multicast map failed ({err})")
        self.uc = device_view(self.uc_ptr, self.size)
        dist.barrier()

    @classmethod
    def from_name(cls, name: str, nbytes: int, members: int, create: bool, rank: Optional[int] = None,
                  timeout_ms: int = 60000) -> "NvlsGroup":
        """Joins (or, with ``create``, creates) the multicast group ``name`` of
        ``members`` processes on this box without torch.distributed: the
        creator hands the group object to the others over an abstract Unix
        socket named after the group (native ``createMulticastGroup`` /
        ``joinMulticastGroup``). ``rank`` (default: 0 for the creator, else
        unset) only selects the slice ``broadcast_from`` pulls."""
        err, g = _native.multicast_group(name, nbytes, members, create, timeout_ms)
        if err:
            raise RuntimeError(f"multicast group {name!r}: error {err}")
        self = cls.__new__(cls)
        self.world = members
        self.rank = (0 if create else -1) if rank is None else rank
        self.dev = g["device"]
        self.size = g["length"]
        self.token = g["token"]
        self.mc, self.mem = g["mc_handle"], g["mem_handle"]
        self.uc_ptr, self.mc_ptr = g["uc_addr"], g["mc_addr"]
        self.uc = device_view(self.uc_ptr, self.size)
        return self

    def broadcast_from(self, root_ptr: int, nbytes: int, max_ctas: int = 0,
                       stream: Optional[torch.cuda.Stream] = None, method: str = "load") -> None:
        """All-source broadcast of ``nbytes`` that sit in the root's HBM at
        ``root_ptr`` (an address this rank can load from: the root's own
        pointer on the root, its CUDA-IPC mapping elsewhere, e.g.
        ``PeerBuffers.ptrs[root]``) into every rank's ``uc``.

        Every rank calls it: rank r loads slice r (1/world of the bytes, 4 KiB
        aligned) from the root over NVLink and ``multimem.st``-s it to the
        multicast address, so all GPUs share the multicast work instead of the
        root issuing it alone (8 B200s: 104 us instead of 134 us for 57.9 MB).
        Completion is stream-ordered per rank; the data is complete on every
        rank once every rank's launch has finished (a barrier, or a flag).

        ``method``: "load" reads the slice with 16-byte loads from every
        thread (nvls_broadcast); "bulk" pulls it into shared memory with bulk
        copies (cp.async.bulk, no multicast qualifier) and multicasts from
        there (gather_bcast with one page), keeping more bytes in flight per
        SM across NVLink.
        """
        if nbytes > self.size or nbytes % 16:
            raise ValueError("nbytes must be a multiple of 16 within the group's size")
        if not 0 <= self.rank < self.world:
            raise ValueError("broadcast_from needs this member's rank (NvlsGroup.from_name(..., rank=r))")
        sl = (nbytes // self.world + 4095) // 4096 * 4096
        off = min(self.rank * sl, nbytes)
        ln = max(0, min(sl, nbytes - off))
        if ln == 0:
            return
        s = stream if stream is not None else torch.cuda.current_stream()
        if method == "bulk":
            if not hasattr(self, "_page0"):
                self._page0 = torch.zeros(1, dtype=torch.int64, device="cuda")
            err = _native.gather_bcast(root_ptr + off, 0, self._page0.data_ptr(), 1, ln, self.mc_ptr + off, [], 0, [],
                                       1, 0, max_ctas, int(s.cuda_stream), 0)
        else:
            err = _native.nvls_broadcast(root_ptr + off, self.mc_ptr + off, ln, max_ctas, int(s.cuda_stream))
        if err:
            raise RuntimeError(f"broadcast_from ({method}) failed with CUDA error {err}")

    def register(self, comm) -> None:
        """Registers this rank's copy with an ``MPComm`` (GPU fabric) as a
        member of this multicast group: ``broadcast_async`` from one member to
        all the others' copies (published and queried as usual) then goes out
        as NVLS multicast stores, one launch per chunk."""
        err = comm.register_multicast_memory(self.uc_ptr, self.size, self.mc_ptr, self.token, self.world)
        if err:
            raise RuntimeError(f"register_multicast_memory failed ({err})")

    def close(self):
        torch.cuda.synchronize()
        _native.multicast_teardown(self.mc, self.mem, self.uc_ptr, self.mc_ptr, self.size, self.dev)
        self.mc = self.mem = self.uc_ptr = self.mc_ptr = 0
