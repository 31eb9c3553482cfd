#!/usr/bin/env python3
"""Minimal MPComm round trip from Python (parity: reference
user_examples/minimal/hello_mpcomm.py:27-89).

    MPCOMM_FABRIC=lo python examples/hello_mpcomm.py          # any host
    python examples/hello_mpcomm.py --gpu                      # B200: HBM <-> DRAM pool
"""
import argparse
import ctypes
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", action="store_true", help="local buffers in HBM, pool in pinned DRAM")
    ap.add_argument("--size", type=int, default=8 << 20)
    a = ap.parse_args()
    if not a.gpu:
        os.environ.setdefault("MPCOMM_FABRIC", "lo")
    import mpcomm

    n = a.size
    target, initiator = mpcomm.MPComm(), mpcomm.MPComm()
    assert target.init("target") == 0 and initiator.init("initiator") == 0
    if a.gpu:
        import torch

        src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
        back = torch.zeros_like(src)
        pool = torch.zeros(n, dtype=torch.uint8).pin_memory()
        ptrs = (src.data_ptr(), back.data_ptr(), pool.data_ptr())
    else:
        bufs = [ctypes.create_string_buffer(os.urandom(n), n), ctypes.create_string_buffer(n),
                ctypes.create_string_buffer(n)]
        ptrs = tuple(ctypes.addressof(b) for b in bufs)
    s, b, p = ptrs
    assert target.register_memory(p, n) == 0 and target.publish_buffer(p, n) == 0
    assert target.start_accept_thread() == 0
    assert initiator.register_memory(s, n) == 0 and initiator.register_memory(b, n) == 0
    port = target.get_tcp_port()
    assert initiator.connect("target", "127.0.0.1", port) == 0
    remote = initiator.query_remote_buffer("target", "127.0.0.1", port)["addr"]
    h = initiator.put_async(s, "target", remote, n)
    assert initiator.wait_transfer(h, 30000) == 0
    print("put:", initiator.get_transfer_result(h))
    initiator.release_transfer(h)
    h = initiator.get_async(b, "target", remote, n)
    assert initiator.wait_transfer(h, 30000) == 0
    initiator.release_transfer(h)
    if a.gpu:
        import torch

        torch.cuda.synchronize()
        ok = torch.equal(src, back)
    else:
        ok = ctypes.string_at(s, n) == ctypes.string_at(b, n)
    print(f"round trip {'OK' if ok else 'FAILED'} (fabric {initiator.get_fabric_name()})")
    initiator.shutdown()
    target.shutdown()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
