"""Target process for tests/test_mp_cpu.py: serves one published host buffer
over the given fabric and obeys line commands on stdin (crc / die / stop)."""
import ctypes
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import mpcomm  # noqa: E402


def main():
    n = int(sys.argv[1])
    c = mpcomm.MPComm()
    assert c.init("target") == 0
    buf = ctypes.create_string_buffer(n)
    ptr = ctypes.addressof(buf)
    assert c.register_memory(ptr, n) == 0
    assert c.publish_buffer(ptr, n) == 0
    assert c.start_accept_thread() == 0
    print(json.dumps({"port": c.get_tcp_port(), "addr": ptr}), flush=True)
    for line in sys.stdin:
        cmd = line.strip()
        if cmd == "crc":
            print(mpcomm.ops.crc32_host(ctypes.string_at(ptr, n)), flush=True)
        elif cmd == "die":
            os._exit(3)  # abrupt: the kernel resets our sockets
        elif cmd == "stop":
            break
    c.shutdown()


if __name__ == "__main__":
    main()
