"""Install self-check (parity: reference deploy/check_install.sh:1-178).

Verifies, without any RDMA hardware or GPU: the package imports, the native
module and libmpcomm.so load and resolve their shared-library dependencies,
the exported API is present (Python names and the library's C entry
point), an MPComm object initialises on the loopback
fabric, and the C++ headers are where get_include_dir() says.

    python -m mpcomm.check_install      # exit code 0 = OK
"""
from __future__ import annotations

import os
import subprocess
import sys


def main() -> int:
    ok = True

    def check(cond, what):
        nonlocal ok
        print(("  OK    " if cond else "  FAIL  ") + what)
        ok &= bool(cond)

    import mpcomm

    print(f"mpcomm {mpcomm.__version__} at {os.path.dirname(mpcomm.__file__)}")
    check(os.path.exists(mpcomm.native_library_path()), f"native module {mpcomm.native_library_path()}")
    for sym in ("MPComm", "MPCommError", "INVALID_TRANSFER_HANDLE", "H2D_MODE_AUTO", "H2D_MODE_SM", "H2D_MODE_TMA"):
        check(hasattr(mpcomm, sym), f"export {sym}")
    lib = os.path.join(mpcomm.get_lib_dir(), "libmpcomm.so")
    check(os.path.exists(lib), f"shared library {lib}")
    if os.path.exists(lib):
        import ctypes
        try:
            so = ctypes.CDLL(lib)
            check(hasattr(so, "mpcomm_crc32_blocks_noalloc"), "C entry point mpcomm_crc32_blocks_noalloc")
        except OSError as e:
            check(False, f"load {lib}: {e}")
    for path in (mpcomm.native_library_path(), lib):
        if os.path.exists(path):
            out = subprocess.run(["ldd", path], capture_output=True, text=True).stdout
            check("not found" not in out, f"ldd {os.path.basename(path)}: all dependencies resolve")
    inc = mpcomm.get_include_dir()
    check(os.path.exists(os.path.join(inc, "mpcomm.h")), f"header {inc}/mpcomm.h")
    os.environ.setdefault("MPCOMM_FABRIC", "lo")
    os.environ.setdefault("MPCOMM_LOG_LEVEL", "1")
    c = mpcomm.MPComm()
    check(c.init("check-install") == 0, "MPComm().init() on the loopback fabric")
    check(c.get_num_nics() > 0, f"rails: {c.get_active_devices()}")
    c.shutdown()
    print("install check", "PASSED" if ok else "FAILED")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
