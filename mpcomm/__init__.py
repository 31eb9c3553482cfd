"""mpcomm — memory-pool communication for Blackwell (B200, sm_100a).

Python surface of the native library: the ``MPComm`` class (same snake_case
methods, arguments and return shapes as UCL-MPComm's ``mpcomm`` module,
reference python/mpcomm_py.cpp:687-900), the ``MPCommError`` enum,
``INVALID_TRANSFER_HANDLE`` and ``H2D_MODE_*`` constants, plus SDK path
helpers (reference python/__init__.py:47-93).

Subpackages:
  * ``mpcomm.ops``      tensor-level wrappers of the sm_100a kernels
                        (paged gather/scatter, CRC32, PXN forward, NVLS).
  * ``mpcomm.parallel`` multi-process plumbing: torch.distributed bootstrap,
                        CUDA IPC handle exchange, NVLS multicast groups.
  * ``mpcomm.models``   workload shapes the benchmarks use (Llama-3-8B paged
                        KV pool, RL rollout / expert-ID batches).
  * ``mpcomm.utils``    timing, clock sampling, seeds.
  * ``mpcomm.harness``  target / initiator command-line harness.
  * ``mpcomm.deploy``   multi-host orchestration (hosts.txt / jobs.txt over
                        SSH), environment profiles, link monitor.
"""
import glob as _glob
import os as _os

_PACKAGE_DIR = _os.path.dirname(_os.path.abspath(__file__))
__version__ = "0.1.0"

try:
    from ._mpcomm import (  # noqa: F401
        H2D_MODE_AUTO,
        H2D_MODE_SM,
        H2D_MODE_TMA,
        INVALID_TRANSFER_HANDLE,
        MPComm,
        MPCommError,
    )
    from . import _mpcomm as _native  # noqa: F401
except ImportError as _e:  # pragma: no cover - exercised only on broken installs
    _so = _glob.glob(_os.path.join(_PACKAGE_DIR, "_mpcomm*.so"))
    if _so:
        raise ImportError(
            f"mpcomm native module found ({_so[0]}) but failed to load: {_e}\n"
            f"Hint: run 'ldd {_so[0]}' to check for missing shared libraries."
        ) from _e
    raise ImportError(
        "mpcomm native module is not built. Build it with "
        "`cmake -S . -B build -G Ninja && cmake --build build` "
        "or `python -c 'import __graft_entry__ as g; g.build()'`."
    ) from _e


_SUBPACKAGES = ("ops", "parallel", "models", "utils", "bench", "harness", "deploy")


def __getattr__(name):
    # Subpackages import torch; load them on first use so `import mpcomm`
    # stays light for C-API-style users.
    if name in _SUBPACKAGES:
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(f"module 'mpcomm' has no attribute {name!r}")


def native_library_path() -> str:
    """Absolute path of the loaded native module (for provenance checks)."""
    return _native.__file__


def get_include_dir() -> str:
    """Directory holding mpcomm.h / mpcomm_log.h (wheel: mpcomm/include; source tree: include/)."""
    inside = _os.path.join(_PACKAGE_DIR, "include")
    return inside if _os.path.isdir(inside) else _os.path.join(_os.path.dirname(_PACKAGE_DIR), "include")


def tool_path(name: str) -> str:
    """Path of a bundled command-line tool (``scatter_test``, ``hello_mpcomm``):
    mpcomm/bin in a wheel, examples/bin in a source-tree build."""
    for d in (_os.path.join(_PACKAGE_DIR, "bin"), _os.path.join(_os.path.dirname(_PACKAGE_DIR), "examples", "bin")):
        p = _os.path.join(d, name)
        if _os.path.isfile(p) and _os.access(p, _os.X_OK):
            return p
    raise FileNotFoundError(f"mpcomm tool '{name}' is not built (looked in mpcomm/bin and examples/bin)")


def get_lib_dir() -> str:
    """Directory holding libmpcomm.so."""
    return _os.path.join(_PACKAGE_DIR, "lib")


def get_cmake_dir() -> str:
    """CMake package directory of an installed build (lib/cmake/mpcomm)."""
    return _os.path.join(_PACKAGE_DIR, "lib", "cmake", "mpcomm")


def get_check_install_script() -> str:
    """Path of the install self-check script."""
    return _os.path.join(_PACKAGE_DIR, "check_install.py")


__all__ = [
    "MPComm",
    "MPCommError",
    "INVALID_TRANSFER_HANDLE",
    "H2D_MODE_AUTO",
    "H2D_MODE_SM",
    "H2D_MODE_TMA",
    "__version__",
    "get_include_dir",
    "get_lib_dir",
    "get_cmake_dir",
    "get_check_install_script",
    "native_library_path",
]
