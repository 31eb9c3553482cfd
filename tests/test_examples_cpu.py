"""The shipped examples and tools run end to end on CPU (loopback fabric)."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = dict(os.environ, MPCOMM_FABRIC="lo", MPCOMM_LOG_LEVEL="1", PYTHONPATH=ROOT)


def _run(cmd, timeout=120):
    r = subprocess.run(cmd, capture_output=True, text=True, env=ENV, cwd=ROOT, timeout=timeout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return r.stdout


def test_hello_cpp():
    assert "round trip OK" in _run([os.path.join(ROOT, "examples", "bin", "hello_mpcomm")])


def test_hello_python():
    assert "round trip OK" in _run([sys.executable, os.path.join(ROOT, "examples", "hello_mpcomm.py")])


def test_scatter_test_both_mode():
    out = _run([os.path.join(ROOT, "examples", "bin", "scatter_test"), "--mode", "both", "--size", "4M",
                "--batch-size", "4", "--iterations", "3", "--warmup", "1", "--test-type",
                "put,get,scatter,gather,broadcast"])
    for t in ("put", "get", "scatter", "gather", "broadcast"):
        assert f"--- {t} Summary" in out


def test_scatter_test_verify_reads_back_every_slot():
    """--verify: after a broadcast (and after a put) every written slot is
    read back with GETs and compared byte for byte."""
    for t in ("put", "broadcast"):
        out = _run([os.path.join(ROOT, "examples", "bin", "scatter_test"), "--mode", "both", "--size", "1M",
                    "--batch-size", "3", "--iterations", "2", "--warmup", "1", "--test-type", t, "--verify",
                    "--json"])
        assert f"verify {t}: 0 of 3 slots differ" in out, out


def test_check_install():
    assert "install check PASSED" in _run([sys.executable, "-m", "mpcomm.check_install"])


def test_scatter_test_nvls_needs_a_gpu():
    """--nvls makes the process a member of a multicast group of GPU copies:
    without --gpu it is refused before any group is formed."""
    r = subprocess.run([os.path.join(ROOT, "examples", "bin", "scatter_test"), "--mode", "both", "--size", "1M",
                        "--nvls", "g:2"], capture_output=True, text=True, env=ENV, cwd=ROOT, timeout=60)
    assert r.returncode == 2 and "--nvls needs --gpu" in r.stderr, r.stdout + r.stderr
