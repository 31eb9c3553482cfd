"""CPU runs of the benches that need no GPU, on small cases: they must
complete, verify their data and print one JSON line of the documented
shape."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(module, *args):
    env = dict(os.environ, PYTHONPATH=ROOT, MPCOMM_LOG_LEVEL="1", MPCOMM_FABRIC="lo")
    r = subprocess.run([sys.executable, "-m", module, *args], capture_output=True, text=True, env=env,
                       cwd=ROOT, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_latency_bench():
    d = _run("mpcomm.bench.latency", "--sizes", "4K,64K", "--gaps-ms", "0,1", "--iters", "20")
    assert d["fabric"] == "lo" and len(d["rows"]) == 2 * 2 * 2
    for row in d["rows"]:
        assert 0 < row["p50_us"] <= row["p90_us"] <= row["p99_us"]


def test_staging_bench_config1_small():
    d = _run("mpcomm.bench.staging", "--blocks", "8", "--block-size", "256K", "--iters", "2")
    assert d["staging"]["crc32_verified"] and d["zero_copy"]["crc32_verified"]
    assert d["staging"]["put_gbs"] > 0 and d["staging"]["get_gbs"] > 0


def test_host_bandwidth_probe():
    """CPU threads alone stream a buffer; both directions report a rate."""
    import mpcomm

    d = mpcomm._native.host_bandwidth(64 << 20, 2, -1, 1)
    assert d["threads"] == 2
    assert d["write_gbs"] > 0 and d["read_gbs"] > 0


def test_reference_arm_reports_why_it_cannot_run():
    """The reference arm tries the reference (installed package, else a CMake
    configure of its source tree) and prints one `unavailable` line with the
    reason it found."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"],
                       capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["unavailable"]
