"""Target/initiator harness over the software socket fabric (two target
processes, one initiator process): every mode verified, multi-buffer and
polling paths, performance JSON, and a mismatch that must be caught."""
import json

import pytest

from harness_util import TargetProc, harness_env, run_initiator


@pytest.fixture
def two_targets(tmp_path):
    env = harness_env(MPCOMM_FABRIC="sock")
    ts = [TargetProc(tmp_path, h, env, "--buffer-size", "4M") for h in ("127.0.0.1:0", "127.0.0.2:0")]
    yield env, ts
    codes = [t.stop() for t in ts]
    assert codes == [0, 0], codes  # clean shutdown on SIGTERM


def _spec(ts, ids=("127.0.0.1", "127.0.0.2")):
    return ",".join(f"{i}:127.0.0.1:{t.port}" for i, t in zip(ids, ts))


def test_all_modes_correctness(two_targets):
    env, ts = two_targets
    r = run_initiator(env, "--targets", _spec(ts), "--mode", "all", "--iterations", "2", "--json")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "[initiator] all tests passed" in r.stdout
    for mode in ("scatter", "gather", "broadcast", "put", "get"):
        assert f"[{mode} verify" in r.stdout
    res = json.loads(r.stdout.strip().splitlines()[-1])["results"]
    assert set(res) == {"scatter", "gather", "broadcast", "put", "get"}
    assert all(v["bytes"] > 0 and v["gbps"] > 0 for v in res.values())


def test_multi_buffer_batch_polling(two_targets):
    env, ts = two_targets
    r = run_initiator(env, "--targets", _spec(ts), "--mode", "both", "--num-numas", "0,0", "--batch-size", "3",
                      "--async-mode", "polling", "--poll-interval-us", "50", "--scatter-seed", "0x1234",
                      "--gather-seed", "zz9", "--min-chunk-size", "4096", "--max-chunk-size", "262144")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("[scatter verify") == 4 and "polls=" in r.stdout


def test_performance_mode_json(two_targets):
    env, ts = two_targets
    r = run_initiator(env, "--targets", _spec(ts), "--mode", "all", "--test-mode", "performance",
                      "--iterations", "3", "--warmup", "1", "--batch-size", "4", "--json")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["test_mode"] == "performance" and line["batch"] == 4
    assert "verify" not in r.stdout


def test_wrong_target_content_is_caught(two_targets):
    """The initiator names target 2 with target 1's id: its GATHER data
    carries the other host's pattern and verification must fail."""
    env, ts = two_targets
    r = run_initiator(env, "--targets", f"127.0.0.1:127.0.0.1:{ts[1].port}", "--mode", "get")
    assert r.returncode != 0
    assert "MISMATCH" in r.stdout and "get verification failed" in r.stderr
