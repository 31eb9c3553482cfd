"""Deployment tooling on one machine: hosts.txt / jobs.txt parsing and its
errors, environment profiles, SSH command shapes (dry run), multi-node and
multi-initiator runs of scatter_test over the socket fabric with every host
on 127.0.0.1, cleanup by exact PIDs, and the link monitor against a fake
sysfs tree and a fake NVML."""
import json
import os
import subprocess
import sys

import pytest

from mpcomm.deploy import HostsError, Runner, exports, parse_hosts, parse_jobs, profile_env
from mpcomm.deploy import monitor as M
from mpcomm.deploy import orchestrate as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOSTS = """# ID IP PORT NUMAS
1 127.0.0.1 {p1} 0
2 127.0.0.1 {p2} -
3 127.0.0.1 {p3}
"""


def _free_ports(n):
    import socket
    socks = [socket.socket() for _ in range(n)]
    for s in socks:
        s.bind(("127.0.0.1", 0))
    ports = [s.getsockname()[1] for s in socks]
    for s in socks:
        s.close()
    return ports


def test_parse_hosts_defaults_and_errors():
    hs = parse_hosts("a 10.0.0.1\nb 10.0.0.2 5000 0,1  # comment\n\nc 10.0.0.3 - -\n")
    assert [(h.id, h.ip, h.port, h.numas) for h in hs] == [("a", "10.0.0.1", 12345, "0"), ("b", "10.0.0.2", 5000, "0,1"),
                                                           ("c", "10.0.0.3", 12345, "0")]
    for bad, msg in [("10.0.0.1 10.0.0.1\nb 10.0.0.2", "not an IP"), ("a 1.1.1.1\na 1.1.1.2", "duplicate"),
                     ("a 1.1.1.1", "at least 2"), ("a\nb 1.1.1.1", "expected"), ("a 1.1.1.1 x\nb 1.1.1.2", "bad port"),
                     ("a 1.1.1.1 1 0;1\nb 1.1.1.2", "NUMA")]:
        with pytest.raises(HostsError, match=msg):
            parse_hosts(bad)


def test_parse_jobs_order_overrides_and_errors():
    hs = parse_hosts("1 1.1.1.1 1 0\n2 1.1.1.2 2 1\n3 1.1.1.3 3 0\n")
    text = """[global]
size = 1G
iterations = 20
[jobs order]
B, A
[A]
initiator = 1
target = 2 3[1]
[B]
initiator = 3[0,1]
target = 1
target = 2
size = 512M
"""
    jobs = parse_jobs(text, hs)
    assert [j.name for j in jobs] == ["B", "A"]
    b, a = jobs
    assert b.initiator.host.id == "3" and b.initiator.numas == "0,1" and [t.host.id for t in b.targets] == ["1", "2"]
    assert b.params == {"size": "512M", "iterations": "20"} and a.params == {"size": "1G", "iterations": "20"}
    assert a.targets[0].numas == "1" and a.targets[1].numas == "1"
    bad = [("[A]\ninitiator = 9\ntarget = 1", "not in hosts"), ("[A]\ninitiator = 1\ntarget = 1", "own initiator"),
           ("[A]\ninitiator = 1\ninitiator = 2\ntarget = 3", "more than one"), ("[A]\ninitiator = 1", "needs one"),
           ("[A]\ninitiator = 1\ntarget = 2\n[B]\ninitiator = 1\ntarget = 3", "one process per host"),
           ("[A]\ninitiator = 1\ntarget = 2\ncolour = red", "unknown key"), ("x = 1", "outside a section"),
           ("[jobs order]\nZ\n[A]\ninitiator = 1\ntarget = 2", "unknown job")]
    for t, msg in bad:
        with pytest.raises(HostsError, match=msg):
            parse_jobs(t, hs)


def test_profiles_and_exports():
    env = profile_env("stage0", ["MPCOMM_LOG_LEVEL=2"], environ={"MPCOMM_FABRIC": "sock", "HOME": "/x"})
    assert env["MPCOMM_MAX_RDMA_TRANSFER_SIZE"] == "65536" and env["MPCOMM_QPS_PER_CONNECTION"] == "4"
    assert env["MPCOMM_FABRIC"] == "sock" and "HOME" not in env and env["MPCOMM_LOG_LEVEL"] == "2"
    assert "export MPCOMM_PCIE_STAT_ENABLE=1; " in exports(env)
    with pytest.raises(KeyError):
        profile_env("nope")
    with pytest.raises(ValueError):
        profile_env(None, ["bad"])


def test_ssh_dry_run_commands(tmp_path):
    seen = []
    r = Runner(ssh_user="me", ssh_options=["-p", "2222"], dry_run=True, echo=seen.append)
    assert r.argv("10.0.0.9", "echo hi")[:3] == ["ssh", "-o", "BatchMode=yes"]
    assert r.argv("10.0.0.9", "echo hi")[-2:] == ["me@10.0.0.9", "echo hi"]
    assert r.argv("127.0.0.1", "echo hi") == ["bash", "-c", "echo hi"]

    class Opts:
        size, buffer_size, batch_size, iterations, warmup, test_type = "1G", "4G", 4, 10, 3, "put,get"
        gpu, num_numas, target_numas, profile, env, tool_path = 0, "", "", "multinode", [], "/opt/st"
        startup_wait, timeout, log_dir, work_dir, run_id, python = 1.0, 10.0, "", str(tmp_path), "r1", "python3"

    hosts = parse_hosts("1 10.0.0.1 5000 0\n2 10.0.0.2 5001 1\n")
    res = O.multi_node(hosts, Opts, r)
    cmds = "\n".join(r.log)
    assert "10.0.0.2: nohup bash -c" in cmds and "--mode target --host-id 2 --tcp-port 5001" in cmds
    assert "--target 2:10.0.0.2:5001" in cmds and "--gpu 0" in cmds and "MPCOMM_QPS_PER_CONNECTION=4" in cmds
    assert "node1/cpulist" in cmds and "kill -TERM" in cmds
    assert res["mode"] == "multi-node"


@pytest.fixture
def hosts_file(tmp_path):
    p = tmp_path / "hosts.txt"
    p.write_text(HOSTS.format(**dict(zip(("p1", "p2", "p3"), _free_ports(3)))))
    return p


def _deploy(tmp_path, *args):
    env = dict(os.environ, PYTHONPATH=ROOT, MPCOMM_FABRIC="sock", MPCOMM_LOG_LEVEL="1")
    r = subprocess.run([sys.executable, "-m", "mpcomm.deploy", *args, "--work-dir", str(tmp_path / "work"),
                        "--run-id", "t", "--log-dir", str(tmp_path / "logs")],
                       capture_output=True, text=True, env=env, cwd=tmp_path, timeout=240)
    return r, json.loads(r.stdout.strip().splitlines()[-1]) if r.stdout.strip() else {}


def _alive(pidfile):
    try:
        os.kill(int(open(pidfile).read()), 0)
        return True
    except (OSError, ValueError):
        return False


def test_multi_node_local(tmp_path, hosts_file):
    r, res = _deploy(tmp_path, "multi-node", "--hosts", str(hosts_file), "--size", "1M", "--buffer-size", "8M",
                     "--batch-size", "2", "--iterations", "2", "--warmup", "1", "--test-type", "put,get,scatter",
                     "--profile", "stage0")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert res["ok"] and [x["test"] for x in res["results"]] == ["put", "get", "scatter"]
    assert all(x["targets"] == 2 and x["gbps"] > 0 for x in res["results"])
    for hid in ("2", "3"):
        assert not _alive(tmp_path / "work" / "t" / f"target.{hid}.pid")
        assert "(ready)" in (tmp_path / "logs" / f"target.{hid}.log").read_text()


def test_multi_initiator_local(tmp_path, hosts_file):
    jobs = tmp_path / "jobs.txt"
    jobs.write_text("[global]\nsize = 1M\niterations = 2\nwarmup = 1\nbuffer-size = 8M\n"
                    "[A]\ninitiator = 1\ntarget = 2 3\n[B]\ninitiator = 2[0]\ntarget = 1\ntest-type = get\n")
    r, res = _deploy(tmp_path, "multi-initiator", "--hosts", str(hosts_file), "--jobs", str(jobs), "--batch-size", "2")
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert res["ok"] and set(res["jobs"]) == {"A", "B"}
    assert [x["test"] for x in res["jobs"]["A"]["results"]] == ["put", "get"]
    assert [x["test"] for x in res["jobs"]["B"]["results"]] == ["get"] and res["jobs"]["B"]["results"][0]["targets"] == 1
    for hid in ("1", "2", "3"):
        assert not _alive(tmp_path / "work" / "t" / f"proc.{hid}.pid")
    r, res = _deploy(tmp_path, "cleanup", "--hosts", str(hosts_file))
    assert res["ok"] and not (tmp_path / "work" / "t").exists()


def test_multi_node_reports_target_failure(tmp_path):
    """A target that cannot start (its port is taken) fails the run with
    its log, and nothing is left running."""
    import socket
    busy = socket.socket()
    busy.bind(("127.0.0.1", 0))
    busy.listen(1)
    p1, = _free_ports(1)
    hosts = tmp_path / "hosts.txt"
    hosts.write_text(f"1 127.0.0.1 {p1}\n2 127.0.0.1 {busy.getsockname()[1]}\n")
    try:
        env = dict(os.environ, PYTHONPATH=ROOT, MPCOMM_FABRIC="sock", MPCOMM_LOG_LEVEL="1")
        r = subprocess.run([sys.executable, "-m", "mpcomm.deploy", "multi-node", "--hosts", str(hosts), "--size", "1M",
                            "--buffer-size", "4M", "--startup-wait", "5", "--work-dir", str(tmp_path / "w"),
                            "--run-id", "t"], capture_output=True, text=True, env=env, timeout=120)
        assert r.returncode != 0 and "not ready" in r.stderr
        assert not _alive(tmp_path / "w" / "t" / "target.2.pid")
    finally:
        busy.close()


def test_monitor_fake_sysfs_and_nvml(tmp_path):
    ctr = tmp_path / "sys/class/infiniband/mlx5_0/ports/1/counters"
    ctr.mkdir(parents=True)
    (ctr / "port_rcv_data").write_text("0\n")
    (ctr / "port_xmit_data").write_text("0\n")
    ticks = iter(range(100))
    state = {"n": 0}

    def sleep(_):
        state["n"] += 1
        (ctr / "port_rcv_data").write_text(str(state["n"] * 250_000_000) + "\n")  # +1 GB per tick

    class FakeNvml:
        NVML_PCIE_UTIL_RX_BYTES, NVML_PCIE_UTIL_TX_BYTES = 1, 0
        nvmlInit = nvmlShutdown = staticmethod(lambda: None)
        nvmlDeviceGetCount = staticmethod(lambda: 2)
        nvmlDeviceGetHandleByIndex = staticmethod(lambda i: i)
        nvmlDeviceGetPcieThroughput = staticmethod(lambda h, c: 1_000_000 * (h + 1) if c == 1 else 0)

    recs = []
    n = M.monitor(1.0, 3, str(tmp_path), None, True, nvml=FakeNvml, emit=recs.append, sleep=sleep,
                  clock=lambda: float(next(ticks)))
    assert n == 3 and all(r["rdma"]["mlx5_0/1"]["rx_gbs"] == 1.0 and r["rdma"]["mlx5_0/1"]["tx_gbs"] == 0 for r in recs)
    assert recs[0]["gpu"]["gpu1"]["rx_gbs"] == round(2_000_000 * 1024 / 1e9, 3)
    with pytest.raises(ValueError):
        M.monitor(0, 1, str(tmp_path))
