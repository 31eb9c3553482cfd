"""Multi-host runs over a Runner (SSH, or local for loopback hosts).

multi_node      hosts.txt: the first host initiates, every other host runs a
                target; targets start, report ready (a file), the initiator
                runs its tests against all of them, the targets are stopped
                and every log is collected.
multi_initiator hosts.txt + jobs.txt: every host involved runs exactly one
                process — "both" (serve + initiate) for a job's initiator,
                "target" otherwise; all initiators start together (go file),
                finish (done files), then are released (hold file).
check / install / cleanup   connectivity + install self-check, wheel
                install, stop-and-remove of a run directory.

The per-host tool is the library's scatter_test (resolved on each host with
``python -m mpcomm.deploy tool-path scatter_test`` unless --tool-path is
given), so hosts need mpcomm importable (installed wheel or PYTHONPATH).

Flow parity: reference deploy/multi_node_test.sh (targets, ready wait,
initiator, cleanup), deploy/multi_initiator_test.sh (one process per host,
synchronised start), deploy/deploy_all.sh / check_install.sh / cleanup_all.sh.
"""
from __future__ import annotations

import json
import os
import shlex
import time
from typing import Dict, List, Optional

from mpcomm.deploy.hosts import Host, Job
from mpcomm.deploy.profiles import exports, profile_env
from mpcomm.deploy.runner import Runner

WORK_ROOT = "/tmp/mpcomm-deploy"


def launch_prefix(numas: Optional[str]) -> str:
    """`exec` prefix that binds the tool to the CPUs of `numas` (first touch
    places its host buffers there) and keeps the PID of the spawned shell."""
    if not numas:
        return "exec "
    files = " ".join(f"/sys/devices/system/node/node{int(n)}/cpulist" for n in numas.split(","))
    return f"CL=$(cat {files} 2>/dev/null | paste -sd, -); exec ${{CL:+taskset -c $CL}} "


def tool_expr(opts) -> str:
    if getattr(opts, "tool_path", ""):
        return shlex.quote(opts.tool_path)
    py = getattr(opts, "python", "python3")
    return f"\"$({py} -m mpcomm.deploy tool-path scatter_test)\""


def run_dir(opts) -> str:
    return os.path.join(getattr(opts, "work_dir", WORK_ROOT), getattr(opts, "run_id", "") or time.strftime("%Y%m%d-%H%M%S"))


def parse_json_lines(text: str) -> List[dict]:
    out = []
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("{") and line.endswith("}"):
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                pass
    return out


def _gpu_arg(gpu) -> str:
    return f" --gpu {int(gpu)}" if gpu not in (None, "", -1, "-1") else ""


def _collect(runner: Runner, ip: str, path: str, log_dir: Optional[str], name: str) -> str:
    text = runner.read(ip, path)
    if log_dir:
        os.makedirs(log_dir, exist_ok=True)
        with open(os.path.join(log_dir, name), "w") as f:
            f.write(text)
    return text


def multi_node(hosts: List[Host], opts, runner: Runner) -> Dict:
    ini, tgts = hosts[0], hosts[1:]
    env = exports(profile_env(opts.profile, opts.env))
    wd = run_dir(opts)
    tool = tool_expr(opts)
    for ip in sorted({h.ip for h in hosts}):
        runner.run(ip, f"mkdir -p {shlex.quote(wd)}", check=True)
    started = []
    summary: Dict = {"mode": "multi-node", "run_dir": wd, "initiator": ini.id, "targets": [t.id for t in tgts]}
    try:
        for t in tgts:
            cmd = (f"{env}{launch_prefix(opts.target_numas or t.numas)}{tool} --mode target --host-id {t.id} "
                   f"--tcp-port {t.port} --buffer-size {opts.buffer_size}{_gpu_arg(opts.gpu)} "
                   f"--ready-file {wd}/ready.{t.id}")
            runner.spawn(t.ip, cmd, f"{wd}/target.{t.id}.log", f"{wd}/target.{t.id}.pid")
            started.append(t)
        for t in tgts:
            if not runner.wait_for(t.ip, f"{wd}/ready.{t.id}", opts.startup_wait):
                tail = runner.read(t.ip, f"{wd}/target.{t.id}.log")[-2000:]
                raise RuntimeError(f"target {t.id} ({t.ip}) not ready after {opts.startup_wait} s:\n{tail}")
        targets = " ".join(f"--target {t.id}:{t.ip}:{t.port}" for t in tgts)
        cmd = (f"{env}{launch_prefix(opts.num_numas or ini.numas)}{tool} --host-id {ini.id} --size {opts.size} "
               f"--batch-size {opts.batch_size} --iterations {opts.iterations} --warmup {opts.warmup} "
               f"--test-type {opts.test_type}{_gpu_arg(opts.gpu)} --json {targets}")
        r = runner.run(ini.ip, cmd, timeout=opts.timeout)
        if opts.log_dir:
            os.makedirs(opts.log_dir, exist_ok=True)
            with open(os.path.join(opts.log_dir, f"initiator.{ini.id}.log"), "w") as f:
                f.write(r.out + r.err)
        summary["results"] = parse_json_lines(r.out)
        summary["rc"] = r.rc
        if r.rc != 0:
            summary["error"] = (r.err or r.out)[-2000:]
    finally:
        for t in started:
            runner.stop(t.ip, f"{wd}/target.{t.id}.pid")
            _collect(runner, t.ip, f"{wd}/target.{t.id}.log", opts.log_dir, f"target.{t.id}.log")
    summary["ok"] = summary.get("rc") == 0 and bool(summary.get("results"))
    return summary


def _job_opt(job: Job, key: str, default):
    return job.params.get(key, default)


def multi_initiator(hosts: List[Host], jobs: List[Job], opts, runner: Runner) -> Dict:
    env = exports(profile_env(opts.profile, opts.env))
    wd = run_dir(opts)
    tool = tool_expr(opts)
    by_id = {h.id: h for h in hosts}
    init_of = {j.initiator.host.id: j for j in jobs}
    involved = {j.initiator.host.id for j in jobs} | {t.host.id for j in jobs for t in j.targets}
    # Buffer a host serves: the largest any job targeting it asks for.
    buf: Dict[str, str] = {}
    numas: Dict[str, str] = {}
    for j in jobs:
        for t in j.targets:
            want = _job_opt(j, "buffer-size", opts.buffer_size)
            buf[t.host.id] = want if t.host.id not in buf else max(buf[t.host.id], want, key=_size_bytes)
            numas.setdefault(t.host.id, t.numas)
        numas[j.initiator.host.id] = j.initiator.numas
    for ip in sorted({by_id[h].ip for h in involved}):
        runner.run(ip, f"mkdir -p {shlex.quote(wd)}", check=True)
    started: List[Host] = []
    summary: Dict = {"mode": "multi-initiator", "run_dir": wd, "jobs": {}}
    try:
        for hid in sorted(involved):
            h = by_id[hid]
            base = (f"{env}{launch_prefix(numas.get(hid))}{tool} --host-id {hid} --tcp-port {h.port} "
                    f"--buffer-size {buf.get(hid, opts.buffer_size)} --ready-file {wd}/ready.{hid}")
            j = init_of.get(hid)
            if j is None:
                cmd = base.replace(f"{tool} --host-id", f"{tool} --mode target --host-id", 1)
            else:
                targets = " ".join(f"--target {t.host.id}:{t.host.ip}:{t.host.port}" for t in j.targets)
                cmd = (f"{base} --mode both --size {_job_opt(j, 'size', opts.size)} "
                       f"--batch-size {_job_opt(j, 'batch-size', opts.batch_size)} "
                       f"--iterations {_job_opt(j, 'iterations', opts.iterations)} "
                       f"--warmup {_job_opt(j, 'warmup', opts.warmup)} "
                       f"--test-type {_job_opt(j, 'test-type', opts.test_type)}"
                       f"{_gpu_arg(_job_opt(j, 'gpu', opts.gpu))} --json --wait-go-file {wd}/go "
                       f"--done-file {wd}/done.{hid} --hold-file {wd}/hold --hold-timeout {int(opts.timeout)} "
                       f"{targets}")
            runner.spawn(h.ip, cmd, f"{wd}/proc.{hid}.log", f"{wd}/proc.{hid}.pid")
            started.append(h)
        for h in started:
            if not runner.wait_for(h.ip, f"{wd}/ready.{h.id}", opts.startup_wait):
                tail = runner.read(h.ip, f"{wd}/proc.{h.id}.log")[-2000:]
                raise RuntimeError(f"host {h.id} ({h.ip}) not ready after {opts.startup_wait} s:\n{tail}")
        ini_ips = sorted({by_id[hid].ip for hid in init_of})
        for ip in ini_ips:
            runner.run(ip, f"touch {wd}/go", check=True)
        deadline = time.monotonic() + opts.timeout
        for hid in init_of:
            if not runner.wait_for(by_id[hid].ip, f"{wd}/done.{hid}", max(1.0, deadline - time.monotonic())):
                raise RuntimeError(f"initiator {hid} did not finish within {opts.timeout} s")
    finally:
        for ip in sorted({h.ip for h in started}):
            runner.run(ip, f"touch {wd}/hold")
        for h in started:
            runner.stop(h.ip, f"{wd}/proc.{h.id}.pid")
        for h in started:
            text = _collect(runner, h.ip, f"{wd}/proc.{h.id}.log", opts.log_dir, f"proc.{h.id}.log")
            j = init_of.get(h.id)
            if j is not None:
                summary["jobs"][j.name] = {"initiator": h.id, "targets": [t.host.id for t in j.targets],
                                           "results": parse_json_lines(text)}
    summary["ok"] = all(v["results"] for v in summary["jobs"].values()) and len(summary["jobs"]) == len(jobs)
    return summary


def _size_bytes(text: str) -> int:
    from mpcomm.harness.common import parse_size
    return parse_size(text)


def check(hosts: List[Host], opts, runner: Runner) -> Dict:
    py = getattr(opts, "python", "python3")
    out = {}
    for h in hosts:
        ping = runner.run(h.ip, "echo ok", timeout=30)
        chk = runner.run(h.ip, f"{py} -m mpcomm.check_install", timeout=300) if ping.rc == 0 else ping
        out[h.id] = {"reachable": ping.rc == 0 and (runner.dry_run or "ok" in ping.out),
                     "install_ok": chk.rc == 0, "detail": (chk.out + chk.err)[-1500:]}
    return {"mode": "check", "hosts": out, "ok": all(v["reachable"] and v["install_ok"] for v in out.values())}


def install(hosts: List[Host], opts, runner: Runner) -> Dict:
    py = getattr(opts, "python", "python3")
    wd = run_dir(opts)
    name = os.path.basename(opts.wheel)
    out = {}
    for ip in sorted({h.ip for h in hosts}):
        runner.run(ip, f"mkdir -p {shlex.quote(wd)}", check=True)
        cp = runner.put(ip, opts.wheel, f"{wd}/{name}")
        r = runner.run(ip, f"{py} -m pip install --no-index --no-deps --force-reinstall {shlex.quote(wd + '/' + name)}",
                       timeout=900) if cp.rc == 0 else cp
        out[ip] = {"ok": r.rc == 0, "detail": (r.out + r.err)[-1500:]}
    return {"mode": "install", "hosts": out, "ok": all(v["ok"] for v in out.values())}


def cleanup(hosts: List[Host], opts, runner: Runner) -> Dict:
    """Stops every process whose PID file is in the run directory (exact PIDs)
    and removes the directory. Only directories under the work root."""
    wd = os.path.normpath(run_dir(opts))
    root = os.path.normpath(getattr(opts, "work_dir", WORK_ROOT))
    if not wd.startswith(root + os.sep):
        raise ValueError(f"refusing to clean {wd}: not under {root}")
    q = shlex.quote(wd)
    for ip in sorted({h.ip for h in hosts}):
        runner.run(ip, f"for f in {q}/*.pid; do [ -s \"$f\" ] && kill -TERM $(cat \"$f\") 2>/dev/null; done; "
                       f"sleep 1; for f in {q}/*.pid; do [ -s \"$f\" ] && kill -KILL $(cat \"$f\") 2>/dev/null; done; "
                       f"rm -rf -- {q}; exit 0", timeout=60)
    return {"mode": "cleanup", "run_dir": wd, "ok": True}
