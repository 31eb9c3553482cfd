"""Command execution on the hosts of a deployment: over SSH (BatchMode, no
password prompts) or, for loopback addresses or with ``local=True``, on this
machine through bash — so a whole multi-host run can be exercised on one box.

Background processes are started with their PID written to a file and are
stopped by that exact PID (never by name or pattern).
"""
from __future__ import annotations

import shlex
import subprocess
import time
from dataclasses import dataclass
from typing import List, Optional, Sequence

LOOPBACK = {"127.0.0.1", "localhost", "::1"}


@dataclass
class Result:
    rc: int
    out: str
    err: str


class Runner:
    def __init__(self, ssh_user: str = "", ssh_options: Sequence[str] = (), local: bool = False,
                 dry_run: bool = False, echo=print):
        self.ssh_user, self.ssh_options = ssh_user, list(ssh_options)
        self.local, self.dry_run, self.echo = local, dry_run, echo
        self.log: List[str] = []  # every command issued (also in dry-run)

    def is_local(self, ip: str) -> bool:
        return self.local or ip in LOOPBACK

    def argv(self, ip: str, cmd: str) -> List[str]:
        if self.is_local(ip):
            return ["bash", "-c", cmd]
        dest = f"{self.ssh_user}@{ip}" if self.ssh_user else ip
        return ["ssh", "-o", "BatchMode=yes", "-o", "ConnectTimeout=10", *self.ssh_options, dest, cmd]

    def run(self, ip: str, cmd: str, timeout: float = 120.0, check: bool = False) -> Result:
        self.log.append(f"{ip}: {cmd}")
        if self.dry_run:
            self.echo(f"[dry-run] {ip}: {cmd}")
            return Result(0, "", "")
        try:
            p = subprocess.run(self.argv(ip, cmd), capture_output=True, text=True, timeout=timeout)
            r = Result(p.returncode, p.stdout, p.stderr)
        except subprocess.TimeoutExpired as e:
            r = Result(124, e.stdout or "" if isinstance(e.stdout, str) else "", f"timed out after {timeout} s")
        if check and r.rc != 0:
            raise RuntimeError(f"{ip}: command failed ({r.rc}): {cmd}\n{r.err[-2000:]}")
        return r

    def spawn(self, ip: str, cmd: str, log: str, pidfile: str) -> Result:
        """Starts `cmd` detached on `ip`, output to `log`, PID to `pidfile`."""
        inner = f"nohup bash -c {shlex.quote(cmd)} > {shlex.quote(log)} 2>&1 < /dev/null & echo $! > {shlex.quote(pidfile)}"
        return self.run(ip, inner, timeout=60, check=True)

    def exists(self, ip: str, path: str) -> bool:
        if self.dry_run:
            return True
        return self.run(ip, f"test -e {shlex.quote(path)}", timeout=30).rc == 0

    def wait_for(self, ip: str, path: str, timeout: float, poll: float = 0.2) -> bool:
        deadline = time.monotonic() + timeout
        while True:
            if self.exists(ip, path):
                return True
            if time.monotonic() >= deadline:
                return False
            time.sleep(poll)

    def read(self, ip: str, path: str) -> str:
        if self.dry_run:
            return ""
        r = self.run(ip, f"cat {shlex.quote(path)} 2>/dev/null", timeout=60)
        return r.out

    def stop(self, ip: str, pidfile: str, grace: float = 10.0) -> None:
        """SIGTERM the PID recorded in `pidfile`, SIGKILL after `grace` s."""
        q = shlex.quote(pidfile)
        self.run(ip, f"if [ -s {q} ]; then p=$(cat {q}); kill -TERM $p 2>/dev/null; "
                     f"for i in $(seq {int(grace * 10)}); do kill -0 $p 2>/dev/null || exit 0; sleep 0.1; done; "
                     f"kill -KILL $p 2>/dev/null; fi; exit 0", timeout=grace + 30)

    def put(self, ip: str, src: str, dst: str, timeout: float = 600.0) -> Result:
        self.log.append(f"{ip}: put {src} -> {dst}")
        if self.dry_run:
            self.echo(f"[dry-run] {ip}: copy {src} -> {dst}")
            return Result(0, "", "")
        if self.is_local(ip):
            argv = ["cp", src, dst]
        else:
            dest = f"{self.ssh_user}@{ip}" if self.ssh_user else ip
            argv = ["scp", "-q", "-o", "BatchMode=yes", *self.ssh_options, src, f"{dest}:{dst}"]
        p = subprocess.run(argv, capture_output=True, text=True, timeout=timeout)
        return Result(p.returncode, p.stdout, p.stderr)


def numa_prefix(numas: Optional[str]) -> str:
    """Shell prefix binding a process to the CPUs of the given NUMA nodes
    (first-touch places its host buffers there); empty on hosts without
    the sysfs node directories."""
    if not numas:
        return ""
    files = " ".join(f"/sys/devices/system/node/node{int(n)}/cpulist" for n in numas.split(","))
    return f'CL=$(cat {files} 2>/dev/null | paste -sd, -); ${{CL:+taskset -c $CL}} '
