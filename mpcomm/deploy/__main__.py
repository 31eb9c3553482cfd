"""python -m mpcomm.deploy <command> ...

    multi-node       --hosts hosts.txt   first host initiates, the rest serve
    multi-initiator  --hosts hosts.txt --jobs jobs.txt
    check            --hosts hosts.txt   reachability + install self-check
    install          --hosts hosts.txt --wheel mpcomm-*.whl
    cleanup          --hosts hosts.txt --run-id ID
    monitor          [--interval 1] [--count N] [--device mlx5_0]
    profiles         list the environment profiles
    tool-path NAME   print the path of a bundled tool (scatter_test, ...)

Hosts whose IP is a loopback address (or all hosts with --local) run through
local bash instead of SSH. Every run command prints one JSON summary line
and exits non-zero when the run failed.
"""
from __future__ import annotations

import argparse
import json
import sys

from mpcomm.deploy import hosts as H
from mpcomm.deploy import monitor as M
from mpcomm.deploy import orchestrate as O
from mpcomm.deploy.profiles import PROFILES
from mpcomm.deploy.runner import Runner


def _common(p):
    p.add_argument("--hosts", default="hosts.txt")
    p.add_argument("--local", action="store_true", help="run every host's commands on this machine")
    p.add_argument("--dry-run", action="store_true", help="print the commands instead of running them")
    p.add_argument("--ssh-user", default="")
    p.add_argument("--ssh-option", action="append", default=[], help="extra ssh -o style arguments (repeat)")
    p.add_argument("--work-dir", default=O.WORK_ROOT, help="per-host run directories live under this")
    p.add_argument("--run-id", default="", help="run directory name (default: a timestamp)")
    p.add_argument("--python", default="python3", help="interpreter on the hosts")
    p.add_argument("--log-dir", default="", help="copy every host's log here")


def _bench(p):
    p.add_argument("--size", default="1G", help="bytes per request (K/M/G)")
    p.add_argument("--buffer-size", default="4G", help="target buffer")
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--iterations", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--test-type", default="put,get", help="put,get,scatter,gather,broadcast")
    p.add_argument("--gpu", type=int, default=-1, help="buffers in HBM of this GPU on every host")
    p.add_argument("--num-numas", default="", help="initiator NUMA override")
    p.add_argument("--target-numas", default="", help="target NUMA override")
    p.add_argument("--profile", default="", help=f"environment profile ({', '.join(sorted(PROFILES))})")
    p.add_argument("--env", action="append", default=[], help="KEY=VALUE exported on every host (repeat)")
    p.add_argument("--tool-path", default="", help="scatter_test path on the hosts (default: resolved there)")
    p.add_argument("--startup-wait", type=float, default=30.0, help="seconds for targets to become ready")
    p.add_argument("--timeout", type=float, default=1800.0, help="seconds for the initiators to finish")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m mpcomm.deploy", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("multi-node")
    _common(p)
    _bench(p)
    p = sub.add_parser("multi-initiator")
    _common(p)
    _bench(p)
    p.add_argument("--jobs", default="jobs.txt")
    p = sub.add_parser("check")
    _common(p)
    p = sub.add_parser("install")
    _common(p)
    p.add_argument("--wheel", required=True)
    p = sub.add_parser("cleanup")
    _common(p)
    p = sub.add_parser("monitor")
    p.add_argument("--interval", type=float, default=1.0)
    p.add_argument("--count", type=int, default=0, help="records to print (0 = until Ctrl-C)")
    p.add_argument("--device", action="append", default=[], help="RDMA device(s) to watch (default: all)")
    p.add_argument("--no-gpu", action="store_true", help="skip NVML PCIe counters")
    p.add_argument("--sysfs-root", default="/")
    sub.add_parser("profiles")
    p = sub.add_parser("tool-path")
    p.add_argument("name")
    a = ap.parse_args(argv)

    if a.cmd == "tool-path":
        import mpcomm
        print(mpcomm.tool_path(a.name))
        return 0
    if a.cmd == "profiles":
        for name, env in sorted(PROFILES.items()):
            print(f"{name}: " + " ".join(f"{k}={v}" for k, v in sorted(env.items())))
        return 0
    if a.cmd == "monitor":
        M.monitor(a.interval, a.count, a.sysfs_root, a.device or None, not a.no_gpu,
                  emit=lambda r: print(json.dumps(r), flush=True))
        return 0

    hosts = H.load_hosts(a.hosts)
    runner = Runner(a.ssh_user, a.ssh_option, local=a.local, dry_run=a.dry_run,
                    echo=lambda s: print(s, file=sys.stderr))
    if a.cmd == "multi-node":
        res = O.multi_node(hosts, a, runner)
    elif a.cmd == "multi-initiator":
        res = O.multi_initiator(hosts, H.load_jobs(a.jobs, hosts), a, runner)
    elif a.cmd == "check":
        res = O.check(hosts, a, runner)
    elif a.cmd == "install":
        res = O.install(hosts, a, runner)
    else:
        if not a.run_id:
            ap.error("cleanup needs --run-id")
        res = O.cleanup(hosts, a, runner)
    print(json.dumps(res), flush=True)
    return 0 if (res.get("ok") or a.dry_run) else 1


if __name__ == "__main__":
    sys.exit(main())
