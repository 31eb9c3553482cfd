"""Multi-host orchestration: hosts.txt / jobs.txt parsing, SSH or local
runners, environment profiles, multi-node and multi-initiator runs of the
scatter_test tool, install/check/cleanup, and a link throughput monitor.
Entry point: ``python -m mpcomm.deploy``."""
from mpcomm.deploy.hosts import Host, HostRef, HostsError, Job, load_hosts, load_jobs, parse_hosts, parse_jobs  # noqa: F401
from mpcomm.deploy.profiles import PROFILES, exports, profile_env  # noqa: F401
from mpcomm.deploy.runner import Runner  # noqa: F401
