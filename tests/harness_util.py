"""Starts harness targets as child processes for the harness tests."""
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def harness_env(**extra):
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), MPCOMM_LOG_LEVEL="1")
    env.update(extra)
    return env


class TargetProc:
    def __init__(self, tmp_path, host_id, env, *extra):
        self.ready = tmp_path / f"ready-{host_id.replace(':', '_')}"
        self.log = open(tmp_path / f"target-{host_id.replace(':', '_')}.log", "w")
        self.proc = subprocess.Popen([sys.executable, "-m", "mpcomm.harness.target", "--host-id", host_id,
                                      "--tcp-port", "0", "--ready-file", str(self.ready), "--duration", "120",
                                      *extra], stdout=self.log, stderr=subprocess.STDOUT, env=env, cwd=ROOT)
        deadline = time.time() + 90
        while not self.ready.exists():
            if self.proc.poll() is not None or time.time() > deadline:
                self.stop()
                raise RuntimeError(f"target {host_id} did not come up: "
                                   f"{open(self.log.name).read()[-2000:]}")
            time.sleep(0.1)
        self.port = int(self.ready.read_text())

    def stop(self):
        if self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(20)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
        self.log.close()
        return self.proc.returncode


def run_initiator(env, *args, timeout=180):
    return subprocess.run([sys.executable, "-m", "mpcomm.harness.initiator", *args], capture_output=True,
                          text=True, env=env, cwd=ROOT, timeout=timeout)
