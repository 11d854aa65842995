"""Run watchdog: decide what to do when a training run stops or misbehaves.

The watchdog polls the run (its process state, the tail of its log, host memory, the
time since the last step line) and returns an action:

  * CUDA out of memory      -> cut MB_TOKENS by 10% in the live env file and resume
                               (at most 3 times)
  * NaN / inf in step stats -> resume once from the last recover checkpoint
  * host memory over limit  -> cut MB_TOKENS and resume (at most 5 times)
  * crash / dead server / no step line for STALL_S seconds -> stop and resume
                               (at most 5 times)
  * a traceback inside octopus_b200 code -> NEEDS-MAIN: stop, a human must look
  * otherwise               -> continue

The policy (`decide`) is pure and testable; `Watchdog.step` gathers the facts, applies
the micro-batch cut to the live env file and returns the action.  `supervise` (the
command line below) is the launcher: it runs the training command in its own process
group with OCTOPUS_LIVE_ENV pointing at the live env file (the trainer re-reads it every
step and resumes from its recover checkpoint on restart), polls, and stops / restarts it
as decided:

    python -m octopus_b200.rl.watchdog --log run.log --live-env live.env [--poll 60] -- \
        python -m octopus_b200.rl.train --config grpo.yaml ...

Reference parity (behaviour): `scripts/rl_env/rl_watchdog.sh:1-80`.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import signal
import subprocess
import sys
import time
from dataclasses import dataclass, field

STALL_S = 7200
LIMITS = {"oom": 3, "nan": 1, "hostmem": 5, "crash": 5}


@dataclass
class Facts:
    running: bool
    exit_code: int | None = None
    log_tail: str = ""
    last_step_t: float | None = None
    now: float = field(default_factory=time.time)
    host_mem_frac: float = 0.0


@dataclass
class Decision:
    action: str            # continue | resume | stop | needs_main
    reason: str = ""
    mb_tokens_factor: float = 1.0


OOM = re.compile(r"CUDA out of memory|OutOfMemoryError|OutOfKV")
NAN = re.compile(r"\b(nan|inf)\b.*(loss|grad_norm)|(loss|grad_norm)[^\n]*\b(nan|inf)\b", re.I)
OWN_TRACE = re.compile(r'File "[^"]*octopus_b200/[^"]*", line \d+')


def decide(f: Facts, counts: dict, host_mem_limit: float = 0.92, stall_s: float = STALL_S) -> Decision:
    tail = f.log_tail[-20000:]
    if not f.running:
        if OOM.search(tail):
            kind = "oom"
            if counts.get(kind, 0) >= LIMITS[kind]:
                return Decision("stop", "out of memory too often")
            return Decision("resume", "out of memory", 0.9)
        if "Traceback" in tail and OWN_TRACE.search(tail) and not OOM.search(tail):
            return Decision("needs_main", "traceback in octopus_b200 code")
        if f.exit_code == 0:
            return Decision("stop", "finished")
        kind = "crash"
        if counts.get(kind, 0) >= LIMITS[kind]:
            return Decision("stop", "crashed too often")
        return Decision("resume", f"exited with {f.exit_code}")
    if NAN.search(tail.splitlines()[-1] if tail.strip() else ""):
        if counts.get("nan", 0) >= LIMITS["nan"]:
            return Decision("stop", "non-finite step stats again")
        return Decision("resume", "non-finite step stats")
    if f.host_mem_frac > host_mem_limit:
        if counts.get("hostmem", 0) >= LIMITS["hostmem"]:
            return Decision("stop", "host memory limit hit too often")
        return Decision("resume", "host memory over limit", 0.9)
    if f.last_step_t is not None and f.now - f.last_step_t > stall_s:
        if counts.get("crash", 0) >= LIMITS["crash"]:
            return Decision("stop", "stalled too often")
        return Decision("resume", f"no step for {int(f.now - f.last_step_t)} s")
    return Decision("continue")


def cut_mb_tokens(live_env_path: str, factor: float, default: int = 262144) -> int:
    """Multiply MB_TOKENS in the live env file by `factor` (creating the line if absent)."""
    lines, cur = [], default
    if os.path.exists(live_env_path):
        for line in open(live_env_path):
            if line.strip().startswith("MB_TOKENS="):
                try:
                    cur = int(line.split("=", 1)[1])
                except ValueError:
                    pass
                continue
            lines.append(line.rstrip("\n"))
    new = max(1024, int(cur * factor) // 1024 * 1024)
    lines.append(f"MB_TOKENS={new}")
    tmp = live_env_path + ".tmp"
    with open(tmp, "w") as f:
        f.write("\n".join(lines) + "\n")
    os.replace(tmp, live_env_path)
    return new


class Watchdog:
    def __init__(self, log_path: str, live_env_path: str | None = None, stall_s: float = STALL_S):
        self.log_path = log_path
        self.live_env_path = live_env_path
        self.stall_s = stall_s
        self.counts: dict[str, int] = {}
        self.offset = 0  # log bytes written before the current run of the command (ignored)

    def mark_restart(self):
        """Ignore what earlier runs wrote to the log (the next facts read only the new run)."""
        self.offset = os.path.getsize(self.log_path) if os.path.exists(self.log_path) else 0

    def facts(self, running: bool, exit_code: int | None = None) -> Facts:
        tail = ""
        last = None
        if os.path.exists(self.log_path):
            with open(self.log_path, "rb") as f:
                f.seek(0, 2)
                n = f.tell()
                f.seek(max(self.offset, n - 65536))
                tail = f.read().decode("utf-8", "replace")
            last = os.path.getmtime(self.log_path)
        mem = 0.0
        try:
            import psutil

            mem = psutil.virtual_memory().percent / 100.0
        except Exception:
            pass
        return Facts(running, exit_code, tail, last, time.time(), mem)

    def step(self, running: bool, exit_code: int | None = None) -> Decision:
        d = decide(self.facts(running, exit_code), self.counts, stall_s=self.stall_s)
        if d.action == "resume":
            kind = ("oom" if "memory" in d.reason and "host" not in d.reason else "hostmem" if "host" in d.reason
                    else "nan" if "non-finite" in d.reason else "crash")
            self.counts[kind] = self.counts.get(kind, 0) + 1
            if d.mb_tokens_factor != 1.0 and self.live_env_path:
                cut_mb_tokens(self.live_env_path, d.mb_tokens_factor)
        return d


def _stop_group(proc, grace_s: float = 30.0) -> int:
    """SIGTERM the child's process group, SIGKILL it after `grace_s`; returns its exit code."""
    if proc.poll() is None:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=grace_s)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
            proc.wait()
        except ProcessLookupError:
            pass
    return proc.returncode


EXIT_CODES = {"finished": 0, "needs_main": 2}


def supervise(cmd: list[str], log_path: str, live_env: str, poll_s: float = 60.0, stall_s: float = STALL_S,
              sleep=time.sleep, report=print) -> int:
    """Run `cmd` under the watchdog until it finishes or the policy gives up.
    Returns 0 when the run finished, 2 when a traceback in this package needs a person,
    1 when it stopped for another reason."""
    wd = Watchdog(log_path, live_env, stall_s)
    env = dict(os.environ, OCTOPUS_LIVE_ENV=os.path.abspath(live_env))

    def launch():
        wd.mark_restart()
        with open(log_path, "ab") as log:
            return subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=env, start_new_session=True)

    proc, restarts = launch(), 0
    while True:
        sleep(poll_s)
        code = proc.poll()
        d = wd.step(code is None, code)
        if d.action == "continue":
            continue
        if code is None:
            code = _stop_group(proc)
        report(json.dumps({"t": round(time.time(), 1), "action": d.action, "reason": d.reason, "exit_code": code,
                           "restarts": restarts, "counts": wd.counts}))
        if d.action == "resume":
            restarts += 1
            proc = launch()
            continue
        if d.action == "needs_main":
            return EXIT_CODES["needs_main"]
        return EXIT_CODES["finished"] if d.reason == "finished" else 1


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" not in argv:
        raise SystemExit("usage: python -m octopus_b200.rl.watchdog --log LOG --live-env FILE [--poll S] -- CMD ...")
    k = argv.index("--")
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.rl.watchdog")
    ap.add_argument("--log", required=True, help="the run's log file (the child's stdout / stderr go here)")
    ap.add_argument("--live-env", required=True, help="live env file (MB_TOKENS=...) the trainer re-reads")
    ap.add_argument("--poll", type=float, default=60.0)
    ap.add_argument("--stall", type=float, default=STALL_S, help="seconds without a log write that count as a stall")
    args = ap.parse_args(argv[:k])
    return supervise(argv[k + 1:], args.log, args.live_env, args.poll, args.stall)


if __name__ == "__main__":
    sys.exit(main())
