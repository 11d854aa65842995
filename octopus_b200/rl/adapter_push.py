"""Push a weight-update directory (an adapter version, or HF weights) to remote rollout
hosts: tar over ssh, with retries when ssh itself fails (exit 255: connection reset,
host briefly unreachable); other failures raise at once.

Reference parity (behaviour): `octopus/rl/adapter_push.py:17-41`.
"""
from __future__ import annotations

import shlex
import subprocess
import time


class PushError(RuntimeError):
    pass


def push_adapter(src: str, hosts: list[str], dest: str, ssh=("ssh", "-o", "BatchMode=yes"), retries: int = 3,
                 delay: float = 2.0, sleep=time.sleep) -> dict:
    """Copy the contents of `src` into `dest` on every host; returns {host: attempts}."""
    out = {}
    for host in hosts:
        remote = f"mkdir -p {shlex.quote(dest)} && tar -C {shlex.quote(dest)} -xf -"
        for attempt in range(1, retries + 1):
            tar = subprocess.Popen(["tar", "-C", src, "-cf", "-", "."], stdout=subprocess.PIPE)
            rc = subprocess.run([*ssh, host, remote], stdin=tar.stdout).returncode
            tar.stdout.close()
            trc = tar.wait()
            if trc != 0:
                raise PushError(f"tar of {src} failed with {trc}")
            if rc == 0:
                out[host] = attempt
                break
            if rc != 255 or attempt == retries:
                raise PushError(f"push to {host} failed with exit {rc} after {attempt} attempt(s)")
            sleep(delay * attempt)
    return out
