"""Run launcher: start / stop / status of a training trial, serve / unserve of a rollout
server, and a settings-only run folder.

    python -m octopus_b200.launch start [--trial NAME] [--gpus N] [--config grpo.yaml] [-- key=value ...]
    python -m octopus_b200.launch stop [--trial NAME]
    python -m octopus_b200.launch status [--trial NAME]
    python -m octopus_b200.launch serve [--name NAME] [--port 30200] [-- server arguments ...]
    python -m octopus_b200.launch unserve [--name NAME]
    python -m octopus_b200.launch settings OUT_DIR [key=value ...]

Every trial is a folder under $OCTOPUS_ROOT (default ./runs): `start` of a new trial
creates it with a live env file (KEY=VALUE lines the trainer re-reads every step, e.g.
MB_TOKENS) and launches the trainer under the watchdog (rl.watchdog: restarts after OOM /
crash / stall, cutting MB_TOKENS on memory errors) in a process group of its own, with
torchrun when --gpus > 1; `start` of an existing trial resumes it from its recover
checkpoint.  `stop` ends the trial's process group, `status` shows whether it runs, its
last step line and its live settings.  `serve` / `unserve` do the same for an HTTP rollout
server (serving.server).  `settings` writes a run folder's config and episode settings
without training (for evaluations that need the run's switches).

Reference parity (behaviour): `scripts/rl_env/rl_run.sh` (serve / start / stop / status /
settings, trials under a root, resume after stop) and `scripts/rl_env/rl_watchdog.sh`.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time
from pathlib import Path

ROOT_ENV = "OCTOPUS_ROOT"


def root() -> Path:
    return Path(os.environ.get(ROOT_ENV, "runs")).resolve()


def _alive(pid: int) -> bool:
    """True while process `pid` runs (an exited child of this process is reaped first; a
    zombie counts as ended)."""
    try:
        done, _ = os.waitpid(pid, os.WNOHANG)
        if done == pid:
            return False
    except ChildProcessError:
        pass
    try:
        os.kill(pid, 0)
    except (ProcessLookupError, PermissionError):
        return False
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().rsplit(")", 1)[1].split()[0] != "Z"
    except OSError:
        return True


def _read_pid(path: Path) -> int | None:
    try:
        pid = int(path.read_text().strip())
    except (OSError, ValueError):
        return None
    return pid if _alive(pid) else None


def _stop_group(pid: int, grace_s: float = 30.0) -> bool:
    try:
        os.killpg(pid, signal.SIGTERM)
    except ProcessLookupError:
        return False
    t0 = time.time()
    while time.time() - t0 < grace_s and _alive(pid):
        time.sleep(0.2)
    if _alive(pid):
        try:
            os.killpg(pid, signal.SIGKILL)
        except ProcessLookupError:
            pass
    return True


def _latest_trial() -> str | None:
    trials = sorted((p for p in root().glob("*") if (p / "trial.json").is_file()),
                    key=lambda p: p.stat().st_mtime)
    return trials[-1].name if trials else None


def trial_command(args, trial_dir: Path) -> list[str]:
    """The watchdog-supervised trainer command of a trial (torchrun for several GPUs)."""
    py = sys.executable
    opts = [x for x in args.overrides if x.startswith("--")]  # trainer options first, then key=value overrides
    train_args = ["--config", args.config, *opts, f"checkpoint.dir={trial_dir}", f"trial_name={trial_dir.name}",
                  *[x for x in args.overrides if not x.startswith("--")]]
    if args.gpus > 1:
        train = [py, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}", "--master-addr",
                 "127.0.0.1", "--master-port", str(args.port), "-m", "octopus_b200.rl.train", *train_args]
    else:
        train = [py, "-m", "octopus_b200.rl.train", *train_args]
    return [py, "-m", "octopus_b200.rl.watchdog", "--log", str(trial_dir / "train.log"), "--live-env",
            str(trial_dir / "live.env"), "--poll", str(args.poll), "--", *train]


def start(args) -> int:
    name = args.trial or time.strftime("trial-%m%d%H%M%S")
    d = root() / name
    pid = _read_pid(d / "pid")
    if pid is not None:
        print(f"trial {name} already runs (pid {pid})")
        return 1
    d.mkdir(parents=True, exist_ok=True)
    live = d / "live.env"
    if not live.exists():
        live.write_text(f"MB_TOKENS={args.mb_tokens}\n")
    meta = d / "trial.json"
    info = json.loads(meta.read_text()) if meta.exists() else {"created": time.time(), "starts": 0}
    cmd = trial_command(args, d)
    info.update(starts=info["starts"] + 1, last_start=time.time(), command=cmd, gpus=args.gpus)
    meta.write_text(json.dumps(info, indent=1))
    with open(d / "launcher.log", "ab") as log:
        proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, start_new_session=True, cwd=os.getcwd())
    (d / "pid").write_text(str(proc.pid))
    print(json.dumps({"trial": name, "pid": proc.pid, "dir": str(d), "resume": info["starts"] > 1}))
    return 0


def stop(args) -> int:
    name = args.trial or _latest_trial()
    if name is None:
        print("no trial")
        return 1
    d = root() / name
    pid = _read_pid(d / "pid")
    if pid is None:
        print(f"trial {name} is not running")
        return 0
    _stop_group(pid)
    print(json.dumps({"trial": name, "stopped": pid}))
    return 0


def status(args) -> int:
    name = args.trial or _latest_trial()
    if name is None:
        print("no trial")
        return 1
    d = root() / name
    pid = _read_pid(d / "pid")
    last = None
    for f in (d / name / "steps.jsonl", *d.glob("**/steps.jsonl")):
        if f.is_file():
            lines = [x for x in f.read_text().splitlines() if x.strip()]
            last = json.loads(lines[-1]) if lines else None
            break
    live = dict(x.split("=", 1) for x in (d / "live.env").read_text().split() if "=" in x) \
        if (d / "live.env").exists() else {}
    print(json.dumps({"trial": name, "running": pid is not None, "pid": pid, "last_step": last, "live": live}))
    return 0


def serve(args) -> int:
    d = root() / "serve"
    d.mkdir(parents=True, exist_ok=True)
    pidf = d / f"{args.name}.pid"
    if _read_pid(pidf) is not None:
        print(f"server {args.name} already runs")
        return 1
    cmd = [sys.executable, "-m", "octopus_b200.serving.server", "--port", str(args.port), *args.overrides]
    with open(d / f"{args.name}.log", "ab") as log:
        proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
    pidf.write_text(str(proc.pid))
    print(json.dumps({"server": args.name, "pid": proc.pid, "port": args.port}))
    return 0


def unserve(args) -> int:
    pid = _read_pid(root() / "serve" / f"{args.name}.pid")
    if pid is None:
        print(f"server {args.name} is not running")
        return 0
    _stop_group(pid)
    print(json.dumps({"server": args.name, "stopped": pid}))
    return 0


def settings(args) -> int:
    from .rl import config as C

    cfg = C.load(args.config, args.overrides)
    C.set_derived_settings(cfg)
    out = Path(args.out_dir)
    out.mkdir(parents=True, exist_ok=True)
    C.save_settings(str(out / "episode_settings.json"))
    (out / "config.json").write_text(json.dumps(cfg.to_dict(), indent=1))
    print(json.dumps({"run_dir": str(out)}))
    return 0


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    extra: list[str] = []
    if "--" in argv:
        k = argv.index("--")
        argv, extra = argv[:k], argv[k + 1:]
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.launch")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("start")
    s.add_argument("--trial", default="")
    s.add_argument("--gpus", type=int, default=1)
    s.add_argument("--config", default=str(Path(__file__).with_name("rl") / "grpo.yaml"))
    s.add_argument("--mb-tokens", type=int, default=262144)
    s.add_argument("--poll", type=float, default=60.0)
    s.add_argument("--port", type=int, default=29500, help="torchrun master port (--gpus > 1)")
    for name in ("stop", "status"):
        p = sub.add_parser(name)
        p.add_argument("--trial", default="")
    sv = sub.add_parser("serve")
    sv.add_argument("--name", default="server0")
    sv.add_argument("--port", type=int, default=30200)
    us = sub.add_parser("unserve")
    us.add_argument("--name", default="server0")
    st = sub.add_parser("settings")
    st.add_argument("out_dir")
    st.add_argument("--config", default=None)
    st.add_argument("overrides", nargs="*")
    args = ap.parse_args(argv)
    if args.cmd != "settings":
        args.overrides = extra
    else:
        args.overrides = list(args.overrides) + extra
    return {"start": start, "stop": stop, "status": status, "serve": serve, "unserve": unserve,
            "settings": settings}[args.cmd](args)


if __name__ == "__main__":
    raise SystemExit(main())
