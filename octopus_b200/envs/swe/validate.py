"""Task validation without a model: a task measures a fix only when its hidden tests fail on
the prepared buggy tree (nop = 0) and pass once the reference fix is applied (oracle = 1).

    python -m octopus_b200.envs.swe.validate tasks.jsonl --out valid.jsonl [--report report.json]
        [--workers 8] [--timeout 120]

Each check prepares a fresh copy of the task's repository (branch setup as for an episode),
so the two runs share nothing.  The report lists nop, oracle and validity per task, with the
error text of a run that could not be prepared or patched.

Reference parity (behaviour): `octopus/envs/swe/data/validate_tasks.py` and `select_valid.py`
(nop = 0 and oracle = 1 select the tasks that measure a fix; fresh environment per check;
per-task report).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
from dataclasses import asdict


def _run(spec, executor, timeout: float, with_fix: bool) -> float:
    from .taskset import prepare_workspace, verify
    from .workspace import _git

    ws = prepare_workspace(spec, executor, timeout)
    try:
        if with_fix:
            r = _git(["apply", "--whitespace=nowarn", "-"], ws.root, check=False, inp=spec.fix_patch.encode())
            if r.returncode != 0:
                raise RuntimeError("reference fix does not apply: " + r.stderr.decode(errors="replace")[-300:])
        return verify(ws, spec)
    finally:
        ws.discard()


def validate_task(spec, executor=None, timeout: float = 120.0) -> dict:
    """{"task", "nop", "oracle", "valid", "error"?} of one task spec."""
    row = {"task": spec.instance_id, "nop": None, "oracle": None, "valid": False}
    try:
        if not spec.fix_patch:
            raise ValueError("no reference fix")
        row["nop"] = _run(spec, executor, timeout, False)
        row["oracle"] = _run(spec, executor, timeout, True)
        row["valid"] = row["nop"] == 0.0 and row["oracle"] == 1.0
    except Exception as e:  # noqa: BLE001  (a task that cannot be checked is invalid, with the reason)
        row["error"] = str(e)[:500]
    return row


def select_valid(specs, executor=None, timeout: float = 120.0, workers: int = 8) -> tuple[list, list[dict]]:
    """(valid specs in input order, per-task rows)."""
    with cf.ThreadPoolExecutor(max(1, workers)) as ex:
        rows = list(ex.map(lambda s: validate_task(s, executor, timeout), specs))
    return [s for s, r in zip(specs, rows) if r["valid"]], rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.envs.swe.validate")
    ap.add_argument("tasks")
    ap.add_argument("--out", required=True)
    ap.add_argument("--report", default="")
    ap.add_argument("--workers", type=int, default=8)
    ap.add_argument("--timeout", type=float, default=120.0)
    args = ap.parse_args(argv)
    from .containers import LocalExec
    from .taskset import load_rows, select_task_specs

    specs = select_task_specs(load_rows(args.tasks))
    valid, rows = select_valid(specs, LocalExec(sandbox=True), args.timeout, args.workers)
    with open(args.out, "w") as f:
        for s in valid:
            f.write(json.dumps(asdict(s)) + "\n")
    if args.report:
        with open(args.report, "w") as f:
            json.dump({r["task"]: r for r in rows}, f, indent=1)
    print(json.dumps({"tasks": len(specs), "valid": len(valid)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
