"""SWE workspace: a git repository the agent edits and tests, with per-branch copies.

Tools: view, edit (exact-match replace), write, shell, test, reproduce (a hypothesis and a
Python reproducer, kept per thread) / rerun_reproduction, done (main), commit / abort
(branches).  Every branch (fork) works in its own copy of its parent's tree; a branch
that commits hands back its patch (git diff against the copy's base), which the parent
applies with a 3-way merge when the fork joins.  snapshot / restore (rewinds) use
`git stash create` (the working tree as a commit object) and a hard reset.

Commands run through an executor (local process, udocker or Singularity) with a time
limit, their own process group, the nokill guard and no network egress.

Reference parity (behaviour): `octopus/envs/swe/agent.py:188-560` (HarborWorkspace: per-
branch copies, stash snapshots, patch capture / 3-way apply, close gate),
`octopus/envs/swe/container_tools.py:140-197`, `octopus/envs/swe/prompt.py`.
"""
from __future__ import annotations

import json
import os
import shlex
import shutil
import subprocess
import sys
import tempfile

from ...runtime.core import DONE_TOOL, _tool
from ...runtime.tree import WorkspaceProvider
from .containers import LocalExec

VIEW = _tool("view", "Show a file (optionally lines start..end, 1-based).",
             {"path": {"type": "string"}, "start": {"type": "integer"}, "end": {"type": "integer"}}, ["path"])
EDIT = _tool("edit", "Replace exactly one occurrence of old with new in a file.",
             {"path": {"type": "string"}, "old": {"type": "string"}, "new": {"type": "string"}},
             ["path", "old", "new"])
WRITE = _tool("write", "Write a whole file.", {"path": {"type": "string"}, "content": {"type": "string"}},
              ["path", "content"])
SHELL = _tool("shell", "Run a shell command in the repository.", {"cmd": {"type": "string"}}, ["cmd"])
TEST = _tool("test", "Run the task's tests.", {}, [])
REPRODUCE = _tool("reproduce", "State a hypothesis about the bug and run Python code that reproduces it.",
                  {"hypothesis": {"type": "string"}, "code": {"type": "string"}}, ["hypothesis", "code"])
RERUN = _tool("rerun_reproduction", "Run the last reproducer again (after a change).", {}, [])
COMMIT = _tool("commit", "Finish this branch and hand its changes to the parent.",
               {"summary": {"type": "string"}}, ["summary"])
ABORT = _tool("abort", "Finish this branch without changes.", {"reason": {"type": "string"}}, ["reason"])

SYSTEM = ("You fix a software repository. Inspect files with view, change them with edit or write, run commands "
          "with shell and the task's tests with test. Fork branches for independent sub-tasks; a branch ends "
          "with commit (its changes merge into its parent) or abort. End the main thread with done.")


def _git(args, cwd, check=True, inp: bytes | None = None) -> subprocess.CompletedProcess:
    return subprocess.run(["git", *args], cwd=cwd, check=check, input=inp, capture_output=True)


class GitWorkspace(WorkspaceProvider):
    report = "what you changed and whether the tests pass"

    def __init__(self, repo: str, test_cmd: str, executor=None, timeout: float = 120.0, max_output: int = 8000,
                 python: str | None = None):
        self.root = repo
        self.test_cmd = test_cmd
        self.exec = executor or LocalExec()
        # the interpreter reproducers run with (in a container: the image's python3)
        self.python = python or (sys.executable if type(self.exec) is LocalExec else "python3")
        self.repro: dict[str, dict] = {}  # thread -> {"hypothesis", "code"} (a fork inherits its parent's)
        self.timeout, self.max_output = timeout, max_output
        self.dirs = {"main": repo}
        self.base = {"main": _git(["rev-parse", "HEAD"], repo).stdout.decode().strip()}
        self.tmp = tempfile.mkdtemp(prefix="octo-swe-")
        self.results: dict[str, dict] = {}

    # ------------------------------------------------------------------ runtime hooks
    def system_prompt(self, task: str) -> str:
        return SYSTEM

    def tools(self):
        return [VIEW, EDIT, WRITE, SHELL, TEST, REPRODUCE, RERUN, DONE_TOOL, COMMIT, ABORT]

    def _dir(self, thread: str) -> str:
        return self.dirs.get(thread, self.root)

    def _path(self, thread: str, path: str) -> str:
        d = os.path.realpath(self._dir(thread))
        p = os.path.realpath(os.path.join(d, path))
        if not (p == d or p.startswith(d + os.sep)):
            raise ValueError("path outside the repository")
        return p

    def _clip(self, s: str) -> str:
        return s if len(s) <= self.max_output else s[: self.max_output // 2] + "\n...\n" + s[-self.max_output // 2:]

    async def dispatch(self, name, args, thread):
        try:
            if name == "view":
                with open(self._path(thread, args["path"]), errors="replace") as f:
                    lines = f.read().splitlines()
                a = max(1, int(args.get("start") or 1))
                b = int(args.get("end") or len(lines))
                return self._clip("\n".join(f"{i}\t{lines[i - 1]}" for i in range(a, min(b, len(lines)) + 1))), False
            if name == "edit":
                p = self._path(thread, args["path"])
                text = open(p).read()
                n = text.count(args["old"])
                if n != 1:
                    return f"edit failed: old text found {n} times (must be exactly once)", False
                with open(p, "w") as f:
                    f.write(text.replace(args["old"], args["new"], 1))
                return "edited", False
            if name == "write":
                p = self._path(thread, args["path"])
                os.makedirs(os.path.dirname(p), exist_ok=True)
                with open(p, "w") as f:
                    f.write(args["content"])
                return f"wrote {args['path']}", False
            if name == "shell":
                r = self.exec.run(args["cmd"], self._dir(thread), self.timeout)
                tag = " (timed out)" if r.timed_out else ""
                return self._clip(f"exit {r.code}{tag}\n{r.output}"), False
            if name == "test":
                r = self.exec.run(self.test_cmd, self._dir(thread), self.timeout)
                return self._clip(f"tests {'passed' if r.code == 0 else 'failed'} (exit {r.code})\n{r.output}"), False
            if name in ("reproduce", "rerun_reproduction"):
                if name == "reproduce":
                    code, hyp = args.get("code"), args.get("hypothesis")
                    if not (isinstance(code, str) and code.strip() and isinstance(hyp, str) and hyp.strip()):
                        return "reproduce needs hypothesis and code", False
                    self.repro[thread] = {"hypothesis": hyp, "code": code}
                rep = self.repro.get(thread)
                if not rep:
                    return "Define and execute a reproducer first.", False
                r = self.exec.run(f"{self.python} -c {shlex.quote(rep['code'])}", self._dir(thread), self.timeout)
                tag = " (timed out)" if r.timed_out else ""
                return self._clip(f"exit {r.code}{tag}\n{r.output}"), False
            if name == "done":
                return f"done: {args.get('answer', '')}", True
            if name == "commit":
                return f"commit: {args.get('summary', '')}", True
            if name == "abort":
                return f"abort: {args.get('reason', '')}", True
        except (OSError, ValueError, KeyError) as e:
            return f"{name} failed: {e}", False
        return f"unknown tool {name}", False

    async def copy(self, parent: str, child: str) -> None:
        src = self._dir(parent)
        dst = os.path.join(self.tmp, child.replace("/", "-"))
        shutil.copytree(src, dst, symlinks=True)
        # the branch's base is its parent's working tree at the fork
        _git(["add", "-A"], dst)
        _git(["-c", "user.name=octopus", "-c", "user.email=octopus@localhost", "commit", "-q", "--allow-empty", "-m",
              f"fork {child}"], dst)
        self.dirs[child] = dst
        self.base[child] = _git(["rev-parse", "HEAD"], dst).stdout.decode().strip()
        if parent in self.repro:
            self.repro[child] = dict(self.repro[parent])

    async def snapshot(self, thread: str):
        d = self._dir(thread)
        _git(["add", "-A"], d)
        h = _git(["stash", "create"], d).stdout.decode().strip()
        return h or "HEAD"

    async def restore(self, thread: str, snap) -> None:
        d = self._dir(thread)
        _git(["reset", "-q", "--hard"], d)
        _git(["clean", "-qfd"], d)
        if snap and snap != "HEAD":
            _git(["stash", "apply", "-q", snap], d)

    async def capture(self, thread: str) -> dict:
        d = self._dir(thread)
        _git(["add", "-A"], d)
        patch = _git(["diff", "--cached", "--binary", self.base.get(thread, "HEAD")], d).stdout
        stat = _git(["diff", "--cached", "--stat", self.base.get(thread, "HEAD")], d).stdout.decode()
        r = self.exec.run(self.test_cmd, d, self.timeout)
        out = {"patch": patch.decode("utf-8", "replace"), "diffstat": stat.strip(), "passed": r.code == 0}
        self.results[thread] = out
        return out

    async def apply(self, thread: str, results: list[dict]) -> str:
        """Merge committed branches' patches into `thread`'s tree (3-way); a summary line each."""
        d = self._dir(thread)
        lines = []
        for res in results:
            # a runtime branch record carries capture()'s output under "result"
            patch = res.get("patch") or (res.get("result") or {}).get("patch")
            if res.get("ended_with") != "commit" or not patch:
                continue
            r = _git(["apply", "--3way", "--whitespace=nowarn", "-"], d, check=False, inp=patch.encode())
            status = "merged" if r.returncode == 0 else "conflict"
            res["merge"] = status
            lines.append(f"{res.get('branch') or res.get('thread', '?')}: {status}")
        return "\n".join(lines)

    async def close(self) -> None:
        if getattr(self, "defer_close", False):  # kept for grading; discard() removes them
            return
        self.discard()

    def discard(self) -> None:
        """Remove the branch copies (and a prepared task's copy of the repository)."""
        shutil.rmtree(self.tmp, ignore_errors=True)
        d = getattr(self, "task_dir", None)
        if d:
            shutil.rmtree(d, ignore_errors=True)

    def state(self) -> dict:
        return {"dirs": self.dirs, "results": {k: {kk: v for kk, v in r.items() if kk != "patch"}
                                                for k, r in self.results.items()}}

    def dumps(self) -> str:
        return json.dumps(self.state())
