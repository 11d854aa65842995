"""Episode switches (``OCTOPUS_*`` environment variables), read where used, no state.

The names are the public switch API shared with the reference (`octopus/runtime/
settings.py:10-144`); each reader documents its default.
"""
from __future__ import annotations

import json
import math
import os


def _int(name: str, default: int = 0) -> int:
    v = os.environ.get(name, "").strip()
    return int(v) if v else default


def _flag(name: str, default: str = "") -> bool:
    return os.environ.get(name, default).strip() == "1"


def branch_fix() -> bool:
    """OCTOPUS_STRATEGY=branch_fix: each branch is one complete fix attempt."""
    return os.environ.get("OCTOPUS_STRATEGY", "").strip() == "branch_fix"


def plan_episode() -> bool:
    """OCTOPUS_PLAN_EPISODE=1: export the fork tree and controls for the verifier."""
    return bool(os.environ.get("OCTOPUS_PLAN_EPISODE"))


def cursor_mode() -> bool:
    """OCTOPUS_CURSOR=1: requests send only the messages after the last reply's cursor."""
    return _flag("OCTOPUS_CURSOR")


def bundle() -> bool:
    """OCTOPUS_BUNDLE=1: the task is a bundle of several problems in one tree."""
    return bool(os.environ.get("OCTOPUS_BUNDLE"))


def auto_merge() -> bool:
    """OCTOPUS_AUTO_MERGE (default 1 in bundle mode): apply committed branch results at each join."""
    return os.environ.get("OCTOPUS_AUTO_MERGE", "1" if bundle() else "0") == "1"


def call_limit() -> int | None:
    """OCTOPUS_MAIN_MAX_CALLS: main's call cap (None: unset)."""
    v = os.environ.get("OCTOPUS_MAIN_MAX_CALLS", "").strip()
    return int(v) if v else None


def branch_turns() -> int:
    """OCTOPUS_BRANCH_MAX_TURNS: a branch's turn cap (default 100)."""
    return _int("OCTOPUS_BRANCH_MAX_TURNS", 100)


def rewind_tool() -> bool:
    """OCTOPUS_REWIND_TOOL=1: every thread may call rewind(to_step, note)."""
    return _flag("OCTOPUS_REWIND_TOOL")


def rewind_max() -> int:
    """OCTOPUS_REWIND_MAX: rewinds per thread (0: no cap)."""
    return _int("OCTOPUS_REWIND_MAX", 0)


def rewind_rule() -> int:
    """OCTOPUS_REWIND: automatic rewinds after repeated failures (0: off)."""
    return _int("OCTOPUS_REWIND", 0)


def thinking() -> bool:
    """OCTOPUS_CHAT_TEMPLATE_KWARGS with enable_thinking not false: notes go as tool results."""
    kw = os.environ.get("OCTOPUS_CHAT_TEMPLATE_KWARGS", "").strip()
    return bool(kw) and json.loads(kw).get("enable_thinking") is not False


def thread_budget() -> int:
    """OCTOPUS_THREAD_BUDGET: a thread's growth cap after its first request (default 32768)."""
    return _int("OCTOPUS_THREAD_BUDGET", 0) or 32_768


def max_reply() -> int:
    """OCTOPUS_MAX_TOKENS: one reply's cap (default 32768)."""
    return _int("OCTOPUS_MAX_TOKENS", 32_768)


def context_window() -> int:
    """OCTOPUS_CONTEXT_WINDOW: the serving context window (default 262144)."""
    return _int("OCTOPUS_CONTEXT_WINDOW", 0) or 262_144


def window_room(context: int) -> int:
    """Tokens a thread holding `context` tokens may still add with one reply left in the window."""
    return context_window() - context - max_reply()


def answer_reserve() -> int:
    """OCTOPUS_ANSWER_RESERVE: tokens of the growth cap kept for the closing call (0: off).

    Clipping counts tokens with the policy's tokenizer (OCTOPUS_TOKENIZER) when it is set,
    else with a 4-characters-per-token estimate.
    """
    return _int("OCTOPUS_ANSWER_RESERVE", 0)


def read_tool() -> bool:
    """OCTOPUS_READ_TOOL=1: threads may read (mount) other threads' steps."""
    return _flag("OCTOPUS_READ_TOOL")


def read_event() -> bool:
    """OCTOPUS_READ_EVENT=1: a sibling's conflicting edit triggers an automatic read."""
    return _flag("OCTOPUS_READ_EVENT")


def conflict_by() -> bool:
    """OCTOPUS_CONFLICT_BY=1: label join conflicts by cause."""
    return _flag("OCTOPUS_CONFLICT_BY")


def plan_control() -> bool:
    """OCTOPUS_PLAN_CONTROL=1: after a forking episode, a no-fork continuation of main from just
    before its first fork (the main-first control) is run and graded."""
    return bool(os.environ.get("OCTOPUS_PLAN_CONTROL"))


def read_control() -> bool:
    """OCTOPUS_READ_CONTROL=1: a read's no-mount counterfactual continuation is graded."""
    return _flag("OCTOPUS_READ_CONTROL")


def auto_fork() -> bool:
    """OCTOPUS_AUTO_FORK=1: the environment forks one branch per bundle task before main starts."""
    return _flag("OCTOPUS_AUTO_FORK")


def fork_depth() -> float:
    """OCTOPUS_FORK_DEPTH: threads fork while their depth is below it (default 2; 0: unlimited)."""
    return _int("OCTOPUS_FORK_DEPTH", 2) or math.inf


def max_threads() -> int:
    """OCTOPUS_MAX_THREADS: threads running at once (main + open branches), default 16."""
    return _int("OCTOPUS_MAX_THREADS", 16)


def max_branches() -> int | None:
    """OCTOPUS_MAX_BRANCHES: branches per episode at every depth (None: no cap)."""
    return _int("OCTOPUS_MAX_BRANCHES", 0) or None


def http_attempts() -> int:
    return _int("OCTOPUS_HTTP_ATTEMPTS", 6)


def http_timeout() -> int:
    return _int("OCTOPUS_HTTP_TIMEOUT", 180)


def tool_format_name() -> str:
    return os.environ.get("OCTOPUS_TOOL_FORMAT") or "qwen3_coder"


EPISODE_KEYS = (
    "OCTOPUS_STRATEGY", "OCTOPUS_CURSOR", "OCTOPUS_AUTO_MERGE", "OCTOPUS_MAIN_MAX_CALLS", "OCTOPUS_BRANCH_MAX_TURNS",
    "OCTOPUS_REWIND_TOOL", "OCTOPUS_REWIND_MAX", "OCTOPUS_REWIND", "OCTOPUS_CHAT_TEMPLATE_KWARGS",
    "OCTOPUS_THREAD_BUDGET", "OCTOPUS_MAX_TOKENS", "OCTOPUS_CONTEXT_WINDOW", "OCTOPUS_ANSWER_RESERVE",
    "OCTOPUS_READ_TOOL", "OCTOPUS_READ_EVENT", "OCTOPUS_CONFLICT_BY", "OCTOPUS_READ_CONTROL", "OCTOPUS_AUTO_FORK",
    "OCTOPUS_FORK_DEPTH", "OCTOPUS_MAX_THREADS", "OCTOPUS_MAX_BRANCHES", "OCTOPUS_TOOL_FORMAT",
    "OCTOPUS_MOUNT_LAYERS",
)


def episode_settings() -> dict:
    """The episode switches currently set (snapshotted into episode_settings.json)."""
    return {k: os.environ[k] for k in EPISODE_KEYS if k in os.environ}
