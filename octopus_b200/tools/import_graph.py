"""Package layering check of octopus_b200: which subpackage may import which.

    python -m octopus_b200.tools.import_graph [--show]     # exit 1 on a forbidden edge or a cycle

Layers (a package imports only packages of a strictly lower layer, or itself):

   0  utils, runtime             host helpers; the agent runtime stands alone
   1  ops                        kernels (the extension) and their CPU references
   2  models                     decoders over flat parameter buffers
   3  parallel.peer              IPC peer buffers
   4  parallel.tp                tensor-parallel groups and weights (used by the serving engine)
   5  serving                    engine, scheduler, chat, HTTP
   6  rl                         trainer, actor, credit, workflow
   7  parallel.fsdp, parallel.dp sharded / data-parallel actors (built on rl's actor)
   8  envs.*                     environments (never each other)
   9  eval                       evaluations
  10  tools                      probes and benches
  11  baselines                  reproductions of the reference's baselines (built on tools)

Every import counts, including imports inside functions.  Entry modules that wire the
layers together for a command line (ENTRY) may import any layer.  The package graph must
also be acyclic once entry modules are left out.
"""
from __future__ import annotations

import argparse
import ast
import sys
from collections import defaultdict
from pathlib import Path

PKG = "octopus_b200"
LAYER = {"utils": 0, "runtime": 0, "ops": 1, "models": 2, "parallel.peer": 3, "parallel.tp": 4, "serving": 5,
         "rl": 6, "parallel.fsdp": 7, "parallel.dp": 7, "envs.dag": 8, "envs.grpo": 8, "envs.search": 8,
         "envs.swe": 8, "eval": 9, "tools": 10, "baselines": 11}
ENTRY = {"octopus_b200.rl.train", "octopus_b200.launch"}


def package_of(module: str) -> str | None:
    parts = module.split(".")
    if parts[0] != PKG or len(parts) < 2:
        return None
    if parts[1] in ("envs", "parallel") and len(parts) > 2:
        name = f"{parts[1]}.{parts[2]}"
        return name if name in LAYER else None
    return parts[1] if parts[1] in LAYER else None


def module_name(root: Path, path: Path) -> str:
    rel = path.relative_to(root).with_suffix("")
    parts = list(rel.parts)
    if parts[-1] == "__init__":
        parts = parts[:-1]
    return ".".join(parts)


def imported(tree: ast.AST, module: str, is_pkg: bool) -> set[str]:
    out: set[str] = set()
    here = module.split(".") if is_pkg else module.split(".")[:-1]
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            out.update(a.name for a in node.names)
        elif isinstance(node, ast.ImportFrom):
            if node.level:
                base = here[: len(here) - (node.level - 1)]
                target = ".".join(base + ([node.module] if node.module else []))
            else:
                target = node.module or ""
            out.add(target)
            out.update(f"{target}.{a.name}" for a in node.names)
    return out


def edges(root: Path) -> dict[tuple[str, str], list[str]]:
    """(from package, to package) -> modules that make the edge."""
    found: dict[tuple[str, str], list[str]] = defaultdict(list)
    for path in sorted((root / PKG).rglob("*.py")):
        mod = module_name(root, path)
        src = package_of(mod)
        if src is None or mod in ENTRY:
            continue
        for target in imported(ast.parse(path.read_text()), mod, path.name == "__init__.py"):
            dst = package_of(target)
            if dst is not None and dst != src:
                found[(src, dst)].append(mod)
    return found


def problems(found: dict) -> list[str]:
    out = []
    for (a, b), mods in sorted(found.items()):
        if LAYER[b] >= LAYER[a]:
            out.append(f"{a} (layer {LAYER[a]}) imports {b} (layer {LAYER[b]}): {', '.join(sorted(set(mods)))}")
    graph = defaultdict(set)
    for a, b in found:
        graph[a].add(b)
    state: dict[str, int] = {}

    def visit(n, stack):
        state[n] = 1
        for m in sorted(graph[n]):
            if state.get(m) == 1:
                out.append("cycle: " + " -> ".join(stack[stack.index(m):] + [m]))
            elif m not in state:
                visit(m, stack + [m])
        state[n] = 2

    for n in sorted(graph):
        if n not in state:
            visit(n, [n])
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m octopus_b200.tools.import_graph")
    ap.add_argument("--root", default=str(Path(__file__).resolve().parents[2]))
    ap.add_argument("--show", action="store_true", help="print every package edge")
    args = ap.parse_args(argv)
    found = edges(Path(args.root))
    if args.show:
        for (a, b), mods in sorted(found.items()):
            print(f"{a} -> {b}  ({len(set(mods))} modules)")
    bad = problems(found)
    for line in bad:
        print(line)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
