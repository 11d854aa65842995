"""The package layering (octopus_b200.tools.import_graph): no subpackage imports a package
of its own or a higher layer, and the package graph has no cycle."""
from octopus_b200.tools import import_graph


def test_layering_holds():
    assert import_graph.main([]) == 0


def test_checker_reports_a_violation(tmp_path):
    pkg = tmp_path / "octopus_b200"
    (pkg / "ops").mkdir(parents=True)
    (pkg / "rl").mkdir()
    (pkg / "ops" / "x.py").write_text("from ..rl import y\n")
    (pkg / "rl" / "y.py").write_text("from ..ops import x\n")
    found = import_graph.edges(tmp_path)
    bad = import_graph.problems(found)
    assert any("ops (layer 1) imports rl" in b for b in bad) and any(b.startswith("cycle") for b in bad)
