"""Engine hop client on CPU against two in-process engines: parent routing, cursor + delta,
placeholder-adjusted mounts, 404 resend of the visible history, prompt-size checks."""
import numpy as np
import pytest
import torch

from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, init_flat
from octopus_b200.serving.engine import CursorNotFound, Engine
from octopus_b200.serving.hop import EngineHop, HopError
from octopus_b200.serving.server import generate_input, generate_output


@pytest.fixture
def pool():
    cfg = get_config("tiny", vocab_size=256, layers=2)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=2, std=0.05), lay)
    engines = {s: Engine(cfg, w, kv_slots=20000, max_batch=8, device="cpu") for s in ("a:1", "b:2")}

    def transport(server, path, body):
        eng = engines[server]
        if path == "/release_cursor":
            eng.release_cursor(body["cursor"])
            return 200, {"ok": True}
        try:
            o = eng.generate([generate_input(body)])[0]
        except CursorNotFound:
            return 404, {"error": "unknown cursor"}
        return 200, generate_output(o)

    return engines, EngineHop(list(engines), transport, pick=lambda s: "b:2" if s == "b" else "a:1")


def test_hop_routes_mounts_and_resends(pool):
    engines, hop = pool
    sp = {"max_new_tokens": 4}
    r1 = hop.generate(list(range(1, 30)), sampling=sp, session="a")
    c1 = r1["cursor"]
    assert hop.where[c1] == "a:1"
    r2 = hop.generate([7, 8, 9], parent=c1, sampling=sp)
    assert hop.where[r2["cursor"]] == "a:1"
    # a reply that mounts rows of c1, then a reply mounting rows of that reply past its placeholders
    r3 = hop.generate([11, 12], mount=[(c1, 3, 10)], sampling=sp, session="a")
    c3 = r3["cursor"]
    assert r3["placeholders"] == 7
    v = hop.visible[c3]
    assert len(v) == 2 + 4
    a, b = hop.rows(c3, 0, 2)  # the first visible tokens of c3 sit after its 7 mounted rows
    assert (a, b) == (7, 9)
    cur = engines["a:1"].cursors.get(c3)
    assert [int(t) for t in cur.tokens[a:b]] == [11, 12]
    r4 = hop.generate([5], mount=[(c3, 0, 2)], sampling=sp, session="a")
    assert r4["placeholders"] == 2
    # 404: the server lost c2; the hop resends the visible history and continues
    c2 = r2["cursor"]
    engines["a:1"].release_cursor(c2)
    r5 = hop.generate([3, 4], parent=c2, sampling=sp)
    assert hop.stats["resent"] == 1 and hop.visible[r5["cursor"]][: len(hop.visible[c2])] == hop.visible[c2]
    # a lost cursor whose history holds mounted rows cannot be re-rendered
    engines["a:1"].release_cursor(c3)
    with pytest.raises(HopError):
        hop.generate([1], parent=c3, sampling=sp)
    # mounts across servers are refused
    rb = hop.generate([1, 2, 3], sampling=sp, session="b")
    with pytest.raises(HopError):
        hop.generate([1], parent=rb["cursor"], mount=[(c1, 0, 2)], sampling=sp)
