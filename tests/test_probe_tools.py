"""Probe / bench tools on CPU: step table, delta-render bench, replay bench."""
import json

from octopus_b200.tools import delta_render_bench, replay_bench, step_stats


def test_step_stats(tmp_path, capsys):
    p = tmp_path / "steps.jsonl"
    p.write_text('{"step": 1, "mean_reward": 0.5, "grad_norm": 1.25, "time": 3.0}\n'
                 '{"step": 2, "mean_reward": 0.75}\n')
    assert step_stats.main([str(p)]) == 0
    out = capsys.readouterr().out.splitlines()
    assert out[0].startswith("step |") and out[1].startswith("1 | 0.5") and " - " in out[2]


def test_delta_render_bench(capsys):
    assert delta_render_bench.main(["--tokens", "2000"]) == 0
    row = json.loads(capsys.readouterr().out.strip())
    assert row["history_tokens"] > 1000 and row["speedup"] > 1


def test_replay_bench_cpu(capsys):
    assert replay_bench.main(["--synthetic", "96", "--branch", "64:32", "--preset", "tiny", "--layers", "2",
                              "--cpu"]) == 0
    row = json.loads(capsys.readouterr().out.strip())
    assert row["tree_tokens"] < row["flat_tokens"]


def test_lora_parity_cpu():
    from octopus_b200.tools.lora_parity import run

    r = run(preset="tiny", rank=4, randomize=True, device="cpu")
    # the engine serves the merged adapter: it matches the trainer with the adapter, not without
    assert r["engine_vs_trainer_lora"] < 1e-3 < r["engine_vs_trainer_base"]
