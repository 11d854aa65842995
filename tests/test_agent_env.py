"""Agent-runtime RL step on CPU: episodes of the cursor runtime through the in-process
chat service and the engine, graded, credited, exported by the workflow glue, and one
actor step on the resulting prefix-tree micro-batches."""
import numpy as np
import torch

from octopus_b200.models.config import get_config
from octopus_b200.rl.actor import Actor, OptimConfig
from octopus_b200.rl.agent_env import AgentEnv
from octopus_b200.rl.trainer import RLTrainer, TrainerConfig
from octopus_b200.runtime.tree import WorkspaceProvider
from octopus_b200.serving.chat import ChatTokenizer
from octopus_b200.serving.engine import Engine
from octopus_b200.serving.local import ChatService


class _WS(WorkspaceProvider):
    report = "the answer"

    def system_prompt(self, task):
        return "Answer the question."


def test_agent_env_rl_step_cpu(monkeypatch):
    monkeypatch.setenv("OCTOPUS_MAIN_MAX_CALLS", "2")
    monkeypatch.setenv("OCTOPUS_MAX_TOKENS", "12")
    tok = ChatTokenizer.tiny()
    cfg = get_config("tiny", vocab_size=((tok.vocab_size + 127) // 128) * 128, layers=2)
    actor = Actor(cfg, "cpu", seed=1, dtype=torch.float32, ckpt=False, optim=OptimConfig(lr=1e-4))
    eng = Engine(cfg, actor.weights, kv_slots=60000, max_batch=16, device="cpu")
    svc = ChatService(eng, tok, window=0.001)
    tasks = [{"question": f"what is {i} plus {i}?", "gold": str(2 * i)} for i in range(3)]
    rng = np.random.default_rng(0)

    def grade(task, answer):
        return float(rng.random() < 0.5)

    env = AgentEnv(svc, tasks, lambda t: _WS(), grade, n_samples=3, batch_size=3, max_main_calls=2)

    class _E:
        def rollout(self, engine):
            return env.rollout(engine)

    tr = RLTrainer(actor, eng, _E(), TrainerConfig(mb_tokens=1 << 16))
    st = tr.step()
    assert st["generated_tokens"] > 0
    assert np.isfinite(st["loss"])
    # every cursor of the step was released
    assert eng.load_stats()["cursors"] == 0
