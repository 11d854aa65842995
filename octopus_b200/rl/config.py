"""Run configuration: typed dataclasses, YAML files with ``key=value`` overrides, derived
settings, episode vs host settings, and the live-tunable env file.

Three layers, as in the reference:
1. a YAML run file (``octopus_b200/rl/grpo.yaml``) + dotted ``key=value`` overrides,
   typed by :class:`RLConfig`;
2. ``OCTOPUS_*`` switches read where used (runtime.settings), snapshotted into
   ``episode_settings.json`` (episode settings) vs machine-local host settings;
3. ``$OCTOPUS_LIVE_ENV``: a file of KEY=VALUE lines re-read per step
   (MB_TOKENS, ACT_GPU_GB, EPISODES_PER_SERVER) so a run can be tuned without a restart.

Reference parity (behaviour): `octopus/rl/config.py:20-204`, `octopus/rl/grpo.yaml:1-192`.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field

import yaml

from ..runtime import settings as S


@dataclass
class ModelSection:
    preset: str = "qwen2.5-7b"
    path: str = ""              # HF checkpoint dir to start from ("" = random init)
    dtype: str = "bfloat16"
    layers: int = 0             # override (0 = preset)


@dataclass
class RolloutSection:
    servers: str = ""           # comma list of host:port (remote engines); "" = in-process colocated engine
    max_head_offpolicyness: int = 2
    kv_gb: float = 24.0
    max_batch: int = 256
    temperature: float = 1.0
    max_new_tokens: int = 8192
    max_tokens: int = 262144
    tool_call_parser: str = "qwen3_coder"
    tp: int = 1
    push_hosts: str = ""        # comma list of remote rollout hosts to push each weight version to ("" = off)
    push_dir: str = ""          # destination folder on those hosts (one v<version> subfolder per push)


@dataclass
class ActorSection:
    lr: float = 2.0e-5
    weight_decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    gradient_clipping: float = 1.0
    eps_clip: float = 0.2
    eps_clip_higher: float = 0.28
    behav_imp_weight_cap: float = 5.0
    reuse_train_logp: bool = True
    mb_tokens: int = 262144     # prefix-tree tokens per micro-batch
    gradient_checkpointing: bool = True
    sharded: bool = True        # ZeRO-sharded optimizer state over ranks
    full_shard: bool = False    # FSDP: weights, gradients and optimizer state sharded per layer (parallel.fsdp.FSDPActor)
    gather_weights: bool = False  # FSDP: gather each layer from the shards instead of reading the serving copy
    fused_collectives: bool = True
    lora_rank: int = 0          # > 0: train LoRA adapters on a frozen base (single-replica actor)
    lora_alpha: float = 32.0
    lora_targets: str = "all-linear"
    ckpt_block: int = 1         # block checkpointing: keep every k-th layer input
    act_gpu_gb: float = -1.0    # >= 0: saved activations past this many GB live in pinned host memory
    chunk_tokens: int = 0       # > 0: micro-batches with more tree rows train chunk-major in chunks of this size
    seq_tile: int = 0           # > 0: each layer's o-projection + MLP run in checkpointed tiles of this many rows


@dataclass
class RLSection:
    kind: str = "dag"           # dag | search | swe
    n_samples: int = 4
    batch_size: int = 32        # prompts (DAG instances) per step
    branch_credit: str = "outcome"
    filter_zero_variance: bool = True
    spool: str = ""             # rollout spool dir ("" = off)
    search_questions: str = ""
    swe_tasks: str = ""         # kind=swe: JSONL task rows (envs.swe.taskset), or a directory of them
    swe_bundle: int = 0         # > 1: bundles of this many tasks of one repository per episode
    swe_timeout: float = 120.0  # seconds per tool / test command
    episodes_per_server: int = 8
    dag_prefix: int = 2048      # kind=dag: the shared task prefix every agent mounts
    dag_turn: int = 512         # kind=dag: tokens per agent turn
    disaggregate: bool = False  # > 1 GPU: rollout GPUs and trainer GPUs run one step apart (rl.disagg)
    rollout_gpus: int = 0       # disaggregate: rollout GPUs (0: half, rounded up)


@dataclass
class CheckpointSection:
    dir: str = ""
    recover_every: int = 1      # steps between recover checkpoints
    save_every: int = 5         # steps between HF weight saves
    keep: int = 2


@dataclass
class RLConfig:
    experiment_name: str = "octopus-b200"
    trial_name: str = "run0"
    seed: int = 1
    total_steps: int = 100
    model: ModelSection = field(default_factory=ModelSection)
    rollout: RolloutSection = field(default_factory=RolloutSection)
    actor: ActorSection = field(default_factory=ActorSection)
    rl: RLSection = field(default_factory=RLSection)
    checkpoint: CheckpointSection = field(default_factory=CheckpointSection)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def _coerce(value: str, typ):
    if typ is bool or isinstance(typ, bool):
        return str(value).lower() in ("1", "true", "yes", "on")
    if typ in (int, float, str):
        return typ(value)
    return yaml.safe_load(value)


def _apply(obj, d: dict, prefix=""):
    for k, v in d.items():
        if not hasattr(obj, k):
            raise KeyError(f"unknown config key {prefix}{k}")
        cur = getattr(obj, k)
        if dataclasses.is_dataclass(cur):
            if not isinstance(v, dict):
                raise TypeError(f"{prefix}{k} is a section")
            _apply(cur, v, prefix + k + ".")
        else:
            setattr(obj, k, type(cur)(v) if cur is not None and not isinstance(cur, bool) else
                    (_coerce(v, bool) if isinstance(cur, bool) else v))


def override(cfg: RLConfig, items: list[str]) -> RLConfig:
    """Apply dotted key=value overrides."""
    for it in items:
        key, _, val = it.partition("=")
        parts = key.strip().split(".")
        obj = cfg
        for p in parts[:-1]:
            obj = getattr(obj, p)
        cur = getattr(obj, parts[-1])
        setattr(obj, parts[-1], _coerce(val, type(cur)))
    return cfg


def load(path: str | None = None, overrides: list[str] | None = None) -> RLConfig:
    cfg = RLConfig()
    if path:
        with open(path) as f:
            _apply(cfg, yaml.safe_load(f) or {})
    return override(cfg, overrides or [])


def set_derived_settings(cfg: RLConfig) -> None:
    """Settings derived from the run config that the runtime reads from the environment."""
    os.environ.setdefault("OCTOPUS_TOOL_FORMAT", cfg.rollout.tool_call_parser)
    os.environ.setdefault("OCTOPUS_MAX_TOKENS", str(cfg.rollout.max_new_tokens))
    os.environ.setdefault("OCTOPUS_CONTEXT_WINDOW", str(cfg.rollout.max_tokens))


HOST_ENV = ("OCTOPUS_HTTP_ATTEMPTS", "OCTOPUS_HTTP_TIMEOUT", "OCTOPUS_HTTP_WORKERS", "OCTOPUS_ROUTE_KV",
            "OCTOPUS_ROUTE_TREE_TOKENS", "OCTOPUS_ROUTE_WAIT", "OCTOPUS_LIVE_ENV", "OCTOPUS_ROLLOUT_SPOOL")


def save_settings(path: str) -> dict:
    """Snapshot the episode switches (what an evaluation must reproduce)."""
    st = S.episode_settings()
    with open(path, "w") as f:
        json.dump(st, f, indent=1, sort_keys=True)
    return st


def run_episode_settings(path: str) -> None:
    """Apply a saved episode_settings.json (eval runs the same episode rules as training)."""
    with open(path) as f:
        st = json.load(f)
    for k in S.EPISODE_KEYS:
        if k in st:
            os.environ[k] = str(st[k])
        else:
            os.environ.pop(k, None)


LIVE_KEYS = {"MB_TOKENS": int, "ACT_GPU_GB": float, "EPISODES_PER_SERVER": int}


def live_env() -> dict:
    """KEY=VALUE lines of $OCTOPUS_LIVE_ENV (re-read each call; unknown keys ignored)."""
    p = os.environ.get("OCTOPUS_LIVE_ENV")
    out = {}
    if not p or not os.path.exists(p):
        return out
    for line in open(p):
        line = line.strip()
        if not line or line.startswith("#") or "=" not in line:
            continue
        k, v = (x.strip() for x in line.split("=", 1))
        if k in LIVE_KEYS:
            try:
                out[k] = LIVE_KEYS[k](v)
            except ValueError:
                continue
    return out
