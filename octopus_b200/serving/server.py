"""HTTP serving front-end of the rollout engine (FastAPI).

Endpoints (wire format shared with the reference's patched SGLang):
  POST /generate               {input_ids, cursor?, mount?, sampling_params{max_new_tokens, temperature,
                                top_p, top_k, stop_token_ids},
                                rid?} -> {output_ids, meta_info{id, cursor, prompt_tokens, cached_tokens,
                                completion_tokens, output_token_logprobs}}
  POST /v1/chat/completions    OpenAI chat body + optional ``cursor`` (send only the messages
                                after that reply) and ``mount`` ([{cursor, start, end}]) -> chat
                                completion with ``cursor`` (the reply's id) and tool_calls parsed
  GET  /v1/loads               token usage and queue of this server (router admission)
  GET  /get_server_info        model and mount capabilities (mount_layers)
  GET  /health
  POST /release_cursor         {cursor}
  POST /flush_cache
  POST /update_weights_from_disk {model_path}   (HF safetensors; bumps the weight version)

Unknown cursors answer 404 (the client then resends the full history); invalid mounts
answer 400.  Requests are batched: concurrent requests arriving within a short window
run as one engine batch (continuous batching at request granularity).

Reference parity: `patches/apply_sglang_cursor.py:1-193` and `patches/apply_sglang_mount.py`
(cursor/mount fields on /generate and chat, 404 on unknown cursor), `octopus/serving/
route.py:75` (server_load reads /v1/loads), `octopus/rl/config.py:92-104` (check_mount_layers
reads /get_server_info).
"""
from __future__ import annotations

import time

from .chat import ChatTokenizer
from .engine import CursorNotFound, Engine, GenInput
from .local import BatchingQueue, ChatService, _top_k, mounts_of  # noqa: F401  (BatchingQueue re-exported)


def generate_input(body: dict) -> GenInput:
    """/generate body -> engine request."""
    sp = body.get("sampling_params") or {}
    return GenInput(list(body.get("input_ids") or []), cursor=body.get("cursor"), mount=mounts_of(body),
                    max_new_tokens=int(sp.get("max_new_tokens", 128)), temperature=float(sp.get("temperature", 1.0)),
                    stop_ids=tuple(sp.get("stop_token_ids") or ()),
                    prefill_only=int(sp.get("max_new_tokens", 1)) == 0,
                    top_p=float(sp.get("top_p", 1.0)), top_k=_top_k(sp.get("top_k")))


def generate_output(o, tokenizer=None) -> dict:
    return {"output_ids": o.output_ids, "text": tokenizer.decode(o.output_ids) if tokenizer else None,
            "meta_info": {"id": o.cursor, "cursor": o.cursor, "prompt_tokens": o.prompt_tokens,
                          "cached_tokens": o.cached_tokens, "completion_tokens": len(o.output_ids),
                          "finish_reason": o.finish_reason, "output_token_logprobs": o.output_logprobs}}


def create_app(engine: Engine, tokenizer: ChatTokenizer | None = None, model_name: str = "octopus-b200"):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse

    app = FastAPI()
    svc = ChatService(engine, tokenizer, model_name)
    q = svc.q
    state = {"started": time.time()}

    async def _run(inp: GenInput):
        try:
            return await q.submit(inp)
        except CursorNotFound as e:
            raise HTTPException(404, f"unknown cursor {e}") from None
        except ValueError as e:
            raise HTTPException(400, str(e)) from None

    @app.get("/health")
    async def health():
        return {"ok": True}

    @app.get("/v1/loads")
    async def loads():
        st = engine.load_stats()
        return {"token_usage": st["token_usage"], "num_used_tokens": st["num_used_slots"],
                "num_waiting_reqs": q.n_waiting, "num_running_reqs": q.n_running, "cursors": st["cursors"]}

    @app.get("/get_server_info")
    async def server_info():
        return {"model_path": model_name, "mount_layers": engine.mount_layers, "page_size": 1,
                "supports_mount": True, "supports_cursor": True, "weight_version": engine.version,
                "max_batch": engine.max_batch, "kv_slots": engine.kv_slots}

    @app.post("/generate")
    async def generate(body: dict):
        o = await _run(generate_input(body))
        return generate_output(o, tokenizer)

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        if tokenizer is None:
            raise HTTPException(400, "server started without a tokenizer")
        try:
            return JSONResponse(await svc.chat(body))
        except CursorNotFound as e:
            raise HTTPException(404, f"unknown cursor {e}") from None
        except ValueError as e:
            raise HTTPException(400, str(e)) from None

    @app.post("/release_cursor")
    async def release(body: dict):
        engine.release_cursor(body["cursor"])
        return {"ok": True}

    @app.post("/flush_cache")
    async def flush():
        engine.reset()
        return {"ok": True}

    @app.post("/update_weights_from_disk")
    async def update(body: dict):
        from ..models.decoder import load_hf
        load_hf(engine.w, body["model_path"])
        return {"ok": True, "weight_version": engine.bump_version()}

    return app


def serve(engine: Engine, tokenizer=None, host: str = "127.0.0.1", port: int = 30000):
    import uvicorn

    uvicorn.run(create_app(engine, tokenizer), host=host, port=port, log_level="warning")


def build_engine(preset: str, model_path: str = "", kv_gb: float = 8.0, max_batch: int = 256, layers: int = 0,
                 device=None):
    """(engine, tokenizer) for a preset: dense presets get the paged engine, hybrid presets
    (models.hybrid.hybrid_config) the hybrid engine; weights from an HF directory (the
    hybrid linear layers from its hybrid_linear.safetensors) or random init."""
    import os

    import torch

    from ..models.config import get_config
    from ..models.decoder import FlatLayout, Weights, init_flat, load_hf
    from ..models.hybrid import HybridWeights, hybrid_config

    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    has_tok = bool(model_path) and os.path.exists(os.path.join(model_path, "tokenizer.json"))
    tok = ChatTokenizer.from_dir(model_path) if has_tok else ChatTokenizer.tiny()
    hc = hybrid_config(preset, layers)
    cfg = hc.base if hc is not None else get_config(preset, **({"layers": layers} if layers else {}))
    kv_slots = max(4096, int(kv_gb * (1 << 30) / (4 * cfg.layers * cfg.kv_width)))
    if hc is not None:
        from .hybrid_engine import HybridEngine

        hw = HybridWeights(hc, dev, dtype=dtype)
        if model_path:
            load_hf(hw.dense, model_path)
            from safetensors.torch import load_file

            st = load_file(os.path.join(model_path, "hybrid_linear.safetensors"))
            with torch.no_grad():
                for k, t in list(hw.t.items()) + list(hw.fp32.items()):
                    t.copy_(st[k].to(t.dtype))
        return HybridEngine(hw, kv_slots=kv_slots, max_batch=max_batch, device=dev), tok
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, dev, dtype=dtype), lay)
    if model_path:
        load_hf(w, model_path)
    return Engine(cfg, w, kv_slots=kv_slots, max_batch=max_batch, device=dev), tok


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(prog="python -m octopus_b200.serving.server")
    ap.add_argument("--preset", default="qwen2.5-7b", help="dense preset or hybrid preset (tiny-hybrid, hybrid-7b)")
    ap.add_argument("--model-path", default="", help="HF checkpoint directory (weights, tokenizer, chat template)")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--kv-gb", type=float, default=24.0)
    ap.add_argument("--max-batch", type=int, default=256)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--device", default=None)
    ap.add_argument("--check", action="store_true", help="build the engine and app, then exit (no listening)")
    args = ap.parse_args(argv)
    eng, tok = build_engine(args.preset, args.model_path, args.kv_gb, args.max_batch, args.layers, args.device)
    if args.check:
        create_app(eng, tok)
        print(f"ok: {type(eng).__name__} {args.preset} on {eng.device}")
        return 0
    serve(eng, tok, args.host, args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
