"""A small HTTP server over the engine: token ids in, generated token ids out.

    python -m eagle4_b200.serve --model qwen3.8-27b [--draft DIR] [--config JSON] [--max-batch 8] [--port 8000]

``POST /v1/generate`` with ``{"prompt_ids": [...], "max_new_tokens": n, "speculative": true}`` returns
``{"output_ids": [...]}``. Requests queue up; a worker thread takes up to ``max_batch`` queued requests with the same
``max_new_tokens`` and runs them as one static batch through :meth:`Engine.generate` (speculative rounds with the
configured harness policy). ``GET /health`` reports the queue depth and the engine's acceptance statistics.
"""

from __future__ import annotations

import argparse
import queue
import threading
from concurrent.futures import Future
from typing import List, Optional

import torch


try:
    from pydantic import BaseModel

    class GenerateRequest(BaseModel):
        prompt_ids: List[int]
        max_new_tokens: int = 128
        speculative: bool = True
except ImportError:  # the HTTP layer is optional; Batcher works without it
    GenerateRequest = None


class Batcher:
    def __init__(self, engine, max_batch: int):
        self.engine, self.max_batch = engine, max_batch
        self.q: "queue.Queue" = queue.Queue()
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, prompt: List[int], max_new_tokens: int, speculative: bool = True) -> Future:
        fut: Future = Future()
        self.q.put((prompt, max_new_tokens, speculative, fut))
        return fut

    def _loop(self) -> None:
        pending = []
        while not self.stop.is_set():
            try:
                pending.append(self.q.get(timeout=0.05))
            except queue.Empty:
                if not pending:
                    continue
            while len(pending) < self.max_batch:
                try:
                    pending.append(self.q.get_nowait())
                except queue.Empty:
                    break
            if not pending:
                continue
            key = pending[0][1:3]
            group = [p for p in pending if p[1:3] == key][: self.max_batch]
            pending = [p for p in pending if p not in group]
            try:
                outs = self.engine.generate([torch.tensor(p[0]) for p in group], key[0], speculative=key[1])
                for p, o in zip(group, outs):
                    p[3].set_result(o)
            except Exception as e:  # noqa: BLE001 - the error goes back to every caller of the batch
                for p in group:
                    p[3].set_exception(e)


def make_app(batcher: Batcher):
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="eagle4_b200")

    @app.post("/v1/generate")
    def generate(req: GenerateRequest):
        if not req.prompt_ids or req.max_new_tokens < 1:
            raise HTTPException(400, "prompt_ids must be non-empty and max_new_tokens positive")
        return {"output_ids": batcher.submit(req.prompt_ids, req.max_new_tokens, req.speculative).result()}

    @app.get("/health")
    def health():
        st = batcher.engine.stats
        return {"queued": batcher.q.qsize(), "rounds": st.rounds, "mean_accept": st.mean_accept}

    return app


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="eagle4_b200.serve")
    ap.add_argument("--model", required=True)
    ap.add_argument("--draft")
    ap.add_argument("--config", help="harness config JSON (inline or a path)")
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    args = ap.parse_args(argv)
    import uvicorn

    from eagle4_b200.api import TreeSpec
    from eagle4_b200.cli import build_llm

    llm = build_llm(args.model, args.draft, max_batch=args.max_batch, max_len=args.max_len, tree=TreeSpec(),
                    config=args.config)
    uvicorn.run(make_app(Batcher(llm.engine, args.max_batch)), host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
