"""HTTP server over the continuous-batching scheduler: token ids in, generated token ids out.

    python -m eagle4_b200.serve --model qwen3.8-27b [--draft DIR] [--config JSON] [--max-batch 8] [--port 8000]
    python -m eagle4_b200.serve --model qwen3.8-27b --no-spec ...        # plain decode (parity reference)

``POST /v1/generate`` with ``{"prompt_ids": [...], "max_new_tokens": n, "stop_token_ids": [...], "eos_token_id": e,
"ignore_eos": false}`` returns ``{"output_ids": [...], "finish_reason": "length" | "stop" | "eos", "meta": {...}}``.
Requests join the running batch between rounds and leave it on their own stop condition
(:class:`~eagle4_b200.runtime.scheduler.Scheduler`); one worker thread owns the engine. ``GET /health`` reports the
queue, the running batch and the engine's acceptance statistics.
"""

from __future__ import annotations

import argparse
import queue
import threading
from concurrent.futures import Future
from typing import List, Optional

from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

try:
    from pydantic import BaseModel

    class GenerateRequest(BaseModel):
        prompt_ids: List[int]
        max_new_tokens: int = 128
        stop_token_ids: List[int] = []
        eos_token_id: Optional[int] = None
        ignore_eos: bool = False
except ImportError:  # the HTTP layer is optional; Batcher works without it
    GenerateRequest = None


class Batcher:
    """The serving loop: submitted requests enter the scheduler between rounds; each caller's future resolves
    when its request finishes."""

    def __init__(self, engine, max_batch: Optional[int] = None, *, speculative: bool = True):
        self.engine = engine
        self.sched = Scheduler(engine, speculative=speculative)
        self.q: "queue.Queue" = queue.Queue()
        self.stop = threading.Event()
        self.futures = {}
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, prompt: List[int], params: RequestParams = RequestParams()) -> Future:
        fut: Future = Future()
        self.q.put((prompt, params, fut))
        return fut

    def _drain(self, block: bool) -> None:
        while True:
            try:
                prompt, params, fut = self.q.get(timeout=0.05) if block else self.q.get_nowait()
            except queue.Empty:
                return
            block = False
            try:
                req = self.sched.submit(prompt, params)
                self.futures[req.rid] = fut
            except Exception as e:  # noqa: BLE001 - a request the scheduler refuses fails alone
                fut.set_exception(e)

    def _loop(self) -> None:
        while not self.stop.is_set():
            self._drain(block=self.sched.idle)
            if self.sched.idle:
                continue
            try:
                finished = self.sched.step()
            except Exception as e:  # noqa: BLE001 - the engine failed: every request in flight gets the error
                for fut in self.futures.values():
                    fut.set_exception(e)
                self.futures.clear()
                self.sched = Scheduler(self.engine, speculative=self.sched.speculative)
                continue
            for req in finished:
                fut = self.futures.pop(req.rid, None)
                if fut is not None:
                    fut.set_result(req)


def make_app(batcher: Batcher):
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="eagle4_b200")

    @app.post("/v1/generate")
    def generate(req: GenerateRequest):
        if not req.prompt_ids or req.max_new_tokens < 1:
            raise HTTPException(400, "prompt_ids must be non-empty and max_new_tokens positive")
        params = RequestParams(max_new_tokens=req.max_new_tokens, stop_token_ids=tuple(req.stop_token_ids),
                               eos_token_id=req.eos_token_id, ignore_eos=req.ignore_eos)
        try:
            r = batcher.submit(req.prompt_ids, params).result()
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        return {"output_ids": r.output, "finish_reason": r.finish_reason,
                "meta": {"rounds": r.rounds, "speculative": batcher.sched.speculative}}

    @app.get("/health")
    def health():
        st = batcher.engine.stats
        return {"queued": batcher.q.qsize() + len(batcher.sched.waiting), "running": len(batcher.sched.running),
                "rounds": st.rounds, "mean_accept": st.mean_accept}

    return app


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="eagle4_b200.serve")
    ap.add_argument("--model", required=True)
    ap.add_argument("--draft")
    ap.add_argument("--config", help="harness config JSON (inline or a path)")
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--no-spec", action="store_true", help="plain decode (the parity reference server)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    args = ap.parse_args(argv)
    import uvicorn

    from eagle4_b200.api import TreeSpec
    from eagle4_b200.cli import build_llm

    llm = build_llm(args.model, args.draft, max_batch=args.max_batch, max_len=args.max_len, tree=TreeSpec(),
                    config=args.config)
    uvicorn.run(make_app(Batcher(llm.engine, speculative=not args.no_spec)), host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
