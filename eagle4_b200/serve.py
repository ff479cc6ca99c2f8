"""HTTP server over the continuous-batching scheduler.

    python -m eagle4_b200.serve --model qwen3.8-27b [--draft DIR] [--config JSON] [--max-batch 8] [--port 8000]
    python -m eagle4_b200.serve --model TARGET_DIR --draft DRAFT_DIR [--tokenizer DIR]   # text in, text out
    python -m eagle4_b200.serve --model qwen3.8-27b --no-spec ...        # plain decode (parity reference)
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m eagle4_b200.serve --model ...
                                                                          # tensor-parallel over 8 GPUs

* ``POST /v1/generate`` with ``{"prompt_ids": [...], "max_new_tokens": n, "stop_token_ids": [...], "eos_token_id": e,
  "ignore_eos": false}`` returns ``{"output_ids": [...], "finish_reason": "length" | "stop" | "eos", "meta": {...}}``.
* ``POST /v1/completions`` (the OpenAI completions shape): ``{"prompt": text or token ids, "max_tokens": n,
  "stop": text(s), "stop_token_ids": [...], "ignore_eos": false}``; text needs a tokenizer (``--tokenizer``, or the
  target directory's own). Stop strings end a request where they appear and are cut from the returned text; the
  tokenizer's end-of-sequence token ends it unless ``ignore_eos``.
* ``POST /v1/chat/completions``: ``{"messages": [...], ...}`` through the tokenizer's chat template; the answer is
  ``choices[0].message``.
* ``"stream": true`` on either returns server-sent events: one chunk per round with the new tokens and the text they
  add (text that could still become a stop string, or ends in an incomplete character, is held back to the next
  chunk), a last chunk with the finish reason and usage, then ``[DONE]``.
* ``GET /health``: queue, running batch, acceptance; ``GET /metrics``: the same and the counters, in Prometheus's
  text format.

Requests join the running batch between rounds and leave it on their own stop condition
(:class:`~eagle4_b200.runtime.scheduler.Scheduler`); one worker thread owns the engine.
"""

from __future__ import annotations

import argparse
import queue
import threading
import time
from concurrent.futures import Future
from typing import Callable, List, Optional, Union

from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

try:
    from pydantic import BaseModel

    class GenerateRequest(BaseModel):
        prompt_ids: List[int]
        max_new_tokens: int = 128
        stop_token_ids: List[int] = []
        eos_token_id: Optional[int] = None
        ignore_eos: bool = False

    class CompletionRequest(BaseModel):
        prompt: Union[str, List[int]]
        max_tokens: int = 16
        stop: Union[str, List[str], None] = None
        stop_token_ids: List[int] = []
        ignore_eos: bool = False
        temperature: Optional[float] = None
        model: Optional[str] = None
        stream: bool = False
        n: int = 1

    class ChatRequest(BaseModel):
        messages: List[dict]
        max_tokens: int = 256
        stop: Union[str, List[str], None] = None
        stop_token_ids: List[int] = []
        ignore_eos: bool = False
        temperature: Optional[float] = None
        model: Optional[str] = None
        stream: bool = False
        n: int = 1
except ImportError:  # the HTTP layer is optional; Batcher works without it
    GenerateRequest = CompletionRequest = ChatRequest = None


class QueueFull(RuntimeError):
    """The server's queue is at its limit (HTTP 503)."""


class Batcher:
    """The serving loop: submitted requests enter the scheduler between rounds; each caller's future resolves
    when its request finishes. With ``lockstep`` (tensor-parallel serving, rank 0) every step's submissions are
    first broadcast to the other ranks, which mirror them (:func:`eagle4_b200.runtime.lockstep.follow`)."""

    def __init__(self, engine, max_batch: Optional[int] = None, *, speculative: bool = True, lockstep=None,
                 detokenize: Optional[Callable[[List[int]], str]] = None, max_queue: Optional[int] = None,
                 batch_prefill: bool = False):
        """``detokenize``: token ids -> text, for requests with stop strings (every rank needs the same one).
        ``max_queue``: requests waiting beyond the running batch above which new ones are refused (``QueueFull``)."""
        self.max_queue = max_queue
        self.engine = engine
        self.detokenize = detokenize
        self.batch_prefill = batch_prefill
        self.sched = Scheduler(engine, speculative=speculative, detokenize=detokenize, batch_prefill=batch_prefill)
        self.lockstep = lockstep
        self.counts = {"requests": 0, "finished": 0, "refused": 0, "prompt_tokens": 0, "generated_tokens": 0}
        self.q: "queue.Queue" = queue.Queue()
        self.stop = threading.Event()
        self.futures = {}
        self.streams = {}  # rid -> [request, queue, tokens already sent]
        self.failed: Optional[BaseException] = None
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, prompt: List[int], params: RequestParams = RequestParams(),
               stream: Optional["queue.Queue"] = None) -> Future:
        """Queue a request; the future resolves with the finished request. ``stream``: a queue that receives each
        round's new tokens (a list) as they are emitted, then ``None`` when the request ends."""
        fut: Future = Future()
        refusal = None
        if self.failed is not None:
            refusal = RuntimeError(f"serving stopped after an engine error: {self.failed}")
        elif self.max_queue is not None and self.queued >= self.max_queue:
            refusal = QueueFull(f"{self.queued} requests are waiting (the limit is {self.max_queue}); retry later")
        if refusal is not None:
            self.counts["refused"] += 1
            fut.set_exception(refusal)
            if stream is not None:
                stream.put(None)
            return fut
        self.q.put((prompt, params, fut, stream))
        return fut

    @property
    def queued(self) -> int:
        """Requests submitted and not yet running."""
        return self.q.qsize() + len(self.sched.waiting)

    def close(self, timeout: Optional[float] = None) -> None:
        """Stop serving (followers are told to stop too); requests still queued are not run."""
        self.stop.set()
        self.thread.join(timeout)

    def _drain(self, block: bool) -> list:
        got = []
        while True:
            try:
                got.append(self.q.get(timeout=0.05) if block and not got else self.q.get_nowait())
            except queue.Empty:
                return got

    def _admit(self, subs: list) -> None:
        from eagle4_b200.runtime.lockstep import Command, apply

        cmd = Command([(p, params) for p, params, _, _ in subs])
        for (_, _, fut, stream), got in zip(subs, apply(self.sched, cmd)):
            if isinstance(got, Exception):
                self.counts["refused"] += 1
                fut.set_exception(got)
                if stream is not None:
                    stream.put(None)
            else:
                self.counts["requests"] += 1
                self.counts["prompt_tokens"] += int(got.prompt.numel())
                self.futures[got.rid] = fut
                if stream is not None:
                    self.streams[got.rid] = [got, stream, 0]

    def _publish(self) -> None:
        """Each streamed request's new tokens; ``None`` after its last."""
        for rid, entry in list(self.streams.items()):
            req, stream, sent = entry
            if len(req.output) > sent:
                stream.put(list(req.output[sent:]))
                entry[2] = len(req.output)
            if req.finished:
                stream.put(None)
                del self.streams[rid]

    def _fail(self, e: BaseException) -> None:
        for fut in self.futures.values():
            fut.set_exception(e)
        self.futures.clear()
        for _, stream, _ in self.streams.values():
            stream.put(None)
        self.streams.clear()

    def _loop(self) -> None:
        import time

        from eagle4_b200.runtime.lockstep import Command

        last = time.monotonic()
        while True:
            stopping = self.stop.is_set()
            subs = [] if stopping else self._drain(block=self.sched.idle)
            if self.lockstep is not None:
                now = time.monotonic()
                if stopping or subs or not self.sched.idle or now - last >= self.lockstep.beat_s:
                    self.lockstep.exchange(Command([(list(map(int, p)), params) for p, params, _, _ in subs],
                                                   stop=stopping))
                    last = now
            if stopping:
                return
            if subs:
                self._admit(subs)
            if self.sched.idle:
                continue
            try:
                finished = self.sched.step()
            except Exception as e:  # noqa: BLE001 - the engine failed: every request in flight gets the error
                self._fail(e)
                if self.lockstep is not None:  # ranks may be out of step: stop serving (a restart recovers)
                    self.failed = e
                    try:  # best effort: followers still waiting for a command end cleanly
                        self.lockstep.exchange(Command(stop=True))
                    except Exception:  # noqa: BLE001 - the group may be gone already
                        pass
                    return
                self.sched = Scheduler(self.engine, speculative=self.sched.speculative, detokenize=self.detokenize,
                                       batch_prefill=self.batch_prefill)
                continue
            self._publish()
            for req in finished:
                self.counts["finished"] += 1
                self.counts["generated_tokens"] += len(req.output)
                fut = self.futures.pop(req.rid, None)
                if fut is not None:
                    fut.set_result(req)


def _cut_at_stop(text: str, stops: List[str]) -> str:
    """The text before the first stop string (OpenAI's convention: the stop string is not returned)."""
    cut = min((i for i in (text.find(s) for s in stops) if i >= 0), default=-1)
    return text if cut < 0 else text[:cut]


def metrics_text(batcher: Batcher) -> str:
    """The server's counters and gauges in Prometheus's text format (read at scrape time)."""
    from prometheus_client import CollectorRegistry, generate_latest
    from prometheus_client.core import CounterMetricFamily, GaugeMetricFamily

    st, c = batcher.engine.stats, batcher.counts

    class _Collector:
        def collect(self):
            for name, doc, value in (("requests", "requests admitted", c["requests"]),
                                     ("requests_finished", "requests finished", c["finished"]),
                                     ("requests_refused", "requests refused at submission", c["refused"]),
                                     ("prompt_tokens", "prompt tokens admitted", c["prompt_tokens"]),
                                     ("generated_tokens", "tokens generated by finished requests",
                                      c["generated_tokens"]),
                                     ("rounds", "engine rounds (speculative or native)", st.rounds),
                                     ("emitted_tokens", "tokens emitted by speculative rounds", st.emitted),
                                     ("draft_kv_holes", "natively decoded positions left without draft KV",
                                      st.draft_kv_holes)):
                yield CounterMetricFamily(f"eagle4_{name}", doc, value=value)
            acc = CounterMetricFamily("eagle4_accepted_per_request_round", "request-rounds by tokens emitted",
                                      labels=["tokens"])
            for k in sorted(st.accepted_hist):
                acc.add_metric([str(k)], st.accepted_hist[k])
            yield acc
            for name, doc, value in (("queued", "requests waiting", batcher.q.qsize() + len(batcher.sched.waiting)),
                                     ("running", "requests in the running batch", len(batcher.sched.running)),
                                     ("mean_accept", "mean tokens per request-round", st.mean_accept),
                                     ("failed", "1 after an engine error stopped serving",
                                      0 if batcher.failed is None else 1)):
                yield GaugeMetricFamily(f"eagle4_{name}", doc, value=value)

    reg = CollectorRegistry()
    reg.register(_Collector())
    return generate_latest(reg).decode()


def make_app(batcher: Batcher, tokenizer=None, model_name: str = "eagle4_b200"):
    """``tokenizer``: a Hugging Face tokenizer for text prompts and text output (optional)."""
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI(title="eagle4_b200")

    def run(prompt_ids, params, n: int = 1):
        """``n`` independent requests of one prompt (they share rounds); their finished requests in order."""
        if not 1 <= n <= 64:
            raise HTTPException(400, "n must be in 1..64")
        futs = [batcher.submit(prompt_ids, params) for _ in range(n)]
        try:
            return [f.result() for f in futs]
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        except QueueFull as e:
            raise HTTPException(503, str(e)) from e

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "eagle4_b200"}]}

    @app.post("/v1/generate")
    def generate(req: GenerateRequest):
        if not req.prompt_ids or req.max_new_tokens < 1:
            raise HTTPException(400, "prompt_ids must be non-empty and max_new_tokens positive")
        params = RequestParams(max_new_tokens=req.max_new_tokens, stop_token_ids=tuple(req.stop_token_ids),
                               eos_token_id=req.eos_token_id, ignore_eos=req.ignore_eos)
        r = run(req.prompt_ids, params)[0]
        return {"output_ids": r.output, "finish_reason": r.finish_reason,
                "meta": {"rounds": r.rounds, "speculative": batcher.sched.speculative}}

    def params_of(req, ids) -> RequestParams:
        if not ids or req.max_tokens < 1:
            raise HTTPException(400, "the prompt must be non-empty and max_tokens positive")
        temp = float(batcher.engine.temperature)
        if req.temperature is not None and abs(req.temperature - temp) > 1e-6:
            raise HTTPException(400, f"this server samples every request at temperature {temp:g}")
        stops = [req.stop] if isinstance(req.stop, str) else list(req.stop or [])
        if stops and tokenizer is None:
            raise HTTPException(400, "stop strings need a tokenizer (start the server with --tokenizer)")
        eos = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None
        return RequestParams(max_new_tokens=req.max_tokens, stop_token_ids=tuple(req.stop_token_ids),
                             eos_token_id=eos, ignore_eos=req.ignore_eos, stop=tuple(stops))

    def text_of(tokens, params, final: bool) -> Optional[str]:
        """The text to show for ``tokens``: cut at a stop string; while streaming, the tail that could still turn
        into a stop string, or that ends in an incomplete character, is held back."""
        if tokenizer is None:
            return None
        text = tokenizer.decode(tokens)
        stops = list(params.stop)
        if stops:
            cut = _cut_at_stop(text, stops)
            if len(cut) < len(text):
                return cut
            if not final:
                text = text[:max(0, len(text) - (max(map(len, stops)) - 1))]
        return text if final else text.rstrip("\ufffd")

    def finish_of(r) -> str:
        return "length" if r.finish_reason == "length" else "stop"

    def usage(n_prompt: int, n_out: int) -> dict:
        return {"prompt_tokens": n_prompt, "completion_tokens": n_out, "total_tokens": n_prompt + n_out}

    def sse(ids, params, chunk):
        """Server-sent events of a streamed request: ``chunk(text delta, new tokens, finish reason)`` per round."""
        import json
        import queue as q_

        stream: "q_.Queue" = q_.Queue()
        fut = batcher.submit(ids, params, stream=stream)
        if fut.done() and fut.exception() is not None:  # refused at submission: an HTTP error, not a stream
            e = fut.exception()
            raise HTTPException(503 if isinstance(e, QueueFull) else 400, str(e))

        def events():
            tokens, shown = [], ""
            while True:
                new = stream.get()
                if new is None:
                    break
                tokens += new
                text = text_of(tokens, params, final=False)
                delta = None
                if text is not None:
                    delta, shown = (text[len(shown):], text) if text.startswith(shown) else ("", shown)
                yield f"data: {json.dumps(chunk(delta, new, None))}\n\n"
            try:
                r = fut.result()
            except Exception as e:  # noqa: BLE001 - the request failed: report it in the stream
                yield f"data: {json.dumps({'error': str(e)})}\n\n"
                return
            text = text_of(r.output, params, final=True)
            delta = None if text is None else text[len(shown):] if text.startswith(shown) else ""
            last = chunk(delta, [], finish_of(r))
            last["usage"] = usage(len(ids), len(r.output))
            yield f"data: {json.dumps(last)}\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(events(), media_type="text/event-stream")

    @app.post("/v1/completions")
    def completions(req: CompletionRequest):
        if isinstance(req.prompt, str):
            if tokenizer is None:
                raise HTTPException(400, "text prompts need a tokenizer (start the server with --tokenizer)")
            ids = list(tokenizer(req.prompt)["input_ids"])
        else:
            ids = list(req.prompt)
        params = params_of(req, ids)
        head = {"object": "text_completion", "created": int(time.time()), "model": req.model or model_name}
        if req.stream:
            if req.n != 1:
                raise HTTPException(400, "streamed completions take n = 1")
            return sse(ids, params, lambda delta, new, fin: dict(head, id="cmpl-stream", choices=[
                {"index": 0, "text": delta, "token_ids": new, "finish_reason": fin}]))
        rs = run(ids, params, req.n)
        return dict(head, id=f"cmpl-{rs[0].rid}", choices=[
            {"index": i, "text": text_of(r.output, params, True), "token_ids": r.output, "finish_reason": finish_of(r)}
            for i, r in enumerate(rs)], usage=usage(len(ids), sum(len(r.output) for r in rs)))

    @app.post("/v1/chat/completions")
    def chat(req: ChatRequest):
        if tokenizer is None or not getattr(tokenizer, "chat_template", None):
            raise HTTPException(400, "chat needs a tokenizer with a chat template (start the server with --tokenizer)")
        enc = tokenizer.apply_chat_template(req.messages, add_generation_prompt=True, tokenize=True)
        ids = list(enc["input_ids"] if hasattr(enc, "keys") else enc)  # a list, or an encoding (newer tokenizers)
        params = params_of(req, ids)
        head = {"created": int(time.time()), "model": req.model or model_name}
        if req.stream:
            if req.n != 1:
                raise HTTPException(400, "streamed completions take n = 1")
            return sse(ids, params, lambda delta, new, fin: dict(head, id="chatcmpl-stream",
                                                                 object="chat.completion.chunk", choices=[
                {"index": 0, "delta": {"content": delta} if delta else {}, "finish_reason": fin}]))
        rs = run(ids, params, req.n)
        return dict(head, id=f"chatcmpl-{rs[0].rid}", object="chat.completion", choices=[
            {"index": i, "message": {"role": "assistant", "content": text_of(r.output, params, True)},
             "finish_reason": finish_of(r)} for i, r in enumerate(rs)],
            usage=usage(len(ids), sum(len(r.output) for r in rs)))

    @app.get("/health")
    def health():
        st = batcher.engine.stats
        tp = batcher.engine.target.tp
        return {"queued": batcher.queued, "running": len(batcher.sched.running),
                "rounds": st.rounds, "mean_accept": st.mean_accept, "tensor_parallel": tp.world if tp else 1,
                "failed": None if batcher.failed is None else str(batcher.failed)}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        return metrics_text(batcher)

    return app


def load_tokenizer(path: Optional[str]):
    """A Hugging Face tokenizer from a local directory (no network), or None."""
    if not path:
        return None
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(path, local_files_only=True)


def main(argv: Optional[List[str]] = None) -> int:
    """One process per GPU: launched by ``torch.distributed.run`` with ``--nproc-per-node N`` the model is
    tensor-parallel over the N ranks; rank 0 serves HTTP and leads, the other ranks follow its scheduler."""
    import os

    ap = argparse.ArgumentParser(prog="eagle4_b200.serve")
    ap.add_argument("--model", required=True)
    ap.add_argument("--draft")
    ap.add_argument("--config", help="harness config JSON (inline or a path)")
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-len", type=int, default=8192)
    ap.add_argument("--no-spec", action="store_true", help="plain decode (the parity reference server)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--tp-backend", default="fused", choices=["fused", "torch"],
                    help="tensor-parallel collectives: fused peer-memory kernels, or NCCL through torch")
    ap.add_argument("--tokenizer", help="tokenizer directory for text prompts (default: the target directory, "
                                        "when it has one)")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="0: greedy (equal to plain greedy decoding); > 0: every request sampled at it "
                         "(tree rejection)")
    ap.add_argument("--seed", type=int, default=0, help="sampling seed")
    ap.add_argument("--tree", default="12,4,16", help="steps,top_k,draft_tokens: the largest tree a round may draft")
    ap.add_argument("--round-log", help="append one JSON line per served round to this file (rank 0)")
    ap.add_argument("--max-queue", type=int, help="waiting requests above which new ones get HTTP 503")
    ap.add_argument("--batch-prefill", action="store_true",
                    help="requests admitted in one step prefill in one target forward (groups of up to 8192 tokens)")
    ap.add_argument("--kv-tokens", type=int, help="KV cache positions shared by the running requests (default: "
                                                 "every row at --max-len; `eagle4-b200 plan` gives what fits)")
    ap.add_argument("--prefill-chunk", type=int, default=8192,
                    help="a longer prompt prefills in pieces of this many tokens (bounds the activations)")
    args = ap.parse_args(argv)
    if args.prefill_chunk < 1:
        ap.error("--prefill-chunk must be >= 1")

    from eagle4_b200.api import TreeSpec
    from eagle4_b200.cli import build_llm

    tp = lockstep = None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch
        import torch.distributed as dist

        from eagle4_b200.parallel.tp import TensorParallel
        from eagle4_b200.runtime.lockstep import Lockstep

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        tp = TensorParallel(backend=args.tp_backend, max_rows=max(256, args.max_batch * 32), max_cols=8192)
        lockstep = Lockstep()
    llm = build_llm(args.model, args.draft, max_batch=args.max_batch, max_len=args.max_len,
                    tree=TreeSpec(*(int(v) for v in args.tree.split(","))), config=args.config, tp=tp,
                    temperature=args.temperature, seed=args.seed, kv_tokens=args.kv_tokens)
    llm.engine.prefill_chunk = args.prefill_chunk
    if tp is not None:  # a dead or stalled rank is named by the heartbeat before the next round's collectives
        from eagle4_b200.parallel.health import process_group_heartbeat

        llm.engine.heartbeat = process_group_heartbeat()
    speculative = not args.no_spec
    tok_dir = args.tokenizer
    if tok_dir is None and os.path.isfile(os.path.join(args.model, "tokenizer_config.json")):
        tok_dir = args.model
    tokenizer = load_tokenizer(tok_dir)
    detokenize = (lambda ids: tokenizer.decode(ids)) if tokenizer is not None else None
    try:
        if lockstep is not None and not lockstep.leader:
            from eagle4_b200.runtime.lockstep import follow

            follow(llm.engine, lockstep, speculative=speculative, detokenize=detokenize,
                   batch_prefill=args.batch_prefill)
            return 0
        import uvicorn

        if args.round_log:
            from eagle4_b200.runtime.recorder import RoundRecorder

            llm.engine.recorder = RoundRecorder(args.round_log)
        batcher = Batcher(llm.engine, speculative=speculative, lockstep=lockstep, detokenize=detokenize,
                          max_queue=args.max_queue, batch_prefill=args.batch_prefill)
        try:
            uvicorn.run(make_app(batcher, tokenizer, os.path.basename(os.path.normpath(args.model))),
                        host=args.host, port=args.port)
        finally:
            batcher.close()
            if llm.engine.recorder is not None:
                llm.engine.recorder.flush()
        return 0 if batcher.failed is None else 1
    finally:
        if tp is not None:
            tp.close()
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    raise SystemExit(main())
