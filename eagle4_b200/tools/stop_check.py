"""Per-request stop conditions under batched speculation: one batch mixes every kind of stop.

    python -m eagle4_b200.tools.stop_check --port 8000 --concurrency 16 --out stop_spec.json [--reference plain.json]
    python -m eagle4_b200.tools.stop_check --model tiny --concurrency 8 --out stop.json          # in-process

Sends ``--concurrency`` greedy requests at once, so they share rounds, cycling four kinds:

* ``ignore_eos``: carries the EOS id with ``ignore_eos``; must run to ``--max-new-tokens``;
* ``stop_token``: ``stop_token_ids=[S]``; S may only be the last output token, and only a stop on S ends it early;
* ``eos``: ``eos_token_id=E``; E may only be the last output token;
* ``plain``: no stop condition; must run to ``--max-new-tokens``.

Every request must end for its own reason only (finish reason and last token agree with its kind). A speculative round
accepts several tokens per request, so an engine that checked one request's stop set for the whole batch, or only the
last accepted token, fails here. S and E default to the two most frequent tokens of a probe pass over the prompts
(random-weight models have no meaningful EOS), so stops really happen mid-round. With ``--reference`` (the output
file of a plain-decode server) rows whose tokens equal the reference's are counted. Exit code 1 on any violation.
(The reference's ``tools/stop_check.py`` checks the same conditions against SGLang / vLLM / TokenSpeed servers.)
"""

from __future__ import annotations

import argparse
import collections
import concurrent.futures
import json
import sys
from typing import Callable, Dict, List, Optional, Sequence, Tuple

KINDS = ("ignore_eos", "stop_token", "eos", "plain")


def request_for(kind: str, prompt: List[int], max_new: int, stop: int, eos: int) -> dict:
    body = {"prompt_ids": prompt, "max_new_tokens": max_new}
    if kind == "ignore_eos":
        body.update(eos_token_id=eos, ignore_eos=True)
    elif kind == "stop_token":
        body.update(stop_token_ids=[stop])
    elif kind == "eos":
        body.update(eos_token_id=eos)
    return body


def violations(kind: str, out: Sequence[int], reason: Optional[str], max_new: int, stop: int, eos: int) -> List[str]:
    """What is wrong with one finished request of ``kind`` (empty when it ended for its own reason only)."""
    bad = []
    if not out:
        return ["empty output"]
    if len(out) > max_new:
        bad.append(f"{len(out)} tokens > max_new_tokens {max_new}")
    last = out[-1]
    ender = {"stop_token": stop, "eos": eos}.get(kind)
    if ender is not None:
        if ender in out[:-1]:
            bad.append(f"{kind} token {ender} inside the output at {out.index(ender)}")
        if last == ender:
            want = "stop" if kind == "stop_token" else "eos"
            if reason != want:
                bad.append(f"ended on its {kind} token with reason {reason!r}")
        elif len(out) != max_new or reason != "length":
            bad.append(f"ended early ({len(out)} tokens, reason {reason!r}) without its {kind} token")
    else:
        if len(out) != max_new or reason != "length":
            bad.append(f"{kind} ended at {len(out)} tokens with reason {reason!r}")
    return bad


def pick_enders(outputs: Sequence[Sequence[int]]) -> Tuple[int, int]:
    """The two most frequent output tokens of a probe pass (stop token, EOS)."""
    counts = collections.Counter(t for o in outputs for t in o[1:])
    common = [t for t, _ in counts.most_common(2)]
    if len(common) < 2:
        raise ValueError("the probe outputs have fewer than two distinct tokens")
    return common[0], common[1]


def check(prompts: List[Tuple[str, List[int]]], post: Callable[[dict], dict], *, concurrency: int, max_new: int,
          stop: Optional[int] = None, eos: Optional[int] = None, reference: Optional[Dict[str, List[int]]] = None,
          probe: Optional[Callable[[dict], dict]] = None) -> dict:
    """Run the mixed batch through ``post`` (payload -> reply with ``output_ids`` and ``finish_reason``)."""
    if stop is None or eos is None:
        outs = [(probe or post)({"prompt_ids": p, "max_new_tokens": max_new})["output_ids"] for _, p in prompts]
        stop, eos = pick_enders(outs)
    jobs = [(pid, KINDS[i % len(KINDS)], p) for i, (pid, p) in enumerate(prompts)]
    with concurrent.futures.ThreadPoolExecutor(max_workers=concurrency) as ex:
        futs = [ex.submit(post, request_for(kind, p, max_new, stop, eos)) for _, kind, p in jobs]
        replies = []
        for f in futs:
            try:
                replies.append(f.result())
            except Exception as e:  # noqa: BLE001 - a failed request is a violation
                replies.append({"error": repr(e)})
    rows, n_bad, equal = [], 0, 0
    for (pid, kind, _), r in zip(jobs, replies):
        if "error" in r:
            bad = [r["error"]]
            out, reason = [], None
        else:
            out, reason = r["output_ids"], r.get("finish_reason")
            bad = violations(kind, out, reason, max_new, stop, eos)
        n_bad += bool(bad)
        row = {"id": pid, "kind": kind, "tokens": len(out), "finish_reason": reason, "violations": bad,
               "output_ids": out}
        if reference is not None and pid in reference:
            ref = reference[pid]
            # the plain-decode reference ran without stops: a stopped row must equal its prefix
            row["equals_reference"] = list(out) == list(ref[:len(out)])
            equal += row["equals_reference"]
        rows.append(row)
    rep = {"stop_token": stop, "eos": eos, "requests": len(rows), "violations": n_bad, "rows": rows}
    if reference is not None:
        rep["equal_to_reference"] = equal
    return rep


def main(argv: Optional[List[str]] = None) -> int:
    from eagle4_b200.tools import parity, prompts as prompt_sets

    ap = argparse.ArgumentParser(prog="eagle4_b200.tools.stop_check", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--port", type=int)
    ap.add_argument("--model", help="in-process server over a named synthetic architecture")
    ap.add_argument("--prompts")
    ap.add_argument("--synthetic", type=int, default=32)
    ap.add_argument("--min-len", type=int, default=32)
    ap.add_argument("--max-len", type=int, default=256)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--concurrency", type=int, default=16)
    ap.add_argument("--max-new-tokens", type=int, default=64)
    ap.add_argument("--stop-token", type=int)
    ap.add_argument("--eos", type=int)
    ap.add_argument("--reference", help="a parity run output of a plain-decode server (same prompts)")
    ap.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    if (args.port is None) == (args.model is None):
        ap.error("exactly one of --port and --model")
    ps = prompt_sets.load(args.prompts) if args.prompts else prompt_sets.synthetic(
        args.synthetic, lo=args.min_len, hi=args.max_len, vocab=args.vocab, seed=args.seed)
    batcher = None
    if args.port is not None:
        post = parity._post(args.port)
    else:
        from eagle4_b200.api import LLM
        from eagle4_b200.runtime.scheduler import RequestParams
        from eagle4_b200.serve import Batcher

        llm = LLM.synthetic(args.model, max_batch=args.concurrency,
                            max_len=args.max_len + args.max_new_tokens + 64, **parity._host_or_gpu())
        batcher = Batcher(llm.engine)

        def post(body: dict) -> dict:
            params = RequestParams(max_new_tokens=body["max_new_tokens"],
                                   stop_token_ids=tuple(body.get("stop_token_ids", ())),
                                   eos_token_id=body.get("eos_token_id"), ignore_eos=body.get("ignore_eos", False))
            req = batcher.submit(body["prompt_ids"], params).result()
            return {"output_ids": req.output, "finish_reason": req.finish_reason}

    reference = None
    if args.reference:
        with open(args.reference, encoding="utf-8") as f:
            reference = {r["id"]: r["output_ids"] for r in json.load(f)["results"]}
    try:
        rep = check(ps, post, concurrency=args.concurrency, max_new=args.max_new_tokens, stop=args.stop_token,
                    eos=args.eos, reference=reference)
    finally:
        if batcher is not None:
            batcher.stop.set()
    with open(args.out, "w", encoding="utf-8") as f:
        json.dump(rep, f, indent=1)
    for row in rep["rows"]:
        if row["violations"]:
            print(row["id"], row["kind"], "; ".join(row["violations"]))
    tail = f", {rep['equal_to_reference']} equal to the reference" if reference is not None else ""
    print(f"{rep['requests']} requests (stop token {rep['stop_token']}, eos {rep['eos']}): "
          f"{rep['violations']} violating{tail}")
    return 1 if rep["violations"] else 0


if __name__ == "__main__":
    sys.exit(main())
