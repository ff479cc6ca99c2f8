"""Greedy parity between a plain-decode run and a speculative run, token for token, with fp32 arbitration.

    python -m eagle4_b200.tools.parity run --port 8000 --synthetic 20 --out spec.json       # a running server
    python -m eagle4_b200.tools.parity run --model tiny --no-spec --synthetic 20 --out plain.json   # in-process
    python -m eagle4_b200.tools.parity compare plain.json spec.json [--model tiny --seed 0] [--out report.json]
    python -m eagle4_b200.tools.parity rejudge report.json --out report.rejudged.json

``run`` generates greedily for every prompt (``--prompts FILE`` of ``{"id", "prompt_ids"}`` rows, or ``--synthetic N``
random prompts) and saves the output ids, the finish reason and the rounds each request took.

``compare`` finds, per prompt, the first position where the candidate's tokens leave the reference's, and gives
each prompt one status: ``identical``; ``length`` (one output is a strict prefix of the other); or, for a divergence,
``near_tie`` / ``fp32_pass`` / ``fp32_argmax`` / ``fail``, decided with the model (``--model``, the server's named
architecture and weight seed) at the common prefix:

* the bf16 model's log-probability gap from its best token to the candidate's token: at most ``--tie-gap`` (0.13,
  one bf16 ulp of a logit in [16, 32)) is a near tie;
* otherwise the same weights in fp32 (the PyTorch definitions, unfolded norms, on the host) give the two tokens'
  logits a, b: ``|a - b| <= 2`` bf16 ulps at ``max(|a|, |b|)`` passes (``fp32_pass``), the candidate's token being
  the fp32 argmax passes (``fp32_argmax``: the bf16 reference is the one that is off), anything else fails.

Without ``--model`` divergences are reported as ``diverged`` (not judged). The exit code is 1 when any prompt fails,
diverges unjudged, or differs in length. The tie gap, the tolerance and the bf16 spacing are the reference's
(``tools/greedy_parity.py``, ``tools/fp32_arbiter.py``) so that parity results of the two frameworks read alike.
``rejudge`` re-decides a saved report from the fp32 logits it recorded, without a model.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time
from dataclasses import asdict, dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

TIE_GAP = 0.13
TOLERANCE_ULPS = 2.0
PASSING = ("identical", "near_tie", "fp32_pass", "fp32_argmax")


def bf16_spacing(x: float) -> float:
    """Distance between adjacent bf16 values around ``|x|`` (8 significant bits): 2^(floor(log2|x|) - 7)."""
    x = abs(x)
    if x == 0.0 or not math.isfinite(x):
        return math.ldexp(1.0, -133)  # the smallest bf16 subnormal
    return math.ldexp(1.0, math.frexp(x)[1] - 8)


@dataclass
class Judgement:
    reference_token: int
    candidate_token: int
    reference_logit: float
    candidate_logit: float
    fp32_best_token: int
    fp32_best_logit: float
    spacing: float
    status: str


def judge(ref_tok: int, cand_tok: int, logit: Callable[[int], float], best: Tuple[int, float],
          tolerance_ulps: float = TOLERANCE_ULPS) -> Judgement:
    """The fp32 verdict on one divergence: within ``tolerance_ulps`` bf16 spacings passes, else the candidate passes
    only as the fp32 argmax (a tie at the top counts)."""
    a, b = float(logit(ref_tok)), float(logit(cand_tok))
    spacing = bf16_spacing(max(abs(a), abs(b)))
    if abs(a - b) <= tolerance_ulps * spacing:
        status = "fp32_pass"
    elif b >= best[1]:
        status = "fp32_argmax"
    else:
        status = "fail"
    return Judgement(ref_tok, cand_tok, a, b, int(best[0]), float(best[1]), spacing, status)


def first_divergence(a: Sequence[int], b: Sequence[int]) -> Optional[int]:
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None


# ------------------------------------------------------------------------------------------------ model scoring
class ModelScorer:
    """Logits at the end of a token prefix from a named synthetic architecture: the serving model (bf16, this
    package's kernels on a GPU) and the same weights in fp32 through the PyTorch definitions on the host."""

    def __init__(self, name: str, *, seed: int = 0, device: Optional[str] = None, max_len: int = 8192):
        import torch

        from eagle4_b200.api import LLM, NAMED
        from eagle4_b200.models import weights
        from eagle4_b200.models.target import TargetModel

        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.bf16 = LLM.synthetic(name, device=device, dtype=torch.bfloat16, seed=seed, draft=False, max_len=max_len)
        cfg = NAMED[name][0]()
        w = weights.init_target(cfg, device="cpu", dtype=torch.bfloat16, seed=seed)
        w32 = {k: v.float() if v.is_floating_point() else v for k, v in w.items()}
        target = TargetModel(cfg, w32, fold_norms=False)
        self.fp32 = LLM(target, None, max_len=max_len)  # same weights, fp32, host PyTorch definitions

    @staticmethod
    def _last_logits(llm, ids: Sequence[int]):
        import torch

        from eagle4_b200.models.target import RowBatch

        eng, dev = llm.engine, llm.target.device
        n = len(ids)
        eng.pages.release(0)
        eng.pages.reserve(0, n + 1)
        eng.tcache.reset_slot(0)
        pos = torch.arange(n, device=dev)
        z = torch.zeros(n, dtype=torch.int32, device=dev)
        rb = RowBatch(ids=torch.tensor(list(ids), dtype=torch.int64, device=dev), pos=pos, req=z,
                      write_slot=eng._slots(torch.tensor(0, device=dev), pos), ctx_start=z, ctx_len=(pos + 1).int(),
                      extra=torch.zeros(n, 1, dtype=torch.int32, device=dev), n_extra=z, parent=(pos - 1).int(),
                      state_slot=z, scan=True, max_keys=n)
        h, _ = llm.target.forward(rb, eng.tcache)
        return llm.target.logits(h[-1:]).float()[0].cpu()

    def gap(self, prefix: Sequence[int], token: int) -> float:
        """bf16 model: log-probability of its best token minus that of ``token`` at the end of ``prefix``."""
        lp = self._last_logits(self.bf16, prefix).double().log_softmax(-1)
        return float(lp.max() - lp[token])


def classify(prompt: Sequence[int], ref: Sequence[int], cand: Sequence[int], scorer: Optional[ModelScorer],
             tie_gap: float = TIE_GAP, tolerance_ulps: float = TOLERANCE_ULPS) -> dict:
    """One prompt's status with its evidence."""
    i = first_divergence(ref, cand)
    if i is None:
        return {"status": "identical" if len(ref) == len(cand) else "length", "index": None,
                "lengths": [len(ref), len(cand)]}
    row = {"index": i, "reference_token": int(ref[i]), "candidate_token": int(cand[i])}
    if scorer is None:
        return {**row, "status": "diverged"}
    prefix = list(prompt) + list(ref[:i])
    t0 = time.time()
    row["bf16_gap"] = scorer.gap(prefix, int(cand[i]))
    if row["bf16_gap"] <= tie_gap:
        return {**row, "status": "near_tie"}
    lg = scorer._last_logits(scorer.fp32, prefix)
    best = int(lg.argmax())
    j = judge(int(ref[i]), int(cand[i]), lambda t: lg[t], (best, float(lg[best])), tolerance_ulps)
    return {**row, "status": j.status, "fp32": asdict(j), "tolerance_ulps": tolerance_ulps,
            "seconds": time.time() - t0}


def rejudge_row(row: dict) -> dict:
    """A saved row decided again from its recorded fp32 logits (rows without them stay as they are)."""
    if "fp32" not in row:
        return dict(row)
    f = row["fp32"]
    logits = {f["reference_token"]: f["reference_logit"], f["candidate_token"]: f["candidate_logit"]}
    j = judge(f["reference_token"], f["candidate_token"], logits.__getitem__,
              (f["fp32_best_token"], f["fp32_best_logit"]), row.get("tolerance_ulps", TOLERANCE_ULPS))
    return {**row, "status": j.status, "fp32": asdict(j)}


def summary(rows: Dict[str, dict]) -> dict:
    counts: Dict[str, int] = {}
    for r in rows.values():
        counts[r["status"]] = counts.get(r["status"], 0) + 1
    return {"counts": counts, "passes": all(r["status"] in PASSING for r in rows.values()), "rows": rows}


# ------------------------------------------------------------------------------------------------ run
def _post(port: int):
    import requests

    def post(payload: dict) -> dict:
        r = requests.post(f"http://127.0.0.1:{port}/v1/generate", json=payload, timeout=3600)
        if not r.ok:
            raise RuntimeError(f"/v1/generate {r.status_code}: {r.text[:500]}")
        return r.json()

    return post


def run_prompts(prompts: List[Tuple[str, List[int]]], max_new_tokens: int, *, post=None, llm=None,
                speculative: bool = True) -> List[dict]:
    """Greedy outputs of every prompt, through an HTTP ``post`` or an in-process ``llm`` (one request at a time)."""
    results = []
    for pid, ids in prompts:
        t0 = time.time()
        if post is not None:
            r = post({"prompt_ids": ids, "max_new_tokens": max_new_tokens})
            out, reason, rounds = r["output_ids"], r.get("finish_reason"), r.get("meta", {}).get("rounds")
        else:
            from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

            sched = Scheduler(llm.engine, speculative=speculative)
            req = sched.submit(ids, RequestParams(max_new_tokens=max_new_tokens))
            sched.run()
            out, reason, rounds = req.output, req.finish_reason, req.rounds
        results.append({"id": pid, "prompt_ids": ids, "output_ids": out, "finish_reason": reason, "rounds": rounds,
                        "seconds": time.time() - t0})
    return results


def compare_docs(ref_doc: dict, cand_doc: dict, scorer: Optional[ModelScorer], tie_gap: float = TIE_GAP,
                 tolerance_ulps: float = TOLERANCE_ULPS) -> dict:
    ref = {r["id"]: r for r in ref_doc["results"]}
    rows = {}
    tokens = rounds = 0
    for c in cand_doc["results"]:
        r = ref[c["id"]]
        rows[c["id"]] = classify(r["prompt_ids"], r["output_ids"], c["output_ids"], scorer, tie_gap, tolerance_ulps)
        if c.get("rounds"):
            tokens += len(c["output_ids"])
            rounds += c["rounds"]
    out = {"tie_gap": tie_gap, "tolerance_ulps": tolerance_ulps, **summary(rows)}
    if rounds:
        out["tokens_per_round"] = tokens / rounds
    return out


def _host_or_gpu() -> dict:
    """In-process models: bf16 on a GPU, fp32 PyTorch definitions on a host without one."""
    import torch

    if torch.cuda.is_available():
        return {"device": "cuda", "dtype": torch.bfloat16}
    return {"device": "cpu", "dtype": torch.float32}


def _prompts(args) -> List[Tuple[str, List[int]]]:
    from eagle4_b200.tools import prompts

    if args.prompts:
        return prompts.load(args.prompts)
    return prompts.synthetic(args.synthetic, lo=args.min_len, hi=args.max_len, vocab=args.vocab, seed=args.seed)


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="eagle4_b200.tools.parity", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--port", type=int)
    r.add_argument("--model", help="in-process: a named synthetic architecture")
    r.add_argument("--no-spec", action="store_true")
    r.add_argument("--prompts")
    r.add_argument("--synthetic", type=int, default=20)
    r.add_argument("--min-len", type=int, default=64)
    r.add_argument("--max-len", type=int, default=512)
    r.add_argument("--vocab", type=int, default=32000)
    r.add_argument("--seed", type=int, default=0)
    r.add_argument("--max-new-tokens", type=int, default=256)
    r.add_argument("--out", required=True)
    c = sub.add_parser("compare")
    c.add_argument("reference")
    c.add_argument("candidate")
    c.add_argument("--model")
    c.add_argument("--seed", type=int, default=0)
    c.add_argument("--tie-gap", type=float, default=TIE_GAP)
    c.add_argument("--tolerance-ulps", type=float, default=TOLERANCE_ULPS)
    c.add_argument("--out")
    j = sub.add_parser("rejudge")
    j.add_argument("report")
    j.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    if args.cmd == "run":
        if (args.port is None) == (args.model is None):
            ap.error("run needs exactly one of --port and --model")
        llm = None
        if args.model:
            from eagle4_b200.api import LLM

            llm = LLM.synthetic(args.model, max_len=args.max_len + args.max_new_tokens + 64, **_host_or_gpu())
        t0 = time.time()
        res = run_prompts(_prompts(args), args.max_new_tokens, post=_post(args.port) if args.port else None, llm=llm,
                          speculative=not args.no_spec)
        with open(args.out, "w", encoding="utf-8") as f:
            json.dump({"source": f"port {args.port}" if args.port else args.model, "wall": time.time() - t0,
                       "results": res}, f)
        return 0
    if args.cmd == "compare":
        with open(args.reference, encoding="utf-8") as f:
            ref_doc = json.load(f)
        with open(args.candidate, encoding="utf-8") as f:
            cand_doc = json.load(f)
        scorer = ModelScorer(args.model, seed=args.seed) if args.model else None
        rep = compare_docs(ref_doc, cand_doc, scorer, args.tie_gap, args.tolerance_ulps)
    else:
        with open(args.report, encoding="utf-8") as f:
            rep = json.load(f)
        rep = {**rep, **summary({k: rejudge_row(v) for k, v in rep["rows"].items()})}
    for pid, row in rep["rows"].items():
        where = "" if row["index"] is None else (f" at {row['index']}: {row['reference_token']} vs "
                                                 f"{row['candidate_token']}")
        print(f"{pid:<12} {row['status']:<11}{where}")
    print(json.dumps(rep["counts"]), "passes" if rep["passes"] else "FAILS")
    if getattr(args, "out", None):
        with open(args.out, "w", encoding="utf-8") as f:
            json.dump(rep, f, indent=1)
    return 0 if rep["passes"] else 1


if __name__ == "__main__":
    sys.exit(main())
