"""Lossless sampling under speculation: speculative sampling must draw from the distribution plain sampling draws from.

    python -m eagle4_b200.tools.sampling_check run --model tiny --temperature 0.05 --no-spec --out plain.json
    python -m eagle4_b200.tools.sampling_check run --model tiny --temperature 0.05 --out spec.json
    python -m eagle4_b200.tools.sampling_check run --port 8000 --out spec.json          # a running server
    python -m eagle4_b200.tools.sampling_check compare plain.json spec.json [--alpha 0.01]

``run`` draws ``--samples`` continuations of ``--tokens`` tokens (3) for each of a few prompts and saves the token
ids. In process, a named synthetic architecture samples at ``--temperature`` with ``--batch`` identical prompts per
generate call, so the samples of one call share speculative rounds; against a server (``--port``, the
``/v1/completions`` API with token-id prompts) ``--concurrency`` requests run at a time and the server's own
temperature applies. The first token comes from the prefill's sampler, every later one from a verify round.

``compare`` tests, per prompt, that the candidate's draws come from the reference's distribution: the joint of the
first tokens, the marginal at every position, and each later token given the reference's most frequent prefix
(the draws of verify rounds from one context). Each test is a two-sample chi-square test of homogeneity in which
cells seen fewer than ``--min-cell`` times in both runs together are pooled; all tests run at the Bonferroni level
``--alpha / tests``; the total variation distance of each is printed. A sampler that verifies greedily, or at another
temperature, fails by a wide margin. Exit code 1 when a test rejects. The tests are the reference's
(``tools/sampling_check.py``) restricted to temperature sampling, which is the sampling this package's engine does.
"""

from __future__ import annotations

import argparse
import json
import sys
from collections import Counter
from typing import Dict, List, Optional, Sequence, Tuple


def synthetic_prompts(n: int, length: int, vocab: int, seed: int = 0) -> List[List[int]]:
    import torch

    g = torch.Generator().manual_seed(seed)
    return [torch.randint(1, vocab, (length,), generator=g).tolist() for _ in range(n)]


def sample_in_process(model: str, prompts: Sequence[Sequence[int]], *, samples: int, tokens: int, temperature: float,
                      speculative: bool, batch: int = 64, seed: int = 0, tree=(4, 2, 8), device: Optional[str] = None
                      ) -> List[List[List[int]]]:
    """``samples`` continuations of every prompt, ``batch`` rows per generate call."""
    import torch

    from eagle4_b200.api import LLM, TreeSpec

    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    dtype = torch.bfloat16 if device == "cuda" else torch.float32
    length = max(len(p) for p in prompts)
    llm = LLM.synthetic(model, device=device, dtype=dtype, tree=TreeSpec(*tree), max_batch=batch,
                        max_len=length + tokens + 64, temperature=temperature, sample_seed=seed)
    out = []
    for p in prompts:
        rows: List[List[int]] = []
        while len(rows) < samples:
            b = min(batch, samples - len(rows))
            ids = torch.tensor(list(p), dtype=torch.int64)[None].expand(b, -1).contiguous()
            rows += llm.generate(ids, tokens, speculative=speculative).tolist()
        out.append(rows)
    return out


def sample_server(port: int, prompts: Sequence[Sequence[int]], *, samples: int, tokens: int, concurrency: int = 16,
                  host: str = "127.0.0.1") -> List[List[List[int]]]:
    import requests
    from concurrent.futures import ThreadPoolExecutor

    url = f"http://{host}:{port}/v1/completions"

    def one(prompt):
        r = requests.post(url, json={"prompt": list(prompt), "max_tokens": tokens, "ignore_eos": True}, timeout=600)
        r.raise_for_status()
        return r.json()["choices"][0]["token_ids"][:tokens]

    with ThreadPoolExecutor(concurrency) as pool:
        return [list(pool.map(one, [p] * samples)) for p in prompts]


# ------------------------------------------------------------------------------------------------ statistics
def homogeneity(a: Counter, b: Counter, min_cell: int = 10) -> Optional[Tuple[float, int, float, float]]:
    """Two-sample chi-square test of homogeneity over the cells of ``a`` and ``b`` (rare cells pooled): (statistic,
    degrees of freedom, p-value, total variation distance), or None when fewer than two cells remain."""
    from scipy.stats import chi2_contingency

    na, nb = sum(a.values()), sum(b.values())
    if not na or not nb:
        return None
    keys = sorted(set(a) | set(b), key=repr)
    tvd = 0.5 * sum(abs(a[k] / na - b[k] / nb) for k in keys)
    kept = [k for k in keys if a[k] + b[k] >= min_cell]
    rows = [[a[k] for k in kept], [b[k] for k in kept]]
    rest = [na - sum(rows[0]), nb - sum(rows[1])]
    if rest[0] + rest[1] > 0:
        rows[0].append(rest[0])
        rows[1].append(rest[1])
    if len(rows[0]) < 2:
        return None
    stat, p, dof, _ = chi2_contingency(rows, correction=False)
    return float(stat), int(dof), float(p), float(tvd)


def tests_of(ref: Sequence[Sequence[int]], cand: Sequence[Sequence[int]], tokens: int) -> Dict[str, Tuple[Counter,
                                                                                                          Counter]]:
    """The distributions compared for one prompt: ``joint``, ``pos<j>`` marginals, ``given<j>`` conditionals on the
    reference's most frequent prefix of length ``j``."""
    out = {"joint": (Counter(tuple(s[:tokens]) for s in ref), Counter(tuple(s[:tokens]) for s in cand))}
    for j in range(tokens):
        out[f"pos{j}"] = (Counter(s[j] for s in ref), Counter(s[j] for s in cand))
    for j in range(1, tokens):
        prefix = Counter(tuple(s[:j]) for s in ref).most_common(1)[0][0]
        out[f"given{j}"] = (Counter(s[j] for s in ref if tuple(s[:j]) == prefix),
                            Counter(s[j] for s in cand if tuple(s[:j]) == prefix))
    return out


def compare(ref: dict, cand: dict, *, alpha: float = 0.01, min_cell: int = 10, log=print) -> bool:
    """True when no test rejects at the Bonferroni-corrected level."""
    tokens = min(ref["meta"]["tokens"], cand["meta"]["tokens"])
    results = []
    for i, (rp, cp) in enumerate(zip(ref["prompts"], cand["prompts"])):
        if rp["prompt_ids"] != cp["prompt_ids"]:
            raise ValueError(f"prompt {i} differs between the runs")
        for name, (a, b) in tests_of(rp["samples"], cp["samples"], tokens).items():
            r = homogeneity(a, b, min_cell)
            if r is not None:
                results.append((i, name, sum(a.values()), sum(b.values())) + r)
    if not results:
        raise ValueError("no test had two cells with enough draws: take more samples or a lower temperature")
    level = alpha / len(results)
    ok = True
    log(f"{len(results)} tests at alpha {alpha} / {len(results)} = {level:.2e}")
    log(f"{'prompt':>6} {'test':>8} {'n_ref':>6} {'n_cand':>6} {'chi2':>9} {'dof':>4} {'p':>9} {'tvd':>6}")
    for i, name, na, nb, stat, dof, p, tvd in results:
        bad = p < level
        ok &= not bad
        log(f"{i:>6} {name:>8} {na:>6} {nb:>6} {stat:>9.2f} {dof:>4} {p:>9.2e} {tvd:>6.3f}{'  REJECT' if bad else ''}")
    return ok


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="eagle4_b200.tools.sampling_check")
    sub = ap.add_subparsers(dest="cmd", required=True)
    run = sub.add_parser("run")
    run.add_argument("--out", required=True)
    run.add_argument("--model", default="tiny", help="named synthetic architecture (in-process runs)")
    run.add_argument("--port", type=int, help="sample a running server instead")
    run.add_argument("--prompts", type=int, default=3)
    run.add_argument("--prompt-len", type=int, default=16)
    run.add_argument("--samples", type=int, default=512)
    run.add_argument("--tokens", type=int, default=3)
    run.add_argument("--temperature", type=float, default=1.0)
    run.add_argument("--batch", type=int, default=64)
    run.add_argument("--concurrency", type=int, default=16)
    run.add_argument("--seed", type=int, default=0)
    run.add_argument("--no-spec", action="store_true")
    cmp_ = sub.add_parser("compare")
    cmp_.add_argument("reference")
    cmp_.add_argument("candidate")
    cmp_.add_argument("--alpha", type=float, default=0.01)
    cmp_.add_argument("--min-cell", type=int, default=10)
    args = ap.parse_args(argv)
    if args.cmd == "run":
        from eagle4_b200.api import NAMED

        vocab = NAMED[args.model][0]().vocab_size if args.model in NAMED else 32000
        prompts = synthetic_prompts(args.prompts, args.prompt_len, vocab, args.seed)
        if args.port:
            samples = sample_server(args.port, prompts, samples=args.samples, tokens=args.tokens,
                                    concurrency=args.concurrency)
        else:
            samples = sample_in_process(args.model, prompts, samples=args.samples, tokens=args.tokens,
                                        temperature=args.temperature, speculative=not args.no_spec, batch=args.batch,
                                        seed=args.seed)
        meta = {"tokens": args.tokens, "temperature": args.temperature, "speculative": not args.no_spec,
                "source": f"port {args.port}" if args.port else args.model}
        with open(args.out, "w", encoding="utf-8") as f:
            json.dump({"meta": meta, "prompts": [{"id": i, "prompt_ids": p, "samples": s}
                                                 for i, (p, s) in enumerate(zip(prompts, samples))]}, f)
        return 0
    with open(args.reference, encoding="utf-8") as f:
        ref = json.load(f)
    with open(args.candidate, encoding="utf-8") as f:
        cand = json.load(f)
    return 0 if compare(ref, cand, alpha=args.alpha, min_cell=args.min_cell) else 1


if __name__ == "__main__":
    sys.exit(main())
