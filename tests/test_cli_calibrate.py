"""CLI, host checks and the engine calibration driver (tiny model on CPU; the GPU run uses the same code)."""

import json
import os

import pytest
import torch

from eagle4_b200 import cli, compat
from eagle4_b200.plugins import contract
from tests.helpers import word_tokenizer


def test_cli_dry_run(capsys, tmp_path):
    assert cli.main(["calibrate", "--model", "tiny", "--output", str(tmp_path / "cal"), "--dry-run"]) == 0
    out = capsys.readouterr().out
    assert '"batch_sizes"' in out and "eagle4_b200.serve" in out
    assert not (tmp_path / "cal").exists()
    with pytest.raises(SystemExit):
        cli.main(["calibrate", "--model", "tiny", "--batch-sizes", "0,1"])


def test_compat_reports_hosts(capsys):
    compat.main([])
    out = capsys.readouterr().out
    for name in ("sglang", "vllm", "tokenspeed"):
        assert name in out


def test_contract_checks_fake_host(tmp_path, monkeypatch):
    pkg = tmp_path / "fakehost"
    pkg.mkdir()
    (pkg / "__init__.py").write_text(
        "class Algo:\n"
        "    def hook(self, a, b): pass\n"
        "    def call(self, a, b, c=1): pass\n"
        "class Data:\n"
        "    field_x = 1\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    H = contract.Hook
    ok = [H("fakehost:Algo.hook", ("a", "b"), contract.OVERRIDE), H("fakehost:Algo.call", ("a", "b")),
          H("fakehost:Data.field_x", (), contract.FIELD), H("fakehost:Nope.x", (), contract.CALL, optional=True)]
    assert contract.problems(ok) == []
    bad = [H("fakehost:Algo.hook", ("a",), contract.OVERRIDE), H("fakehost:Algo.call", ("z",)),
           H("fakehost:Data.missing", (), contract.FIELD), H("fakehost:Gone.x")]
    assert len(contract.problems(bad)) == 4


def test_calibrate_tiny_on_cpu(tmp_path):
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.core.cost_table import load_cost_tables
    from eagle4_b200.runtime.calibrate import calibrate

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=512)
    problems = calibrate(llm.engine, str(tmp_path), batch_sizes=[1], context_step=64, context_stop=256, repeats=2,
                         progress=lambda s: None)
    assert set(problems) == {1}
    tables = load_cost_tables(os.path.join(tmp_path, "cost"))
    t = tables[1]
    assert len(t.intervals) == 3 and t.intervals[0].target.value[0] > 0
    with open(os.path.join(tmp_path, "config", "measure_config.json")) as f:
        assert json.loads(f.readline())["batch_size"] == 1


def test_serve_app_round_trip():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.serve import Batcher, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2, max_len=256)
    prompt = list(range(1, 20))
    b = Batcher(llm.engine)
    try:
        client = TestClient(make_app(b))
        r = client.post("/v1/generate", json={"prompt_ids": prompt, "max_new_tokens": 6})
        assert r.status_code == 200 and r.json()["finish_reason"] == "length"
        out = r.json()["output_ids"]
        assert len(out) == 6
        stop = out[2]
        s = client.post("/v1/generate", json={"prompt_ids": prompt, "max_new_tokens": 6, "stop_token_ids": [stop]})
        assert s.json()["finish_reason"] == "stop"
        assert s.json()["output_ids"] == out[:out.index(stop) + 1]
        assert client.post("/v1/generate", json={"prompt_ids": [], "max_new_tokens": 6}).status_code in (400, 422)
        assert client.get("/health").json()["rounds"] >= 1
    finally:
        b.stop.set()
        b.thread.join()
    plain = llm.generate([torch.tensor(prompt)], 6, speculative=False)[0].tolist()
    assert plain == out


def test_chain_calibration_on_cpu(tmp_path):
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.core.chain_width import chain_widths, load_accept_profile, load_round_times
    from eagle4_b200.runtime.calibrate import calibrate_chain

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(3, 1, 4), max_len=256,
                        config='{"mode": "serve"}')
    calibrate_chain(llm.engine, str(tmp_path), batch_sizes=[1], prompt_len=16, new_tokens=6, progress=lambda s: None)
    rounds = load_round_times(str(tmp_path))
    assert set(rounds[1]) == {1, 2, 3, 4}
    assert load_accept_profile(str(tmp_path)) is not None
    assert chain_widths(str(tmp_path), 4, 8)[0][0] == 1


def test_tp_dry_run_prints_the_worker_launch_and_a_tensor_parallel_serve_command(capsys, tmp_path):
    out_dir = tmp_path / "cal"
    assert cli.main(["calibrate", "--model", "tiny", "--output", str(out_dir), "--tp", "2", "--dry-run"]) == 0
    lines = capsys.readouterr().out.strip().splitlines()
    launch, serve = lines[-2], lines[-1]
    assert "torch.distributed.run" in launch and "--nproc-per-node 2" in launch and "--worker" in launch
    assert "--master-addr 127.0.0.1" in launch and str(out_dir) in launch
    assert "torch.distributed.run" in serve and "eagle4_b200.serve" in serve
    assert not out_dir.exists()


def _group_alive(pid: int) -> bool:
    try:
        with open(f"/proc/{pid}/status") as f:
            return not any(line.startswith("State:") and "Z" in line.split()[1] for line in f)
    except FileNotFoundError:
        return False


@pytest.mark.parametrize("case", ["timeout", "failure"])
def test_supervisor_ends_the_whole_process_group(tmp_path, case):
    import sys
    import time

    from eagle4_b200.runtime.supervise import supervise

    pid_file = tmp_path / "grandchild"
    code = ("import subprocess, sys, time\n"
            "p = subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(120)'])\n"
            f"open({str(pid_file)!r}, 'w').write(str(p.pid))\n"
            + ("time.sleep(120)\n" if case == "timeout" else "time.sleep(0.5)\nraise SystemExit(3)\n"))
    t0 = time.monotonic()
    out = supervise([sys.executable, "-c", code], timeout=5.0, grace=2.0)
    assert time.monotonic() - t0 < 30
    if case == "timeout":
        assert out.timed_out and out.code == 124 and not out.ok
    else:
        assert out.code == 3 and not out.timed_out and not out.ok
    grandchild = int(pid_file.read_text())
    for _ in range(50):
        if not _group_alive(grandchild):
            break
        time.sleep(0.1)
    assert not _group_alive(grandchild)


def test_supervisor_success():
    import sys

    from eagle4_b200.runtime.supervise import supervise

    assert supervise([sys.executable, "-c", "pass"], timeout=60).ok


def _tp_calibrate_worker(rank, world, port, path, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    try:
        from eagle4_b200.api import LLM, TreeSpec
        from eagle4_b200.parallel.tp import TensorParallel
        from eagle4_b200.runtime.calibrate import calibrate

        tp = TensorParallel(backend="torch")
        llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=512, tp=tp)
        seen = []
        problems = calibrate(llm.engine, path, batch_sizes=[1], context_step=64, context_stop=128, repeats=2,
                             progress=seen.append)
        out[rank] = {"problems": problems, "messages": len(seen), "files": os.path.isdir(os.path.join(path, "cost"))}
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_calibration_rank0_writes_every_rank_checks(tmp_path):
    import socket

    import torch.multiprocessing as mp

    from eagle4_b200.core.cost_table import load_cost_tables

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_tp_calibrate_worker, args=(2, port, str(tmp_path), out), nprocs=2, start_method="spawn",
                           join=True)
        res = dict(out)
    assert res[0]["problems"] == res[1]["problems"] and set(res[0]["problems"]) == {1}
    assert res[0]["messages"] > 0 and res[1]["messages"] == 0 and res[1]["files"]
    assert 1 in load_cost_tables(os.path.join(tmp_path, "cost"))


def test_completions_text_stop_strings_and_metrics():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.serve import Batcher, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2, max_len=256)
    tok = word_tokenizer(4096)
    prompt_ids = list(range(5, 25))
    plain = llm.generate([torch.tensor(prompt_ids)], 8, speculative=False)[0].tolist()
    b = Batcher(llm.engine, detokenize=lambda ids: tok.decode(ids))
    try:
        client = TestClient(make_app(b, tok, "tiny"))
        text = " ".join(f"<{i}>" for i in prompt_ids)
        r = client.post("/v1/completions", json={"prompt": text, "max_tokens": 8, "ignore_eos": True}).json()
        assert r["choices"][0]["token_ids"] == plain and r["choices"][0]["finish_reason"] == "length"
        assert r["choices"][0]["text"] == tok.decode(plain) and r["usage"]["prompt_tokens"] == 20
        stop = f"<{plain[3]}>"
        first = plain.index(plain[3])
        s = client.post("/v1/completions", json={"prompt": prompt_ids, "max_tokens": 8, "stop": stop,
                                                  "ignore_eos": True}).json()
        assert s["choices"][0]["finish_reason"] == "stop"
        assert s["choices"][0]["token_ids"] == plain[:first + 1]
        full = tok.decode(plain[:first + 1])
        assert s["choices"][0]["text"] == full[:full.index(stop)]  # the stop string is cut from the text
        bad = client.post("/v1/completions", json={"prompt": prompt_ids, "max_tokens": 4, "temperature": 0.7})
        assert bad.status_code == 400
        m = client.get("/metrics").text
        assert "eagle4_requests_total 2.0" in m and "eagle4_generated_tokens_total" in m
        assert 'eagle4_accepted_per_request_round_total{tokens="' in m
        assert "eagle4_draft_kv_holes_total" in m
    finally:
        b.close(timeout=60)


def test_completions_need_a_tokenizer_for_text():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.serve import Batcher, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=1, max_len=256)
    b = Batcher(llm.engine)
    try:
        client = TestClient(make_app(b))
        assert client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 2}).status_code == 400
        assert client.post("/v1/completions", json={"prompt": [3, 4], "max_tokens": 2, "stop": "x"}).status_code == 400
        ok = client.post("/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 2}).json()
        assert ok["choices"][0]["text"] is None and len(ok["choices"][0]["token_ids"]) == 2
    finally:
        b.close(timeout=60)


def _events(resp):
    import json as json_

    out = []
    for line in resp.iter_lines():
        line = line if isinstance(line, str) else line.decode()
        if line.startswith("data: "):
            out.append(line[6:] if line[6:] == "[DONE]" else json_.loads(line[6:]))
    return out


def test_streamed_completions_and_chat():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.serve import Batcher, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2, max_len=256)
    tok = word_tokenizer(4096)
    tok.chat_template = ("{% for m in messages %}<{{ loop.index + 10 }}> {{ m['content'] }} {% endfor %}"
                         "{% if add_generation_prompt %}<9>{% endif %}")
    prompt_ids = list(range(30, 45))
    plain = llm.generate([torch.tensor(prompt_ids)], 10, speculative=False)[0].tolist()
    b = Batcher(llm.engine, detokenize=lambda ids: tok.decode(ids))
    try:
        client = TestClient(make_app(b, tok, "tiny"))
        with client.stream("POST", "/v1/completions", json={"prompt": prompt_ids, "max_tokens": 10,
                                                             "ignore_eos": True, "stream": True}) as r:
            ev = _events(r)
        assert ev[-1] == "[DONE]" and ev[-2]["choices"][0]["finish_reason"] == "length"
        chunks = ev[:-1]
        assert sum((c["choices"][0]["token_ids"] for c in chunks), []) == plain
        assert "".join(c["choices"][0]["text"] or "" for c in chunks) == tok.decode(plain)
        assert ev[-2]["usage"]["completion_tokens"] == 10
        # a stop string inside the stream: the streamed text never shows it
        stop = f"<{plain[4]}>"
        with client.stream("POST", "/v1/completions", json={"prompt": prompt_ids, "max_tokens": 10, "stop": stop,
                                                             "ignore_eos": True, "stream": True}) as r:
            ev = _events(r)
        text = "".join(c["choices"][0]["text"] or "" for c in ev[:-1])
        full = tok.decode(plain[:plain.index(plain[4]) + 1])
        assert text == full[:full.index(stop)] and ev[-2]["choices"][0]["finish_reason"] == "stop"
        # chat: the template's prompt, the same tokens as the equivalent completion
        msgs = [{"role": "user", "content": "<30> <31> <32>"}]
        want_ids = list(tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True)["input_ids"])
        c = client.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 5, "ignore_eos": True}).json()
        cmp = client.post("/v1/completions", json={"prompt": want_ids, "max_tokens": 5, "ignore_eos": True}).json()
        assert c["object"] == "chat.completion" and c["choices"][0]["message"]["content"] == cmp["choices"][0]["text"]
        assert c["usage"]["prompt_tokens"] == len(want_ids)
        with client.stream("POST", "/v1/chat/completions", json={"messages": msgs, "max_tokens": 5,
                                                                  "ignore_eos": True, "stream": True}) as r:
            ev = _events(r)
        assert "".join(e["choices"][0]["delta"].get("content", "") for e in ev[:-1]) == cmp["choices"][0]["text"]
    finally:
        b.close(timeout=60)


def test_memory_plan_matches_the_engine_allocations(capsys):
    from eagle4_b200.api import NAMED, LLM, TreeSpec
    from eagle4_b200.runtime.memory import plan

    tcfg = NAMED["tiny"][0]()
    dcfg = NAMED["tiny"][1](tcfg)
    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=3, max_len=200,
                        kv_tokens=1024)
    eng = llm.engine

    def nbytes(ts):
        seen, n = set(), 0
        for t in ts:
            if torch.is_tensor(t) and id(t) not in seen:
                seen.add(id(t))
                n += t.numel() * t.element_size()
        return n

    p = plan(tcfg, dcfg, max_batch=3, max_len=200, kv_tokens=1024, tree=(4, 2, 8), dtype=torch.float32,
             reserve_gb=0)
    assert p.state_bytes == nbytes(eng.tcache.conv + eng.tcache.ssm)
    slots = eng.tcache.k[0].shape[0]
    kv = nbytes(eng.tcache.k + eng.tcache.v) + nbytes([eng.dcache.k, eng.dcache.v])
    assert p.kv_bytes_per_token * slots == kv
    model_w = nbytes(list(llm.target.w.values()) + list(llm.draft.w.values()))
    assert abs(p.weights - model_w) <= 0.02 * model_w  # the engine may fold norms into projection copies
    assert p.kv_tokens_within(p.weights + p.state_bytes + p.prefill + 10 * p.kv_bytes_per_token * 1024) == 10 * 1024
    # the prefill transient: one piece through the widest projection and the aux rows of a max_len prompt
    widest = max(t.shape[0] for n, t in llm.target.w.items() if t.dim() == 2 and n not in ("embed", "lm_head"))
    assert p.prefill == (200 * (widest + 4 * tcfg.hidden_size) + 200 * dcfg.num_aux * tcfg.hidden_size) * 4
    assert cli.main(["plan", "--model", "qwen3.8-27b", "--max-batch", "64", "--max-len", "8192"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["fits"] and 50 < out["weights"] < 60 and out["max_kv_tokens"] > out["kv_tokens"]
    assert cli.main(["plan", "--model", "qwen3.8-27b", "--max-batch", "512", "--max-len", "32768"]) == 1


def test_queue_limit_and_models_endpoint():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.runtime.scheduler import RequestParams
    from eagle4_b200.serve import Batcher, QueueFull, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=1, max_len=256)
    b = Batcher(llm.engine, max_queue=0)
    try:
        client = TestClient(make_app(b, None, "tiny"))
        assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
        r = client.post("/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 2})
        assert r.status_code == 503
        with client.stream("POST", "/v1/completions", json={"prompt": [3, 4], "max_tokens": 2, "stream": True}) as s:
            assert s.status_code == 503
        assert b.counts["refused"] == 2
    finally:
        b.close(timeout=60)
    # a burst larger than the queue: some run, the rest are refused, none is lost
    b = Batcher(llm.engine, max_queue=1)
    try:
        futs = [b.submit([5, 6, 7], RequestParams(max_new_tokens=3)) for _ in range(6)]
        results = []
        for f in futs:
            try:
                results.append(len(f.result(timeout=120).output))
            except QueueFull:
                results.append("full")
        assert results.count(3) >= 1 and all(r in (3, "full") for r in results)
    finally:
        b.close(timeout=60)


def test_n_choices_sample_independently():
    from fastapi.testclient import TestClient

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.serve import Batcher, make_app

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=4, max_len=256,
                        temperature=0.05, sample_seed=3)
    b = Batcher(llm.engine)
    try:
        client = TestClient(make_app(b, None, "tiny"))
        r = client.post("/v1/completions", json={"prompt": list(range(5, 17)), "max_tokens": 6, "n": 4}).json()
        assert [c["index"] for c in r["choices"]] == [0, 1, 2, 3]
        outs = [tuple(c["token_ids"]) for c in r["choices"]]
        assert all(len(o) == 6 for o in outs) and len(set(outs)) > 1  # independent draws
        assert r["usage"]["completion_tokens"] == 24
        bad = client.post("/v1/completions", json={"prompt": [5, 6], "max_tokens": 2, "n": 2, "stream": True})
        assert bad.status_code == 400
    finally:
        b.close(timeout=60)


def test_calibration_report(tmp_path, capsys):
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.core.chain_width import merge_tree_rounds
    from eagle4_b200.core.live_costs import CostKey
    from eagle4_b200.runtime.calibrate import calibrate

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=512)
    key = CostKey(gpu="cpu", gpu_count=1, model="tiny", draft="", engine="eagle4_b200", dtype="float32")
    calibrate(llm.engine, str(tmp_path), batch_sizes=[1], context_step=64, context_stop=128, repeats=2, key=key,
              progress=lambda s: None)
    merge_tree_rounds(str(tmp_path), [{"batch_size": 1, "width": 8, "round_us": 9000.0, "accept": 2.0, "count": 9},
                                      {"batch_size": 1, "width": 4, "round_us": 5000.0, "accept": 1.9, "count": 9}])
    rep = cli.calibration_report(tmp_path, max_verify_width=8)
    assert rep["key"]["model"] == "tiny" and set(rep["cost_tables"]) == {"1"}
    assert rep["cost_tables"]["1"]["intervals"] >= 1 and rep["tree_rounds"] == [1]
    assert rep["accept_profile"] is None and rep["chain_schedule"] is None
    code = cli.main(["report", str(tmp_path), "--max-verify-width", "8"])
    out = json.loads(capsys.readouterr().out)
    assert out["data_path"] == str(tmp_path) and code in (0, 1)
    assert cli.main(["report", str(tmp_path / "missing")]) == 1
