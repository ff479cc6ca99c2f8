"""CLI, host checks and the engine calibration driver (tiny model on CPU; the GPU run uses the same code)."""

import json
import os

import pytest
import torch

from eagle4_b200 import cli, compat
from eagle4_b200.plugins import contract


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
