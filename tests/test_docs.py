"""The user documentation names only flags the commands accept (docs/*.md against each parser's --help)."""

import pathlib
import re

import pytest

DOCS = pathlib.Path(__file__).resolve().parent.parent / "docs"


def _help(main, argv, capsys) -> str:
    with pytest.raises(SystemExit):
        main(argv)
    return capsys.readouterr().out


def _flags_after(marker: str) -> set:
    """``--flags`` on documentation lines (and their continuation lines) that run ``marker``."""
    found = set()
    for md in DOCS.glob("*.md"):
        lines = md.read_text().splitlines()
        for i, line in enumerate(lines):
            if marker not in line:
                continue
            block = [line]
            j = i
            while block[-1].rstrip().endswith("\\") or (j + 1 < len(lines) and lines[j + 1].startswith("    ")
                                                          and "--" in lines[j + 1] and "python" not in lines[j + 1]):
                j += 1
                if j >= len(lines):
                    break
                block.append(lines[j])
            text = " ".join(block).split(marker, 1)[1]
            found |= set(re.findall(r"(--[a-z][a-z0-9-]*)", text))
    return found


def test_serve_flags_in_the_docs_exist(capsys):
    from eagle4_b200 import serve

    flags = _flags_after("eagle4_b200.serve")
    assert "--tokenizer" in flags and "--model" in flags
    text = _help(serve.main, ["--help"], capsys)
    missing = sorted(f for f in flags if f not in text)
    assert not missing, missing


def test_calibrate_flags_in_the_docs_exist(capsys):
    from eagle4_b200 import cli

    flags = _flags_after("cli calibrate")
    assert "--tp" in flags and "--output" in flags
    text = _help(cli.main, ["calibrate", "--help"], capsys)
    missing = sorted(f for f in flags if f not in text)
    assert not missing, missing


def test_docs_link_to_existing_pages():
    for md in DOCS.glob("*.md"):
        for target in re.findall(r"\]\(([a-z0-9_-]+\.md)\)", md.read_text()):
            assert (DOCS / target).exists(), (md.name, target)
