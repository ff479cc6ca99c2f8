"""Which serving hosts this package plugs into, and the load-time check of the installed ones.

    python -m eagle4_b200.compat [--kernels]      # also: eagle4-b200 check

prints a report per host and exits 1 when an installed host lacks a hook its adapter needs, when no host and no
native engine are usable, or (``--kernels``) when the native CUDA library does not load. This package's own engine
(``eagle4_b200.runtime``) needs no host; the hosts are for serving through SGLang, vLLM or TokenSpeed (reference
``eagle_harness/compat.py:35-194``: same host list, version ranges and refusal rules).
"""

from __future__ import annotations

import argparse
import importlib
import importlib.metadata
import logging
import sys
from dataclasses import dataclass
from typing import List, Optional, Sequence

from packaging.specifiers import SpecifierSet
from packaging.version import InvalidVersion, Version

from eagle4_b200 import __version__

log = logging.getLogger(__name__)


@dataclass(frozen=True)
class Host:
    name: str
    versions: SpecifierSet
    problems: str  # "module:function" listing the installed host's hook mismatches


HOSTS = (
    Host("sglang", SpecifierSet(">=0.5.23.dev0,<0.6"), "eagle4_b200.plugins.sglang.hooks:hook_problems"),
    Host("vllm", SpecifierSet(">=0.32.0rc1.dev283,!=0.32.0"), "eagle4_b200.plugins.vllm.hooks:missing_hooks"),
    Host("tokenspeed", SpecifierSet(">=0.1.1,<0.2"), "eagle4_b200.plugins.tokenspeed.hooks:hook_problems"),
)


@dataclass(frozen=True)
class Report:
    host: Host
    version: Optional[str]
    problems: List[str]

    @property
    def installed(self) -> bool:
        return self.version is not None

    @property
    def ok(self) -> bool:
        return self.installed and not self.problems

    @property
    def tested_version(self) -> bool:
        try:
            return Version(self.version or "") in self.host.versions
        except InvalidVersion:
            return False

    def refusal(self) -> str:
        return (f"eagle4_b200 {__version__} is disabled on {self.host.name} {self.version}: it lacks "
                f"{len(self.problems)} hook(s) ({'; '.join(self.problems)}). Install {self.host.name} with the "
                f"EAGLE harness hooks ({self.host.name}{self.host.versions}).")


def host(name: str) -> Host:
    return next(h for h in HOSTS if h.name == name)


def host_version(name: str) -> Optional[str]:
    try:
        module = importlib.import_module(name)
    except Exception:  # noqa: BLE001 - a host that fails to import is not usable
        return None
    v = getattr(module, "__version__", None)
    if v is None:
        try:
            v = importlib.metadata.version(name)
        except importlib.metadata.PackageNotFoundError:
            v = "unknown"
    return str(v)


def check(name: str) -> Report:
    spec = host(name)
    version = host_version(name)
    if version is None:
        return Report(spec, None, [])
    module, _, fn = spec.problems.partition(":")
    return Report(spec, version, getattr(importlib.import_module(module), fn)())


def check_for_registration(name: str) -> bool:
    """Logs the refusal (or the untested-version warning); True when the plugin may register."""
    r = check(name)
    if not r.ok:
        log.error(r.refusal() if r.installed else f"{name} is not installed")
        return False
    if not r.tested_version:
        log.warning("eagle4_b200: %s %s is outside %s%s; every hook matches, registering", name, r.version, name,
                    r.host.versions)
    return True


def kernels_line():
    try:
        from eagle4_b200.ops.build import load

        mod = load()
        return True, f"native CUDA kernels: {mod.__file__}"
    except Exception as e:  # noqa: BLE001
        return False, f"native CUDA kernels: not loaded ({e})"


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="Check eagle4_b200 against the installed serving hosts.")
    ap.add_argument("--kernels", action="store_true", help="also load the native CUDA library")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.WARNING, format="%(levelname)s %(message)s")
    import eagle4_b200

    print(f"eagle4_b200 {__version__} ({eagle4_b200.__file__})")
    failed = False
    for r in (check(h.name) for h in HOSTS):
        n = r.host.name
        if not r.installed:
            print(f"{n}: not installed")
        elif r.ok:
            note = "" if r.tested_version else f" (untested version, expected {n}{r.host.versions})"
            print(f"{n} {r.version}: ok, every hook matches{note}")
        else:
            failed = True
            print(f"{n} {r.version}: FAILED\n  {r.refusal()}")
    print("native engine (eagle4_b200.runtime): available")
    if args.kernels:
        ok, line = kernels_line()
        failed |= not ok
        print(line)
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
