"""Fake serving hosts for the plugin tests: a module tree generated from a hook table, so every hooked attribute
exists with the parameters the adapter relies on, plus the few registry behaviours registration needs."""

from __future__ import annotations

import os
import textwrap
from collections import defaultdict


def write_fake_host(root: str, hooks, extra: dict = None) -> None:
    """Write modules under ``root`` defining every ``module:Class.attr`` / ``module:func`` of ``hooks``."""
    mods = defaultdict(lambda: defaultdict(dict))  # module -> class ('' for module level) -> attr -> params
    for h in hooks:
        for alt in h.path.split("|"):
            module, _, attrs = alt.strip().partition(":")
            parts = attrs.split(".")
            owner, attr = ("", parts[0]) if len(parts) == 1 else (parts[0], parts[1] if len(parts) == 2 else None)
            slot = mods[module][owner]
            if attr is None:
                continue
            kind, old = slot.get(attr, (h.kind, ()))
            slot[attr] = (kind, tuple(old) + tuple(p for p in h.params if p not in old))
    names = set(mods) | set(extra or {})
    _PACKAGES.clear()
    _PACKAGES.update(m for m in names if any(o.startswith(m + ".") for o in names))
    for module, classes in mods.items():
        src = ["from dataclasses import dataclass, field", ""]
        for name, (kind, params) in classes.get("", {}).items():
            if kind == "exists":
                src.append(f"{name} = 4")
            else:
                args = ", ".join(params)
                src.append(f"def {name}({args + ', ' if args else ''}**kwargs):\n    return None")
        for cls, attrs in classes.items():
            if cls == "":
                continue
            fields = [a for a, (k, _) in attrs.items() if k == "field"]
            if attrs.get("__init__") is None and any(k == "call" for _, (k, p) in attrs.items() if _ == "__init__"):
                pass
            body = []
            for a, (kind, params) in attrs.items():
                if kind == "field":
                    body.append(f"    {a} = None")
                elif a == "__init__":
                    args = ", ".join(params)
                    body.append(f"    def __init__(self{', ' + args if args else ''}, **kwargs):\n        pass")
                elif kind == "exists":
                    body.append(f"    def {a}(self):\n        return None")
                else:
                    args = ", ".join(params)
                    body.append(f"    def {a}(self{', ' + args if args else ''}):\n        return None")
            if not body:
                body = ["    pass"]
            src.append(f"class {cls}:\n" + "\n".join(body))
        src += (extra or {}).get(module, [])
        _write(root, module, "\n\n".join(src) + "\n")
    for module, lines in (extra or {}).items():
        if module not in mods:
            _write(root, module, "from dataclasses import dataclass\n\n" + "\n\n".join(lines) + "\n")
    # package markers
    for dirpath, dirs, files in os.walk(root):
        if dirpath != root and "__init__.py" not in files:
            open(os.path.join(dirpath, "__init__.py"), "a").close()


_PACKAGES: set = set()


def _write(root: str, module: str, text: str) -> None:
    parts = module.split(".")
    pkg_dir = os.path.join(root, *parts)
    is_pkg = module in _PACKAGES or len(parts) == 1
    path = os.path.join(pkg_dir, "__init__.py") if is_pkg else pkg_dir + ".py"
    os.makedirs(os.path.dirname(path), exist_ok=True)
    mode = "a" if os.path.exists(path) else "w"
    with open(path, mode) as f:
        f.write(text)


def call_fields_as_dataclasses(hooks):
    """``module:Class`` CALL hooks whose class must accept keyword fields (dataclass constructors)."""
    out = []
    for h in hooks:
        module, _, attrs = h.path.partition(":")
        if "." not in attrs and attrs[:1].isupper():
            out.append((module, attrs, h.params))
    return out


def dataclass_src(name: str, params) -> str:
    fields = "\n".join(f"    {p}: object = None" for p in params) or "    pass"
    return f"@dataclass\nclass {name}:\n{fields}"


SGLANG_REGISTRY = {
    "sglang.srt.speculative.spec_info": [textwrap.dedent('''
        class SpeculativeAlgorithm:
            _registry = {}
            @classmethod
            def register(cls, name, supports_overlap=False, spec_class=None):
                def deco(fn):
                    cls._registry[name] = (fn, spec_class, supports_overlap)
                    return fn
                return deco
            @classmethod
            def from_string(cls, name):
                if name not in cls._registry:
                    raise ValueError(name)
                return cls._registry[name]
        ''')],
    "sglang.srt.models.registry": [textwrap.dedent('''
        class _Registry:
            def __init__(self):
                self.packages = []
            def get_supported_archs(self):
                return []
            def register(self, package, strict=False):
                self.packages.append(package)
        ModelRegistry = _Registry()
        ''')],
    "sglang": ['__version__ = "0.5.23.dev252"'],
}
