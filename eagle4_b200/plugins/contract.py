"""Hook contracts with serving hosts: which host attributes an adapter overrides, calls or reads, checked at load.

A :class:`Hook` names a host attribute (``"module:Class.attr"``) and the parameter names the adapter relies on:

* ``override``: the adapter's subclass overrides it, so the host's parameter names must equal ``params`` exactly;
* ``call``: the adapter calls it, so ``params`` must be among the host's (the host may add optional ones); for a class
  the constructor is checked, whether it is a dataclass or a ``msgspec.Struct``;
* ``field``: a field (dataclass / msgspec / pydantic) or class attribute must exist;
* ``exists``: the attribute must exist (module constants, enum members).

``optional`` hooks only report when present with the wrong shape. Each host adapter keeps its table in its
``hooks`` module; its plugin refuses to register while :func:`problems` reports anything, so a host refactor fails at
load time with the reason instead of in a GPU run (the same rule as reference ``eagle_harness/sglang/hooks.py:1-16``
and ``eagle_harness/tokenspeed/hooks.py:1-30``).
"""

from __future__ import annotations

import importlib
import inspect
from typing import Iterable, List, NamedTuple, Optional, Tuple

OVERRIDE, CALL, FIELD, EXISTS = "override", "call", "field", "exists"


class Hook(NamedTuple):
    path: str
    params: Tuple[str, ...] = ()
    kind: str = CALL
    owner: str = ""  # "module:Class" of this package that overrides it (OVERRIDE only)
    optional: bool = False


def resolve(path: str):
    """The object at ``"module:attr.attr"`` (or ``"a | b"`` alternatives: the first that resolves)."""
    err: Optional[Exception] = None
    for alt in (p.strip() for p in path.split("|")):
        module, _, attrs = alt.partition(":")
        try:
            obj = importlib.import_module(module)
            for part in filter(None, attrs.split(".")):
                obj = getattr(obj, part)
            return obj
        except (ImportError, AttributeError) as e:
            err = e
    raise err if err else ImportError(path)


def field_names(cls) -> Tuple[str, ...]:
    return (*getattr(cls, "__struct_fields__", ()), *getattr(cls, "__dataclass_fields__", ()),
            *getattr(cls, "model_fields", ()))


def parameter_names(func) -> Tuple[str, ...]:
    """Named parameters (``*args`` / ``**kwargs`` excluded) after the receiver of a method defined in a class; a
    class gives its constructor's. A module-level function keeps a first parameter named ``cls``."""
    ps = [p for p in inspect.signature(func).parameters.values()
          if p.kind not in (inspect.Parameter.VAR_POSITIONAL, inspect.Parameter.VAR_KEYWORD)]
    in_class = "." in getattr(func, "__qualname__", "") and not inspect.isclass(func)
    if ps and ps[0].name in ("self", "cls") and in_class:
        ps = ps[1:]
    return tuple(p.name for p in ps)


def problem(hook: Hook) -> Optional[str]:
    if hook.kind == FIELD:
        owner, _, name = hook.path.rpartition(".")
        try:
            cls = resolve(owner)
        except (ImportError, AttributeError):
            return None if hook.optional else f"{owner} is missing"
        return None if name in field_names(cls) or hasattr(cls, name) else f"{hook.path} is missing"
    try:
        obj = resolve(hook.path)
    except (ImportError, AttributeError):
        return None if hook.optional else f"{hook.path} is missing"
    if hook.kind == EXISTS:
        return None
    found = parameter_names(obj)
    if hook.kind == OVERRIDE and found != tuple(hook.params):
        return f"{hook.path}{found} is not {tuple(hook.params)}"
    if hook.kind == CALL and not set(hook.params) <= set(found):
        return f"{hook.path}{found} lacks {tuple(p for p in hook.params if p not in found)}"
    return None


def problems(hooks: Iterable[Hook]) -> List[str]:
    return [p for p in map(problem, hooks) if p is not None]


def override_mismatches(hooks: Iterable[Hook]) -> List[str]:
    """Overrides of this package whose signature differs from the table (checked without the host installed)."""
    out = []
    for h in hooks:
        if h.kind != OVERRIDE or not h.owner:
            continue
        name = h.path.rpartition(".")[2]
        try:
            found = parameter_names(getattr(resolve(h.owner), name))
        except (ImportError, AttributeError):
            out.append(f"{h.owner}.{name} is missing")
            continue
        if found != tuple(h.params):
            out.append(f"{h.owner}.{name}{found} is not {tuple(h.params)}")
    return out
