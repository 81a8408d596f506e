"""Every public function, class and method of the reference has a counterpart
here that accepts the same calls (the reference is installed under
``baseline/_ref``, or the directory named by ``NMB_REFERENCE_PATH``; skipped
when neither holds the ``nano_megatron`` package).

A counterpart is compatible when each reference parameter appears at the same
position with the same name, kind and default; parameters this package adds
must have defaults. Annotations are not compared.
"""

import importlib
import inspect
import os
import sys

import pytest

REF = os.environ.get("NMB_REFERENCE_PATH") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")

# reference module -> the module of this package that holds its public names
MODULES = {
    "nano_megatron": "nano_megatron_b200",
    "nano_megatron.parallel": "nano_megatron_b200.parallel",
    "nano_megatron.mappings": "nano_megatron_b200.parallel",
    "nano_megatron.tp_layers": "nano_megatron_b200.models",
    "nano_megatron.cross_entropy": "nano_megatron_b200.models",
    "nano_megatron.model": "nano_megatron_b200.models",
    "nano_megatron.pipeline": "nano_megatron_b200.parallel.pipeline",
    "nano_megatron.grads": "nano_megatron_b200.parallel.grads",
    "nano_megatron.data": "nano_megatron_b200.utils.data",
    "nano_megatron.checkpoint": "nano_megatron_b200.utils.checkpoint",
    "nano_megatron.train": "nano_megatron_b200.train",
}


def _incompatible(ref_fn, our_fn) -> str | None:
    try:
        ref_sig, our_sig = inspect.signature(ref_fn), inspect.signature(our_fn)
    except (TypeError, ValueError):
        return None
    ours = list(our_sig.parameters.values())
    for i, p in enumerate(ref_sig.parameters.values()):
        q = our_sig.parameters.get(p.name)
        if q is None:
            return f"parameter {p.name!r} missing"
        if q.kind != p.kind:
            return f"parameter {p.name!r} is {q.kind.description}, not {p.kind.description}"
        if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD) and ours.index(q) != i:
            return f"parameter {p.name!r} at position {ours.index(q)}, not {i}"
        if (p.default is p.empty) != (q.default is q.empty):
            return f"parameter {p.name!r}: default differs in presence"
        if p.default is not p.empty and p.default != q.default:
            return f"parameter {p.name!r}: default {q.default!r}, not {p.default!r}"
    for q in ours:
        if q.name not in ref_sig.parameters and q.default is q.empty and q.kind not in (
                q.VAR_POSITIONAL, q.VAR_KEYWORD):
            return f"added parameter {q.name!r} has no default"
    return None


def _public(module):
    for name, obj in vars(module).items():
        if name.startswith("_") or not (inspect.isfunction(obj) or inspect.isclass(obj)):
            continue
        if module.__name__ != "nano_megatron" and obj.__module__ != module.__name__:
            continue  # imported from elsewhere; checked at its own module
        if obj.__module__.split(".")[0] == "nano_megatron":
            yield name, obj


def test_public_names_accept_the_reference_calls():
    if not os.path.isdir(os.path.join(REF, "nano_megatron")):
        pytest.skip(f"reference package not found under {REF}")
    sys.path.insert(0, REF)
    try:
        problems, checked = [], 0
        for ref_name, our_name in MODULES.items():
            ref_mod, our_mod = importlib.import_module(ref_name), importlib.import_module(our_name)
            for name, obj in _public(ref_mod):
                mine = getattr(our_mod, name, None)
                if mine is None:
                    problems.append(f"{ref_name}.{name}: no counterpart in {our_name}")
                    continue
                calls = [(name, obj, mine)]
                if inspect.isclass(obj):
                    for attr, member in vars(obj).items():
                        if (attr.startswith("_") and attr != "__init__") or isinstance(member, property):
                            continue
                        if not callable(getattr(obj, attr)):
                            continue
                        if not hasattr(mine, attr):
                            problems.append(f"{ref_name}.{name}.{attr}: missing")
                            continue
                        calls.append((f"{name}.{attr}", getattr(obj, attr), getattr(mine, attr)))
                    for attr, member in vars(obj).items():
                        if isinstance(member, property) and not hasattr(mine, attr):
                            problems.append(f"{ref_name}.{name}.{attr}: property missing")
                for label, ref_fn, our_fn in calls:
                    checked += 1
                    why = _incompatible(ref_fn, our_fn)
                    if why:
                        problems.append(f"{ref_name}.{label}: {why}")
        assert checked > 50
        assert not problems, "\n".join(problems)
    finally:
        sys.path.remove(REF)
