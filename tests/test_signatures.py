"""The drop-in boundary's Python signatures equal the reference's.

``tests/golden/signatures.json`` holds the reference's parameter names, kinds and
default values (recorded from its sources by ``tests/golden/make_signatures.py``).
Set ``TRIFUSION_REFERENCE`` to the reference project's root to also compare with the
sources themselves.
"""

from __future__ import annotations

import ast
import inspect
import json
import os
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden" / "signatures.json").read_text())


def _ours(qual):
    import trifusion_b200
    from trifusion_b200 import runtime

    if qual == "fused_mamba":
        return trifusion_b200.fused_mamba
    head, _, tail = qual.partition(".")
    obj = getattr(runtime, head)
    return getattr(obj, tail) if tail else obj


def _params(fn):
    kinds = {inspect.Parameter.POSITIONAL_ONLY: "positional", inspect.Parameter.POSITIONAL_OR_KEYWORD: "positional",
             inspect.Parameter.VAR_POSITIONAL: "var_positional", inspect.Parameter.KEYWORD_ONLY: "keyword_only",
             inspect.Parameter.VAR_KEYWORD: "var_keyword"}
    out = []
    for p in inspect.signature(inspect.unwrap(fn)).parameters.values():
        default = None if p.default is inspect.Parameter.empty else p.default
        out.append([p.name, kinds[p.kind], default])
    return out


def _same(ours, ref):
    assert [p[:2] for p in ours] == [p[:2] for p in ref]
    for (name, _, mine), (_, _, text) in zip(ours, ref):
        theirs = None if text is None else ast.literal_eval(text)
        assert mine == theirs and type(mine) is type(theirs), f"default of {name}: {mine!r} vs {text}"


@pytest.mark.parametrize("qual", sorted(GOLDEN))
def test_signature_matches_reference(qual):
    _same(_params(_ours(qual)), GOLDEN[qual]["params"])


def test_golden_matches_reference_sources():
    root = os.environ.get("TRIFUSION_REFERENCE")
    if not root or not Path(root).is_dir():
        pytest.skip("TRIFUSION_REFERENCE not set")
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_signatures", HERE / "golden" / "make_signatures.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.reference_signatures(Path(root)) == GOLDEN
