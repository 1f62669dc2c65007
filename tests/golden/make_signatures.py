"""Record the reference's public Python signatures (the drop-in boundary) as JSON.

    python tests/golden/make_signatures.py --reference <path to the reference project>

Parses the reference sources with ``ast`` (nothing is imported or run) and writes
``tests/golden/signatures.json``: for each public callable, its parameter names,
kinds and default values as source text. ``tests/test_signatures.py`` compares
this package's callables with the file (and with the reference tree itself when
it is present).
"""

from __future__ import annotations

import argparse
import ast
import json
from pathlib import Path

HERE = Path(__file__).resolve().parent
# (module file under src/trifusion_l4, qualified name)
PUBLIC = [
    ("mamba_fused.py", "fused_mamba"),
    ("runtime.py", "load_student"),
    ("runtime.py", "configure_runtime"),
    ("runtime.py", "prepare_static_weights"),
    ("runtime.py", "InferenceEngine.__init__"),
    ("runtime.py", "InferenceEngine.eager"),
    ("runtime.py", "InferenceEngine.__call__"),
    ("runtime.py", "InferenceEngine.clear"),
]


def _params(fn: ast.FunctionDef):
    a = fn.args
    out = []
    pos = a.posonlyargs + a.args
    defaults = [None] * (len(pos) - len(a.defaults)) + list(a.defaults)
    for arg, d in zip(pos, defaults):
        out.append([arg.arg, "positional", None if d is None else ast.unparse(d)])
    if a.vararg:
        out.append([a.vararg.arg, "var_positional", None])
    for arg, d in zip(a.kwonlyargs, a.kw_defaults):
        out.append([arg.arg, "keyword_only", None if d is None else ast.unparse(d)])
    if a.kwarg:
        out.append([a.kwarg.arg, "var_keyword", None])
    return out


def reference_signatures(root: Path):
    src = root / "src" / "trifusion_l4"
    sigs = {}
    for fname, qual in PUBLIC:
        tree = ast.parse((src / fname).read_text())
        body = tree.body
        node = None
        for part in qual.split("."):
            node = next(n for n in body if isinstance(n, (ast.FunctionDef, ast.ClassDef)) and n.name == part)
            body = node.body
        sigs[qual] = {"file": f"src/trifusion_l4/{fname}", "line": node.lineno, "params": _params(node)}
    return sigs


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, type=Path, help="root of the reference project")
    root = ap.parse_args().reference
    out = HERE / "signatures.json"
    out.write_text(json.dumps(reference_signatures(root), indent=1) + "\n")
    print(out)


if __name__ == "__main__":
    main()
