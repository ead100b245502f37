"""Import the reference's ``modeling_qwen3pkm.py`` from the reference tree.

Used by the golden-fixture script and the model drop-in test, in the
container that holds the reference tree (nothing on a GPU box imports it).
The file is imported as ``<pkg>.modeling_qwen3pkm`` under a synthetic
package whose path is the reference tree, so its relative imports
(``modeling_qwen3pkm.py:20-24``) resolve either to the reference's own
``pkm`` / ``fwpkm`` packages or, with ``ours=True``, to this repository's.
``configuration_qwen3pkm.py`` does not parse as shipped (an unterminated
string at ``:99``); it is compiled from its text with that string closed,
in memory, without touching the file.
"""
from __future__ import annotations

import importlib
import os
import sys
import types

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("MODELOS_REF", os.path.join(os.path.dirname(REPO), "reference"))


def available() -> bool:
    return os.path.isfile(os.path.join(REF, "modeling_qwen3pkm.py"))


def _config_module(pkg: str):
    path = os.path.join(REF, "configuration_qwen3pkm.py")
    with open(path) as f:
        src = f.read()
    broken = "\"fwpkm_value_src='hidden' \n"
    if broken in src:
        src = src.replace(broken, "\"fwpkm_value_src='hidden'\"\n")
    mod = types.ModuleType(pkg + ".configuration_qwen3pkm")
    mod.__package__ = pkg
    mod.__file__ = path
    sys.modules[mod.__name__] = mod
    exec(compile(src, path, "exec"), mod.__dict__)
    return mod


def load(pkg: str, ours: bool):
    """The model module imported as ``pkg.modeling_qwen3pkm``."""
    if pkg + ".modeling_qwen3pkm" in sys.modules:
        return sys.modules[pkg + ".modeling_qwen3pkm"]
    root = types.ModuleType(pkg)
    root.__path__ = [REF]
    sys.modules[pkg] = root
    _config_module(pkg)
    if ours:
        if REPO not in sys.path:
            sys.path.insert(0, REPO)
        for name in ("pkm", "pkm.memory", "fwpkm", "fwpkm.fwpkm", "fwpkm.fwmlp"):
            sys.modules[f"{pkg}.{name}"] = importlib.import_module("modelos_b200." + name)
    return importlib.import_module(pkg + ".modeling_qwen3pkm")
