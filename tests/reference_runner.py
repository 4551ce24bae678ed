"""Load the reference Pantheon runner (its pantheon.py) for the tests, if present.

The runner module decides how a workload's stdout is read, what verdict a GPU
gets and whether a prebuilt workload binary is used; these tests hold the
drop-in binaries to that module itself.  It is looked for in the directory
named by the PANTHEON_REFERENCE environment variable, else in a checkout
called `reference` beside this repository.  Each call imports a fresh copy
(the runner keeps its build directory in module globals), without writing
byte-code into the reference tree.  Returns None when no runner is found; the
tests that need it then skip, and the committed fixtures made from it
(tests/golden/runner_readings.json) still hold the restated reader.
"""
from __future__ import annotations

import importlib.util
import itertools
import os
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parent.parent
_counter = itertools.count()


def reference_dir() -> Path | None:
    env = os.environ.get("PANTHEON_REFERENCE", "").strip()
    for cand in ([Path(env)] if env else []) + [_ROOT.parent / "reference"]:
        if (cand / "pantheon.py").is_file():
            return cand.resolve()
    return None


def load_runner():
    """A freshly imported copy of the reference's pantheon module, or None."""
    ref = reference_dir()
    if ref is None:
        return None
    name = f"_pantheon_reference_{next(_counter)}"
    spec = importlib.util.spec_from_file_location(name, ref / "pantheon.py")
    mod = importlib.util.module_from_spec(spec)
    old = sys.dont_write_bytecode
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref))          # the runner imports its sibling module `monitor`
    try:
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    finally:
        sys.path.remove(str(ref))
        sys.dont_write_bytecode = old
    return mod
