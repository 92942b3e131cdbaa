"""Writes tests/golden/ref_abi.json: the ctypes signature (argtypes and
restype, by type name) that the reference's loader, tinygiant/_lib.py
load_tinygiant_lib, gives each symbol it binds.

The reference's loader is imported from its checkout ($TG_REFERENCE_DIR, else
`reference` beside this repository) and run against a recording stand-in for
ctypes.CDLL, so no library is loaded.  Tests bind this library with exactly
these signatures, on hosts without the reference checkout.

    python tests/golden/make_ref_abi.py
"""
import ctypes
import importlib.util
import json
import os
import sys
from pathlib import Path

REF = Path(os.environ.get("TG_REFERENCE_DIR", Path(__file__).resolve().parents[3] / "reference"))


class _Fn:
    def __init__(self):
        self.argtypes = None
        self.restype = ctypes.c_int   # ctypes' default


class _Recorder:
    def __init__(self, *a, **k):
        self.fns = {}

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return self.fns.setdefault(name, _Fn())


def main():
    spec = importlib.util.spec_from_file_location("ref_lib", REF / "tinygiant" / "_lib.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    real = ctypes.CDLL
    holder = {}

    def fake(path, *a, **k):
        holder["lib"] = _Recorder()
        return holder["lib"]

    mod.ctypes.CDLL = fake
    try:
        mod.load_tinygiant_lib("/nonexistent/libtinygiant.so")
    finally:
        mod.ctypes.CDLL = real

    def name(t):
        return None if t is None else t.__name__

    out = {n: {"argtypes": [name(t) for t in (f.argtypes or [])], "restype": name(f.restype)}
           for n, f in sorted(holder["lib"].fns.items())}
    Path(__file__).with_name("ref_abi.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"{len(out)} symbols", file=sys.stderr)


if __name__ == "__main__":
    main()
