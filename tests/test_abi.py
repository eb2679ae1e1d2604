"""The C ABI library loads on a machine without a GPU and exports every entry point include/od_b200.h declares,
with the argument list the ctypes binding uses (no compute calls here)."""
import ctypes
import re

from opendecider_b200 import _lib


def declared_symbols():
    text = open(_lib.HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:OD_API\s+)?(?:const\s+)?\w+\s*\*?\s*(od_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_bound_symbols():
    decl = declared_symbols()
    assert set(decl) == set(_lib.SIGNATURES), (sorted(decl), sorted(_lib.SIGNATURES))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.od_version().decode().startswith("od_b200")
    # only the C ABI is exported (the build hides every other symbol)
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert {s for s in exported if s.startswith("od_")} == set(declared_symbols())


def test_argument_counts_match_header():
    text = re.sub(r"/\*.*?\*/", "", open(_lib.HEADER).read(), flags=re.S)
    for name, args in _lib.SIGNATURES.items():
        m = re.search(name + r"\s*\(([^)]*)\)", text)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), name


def test_cpu_tensors_are_rejected():
    import pytest
    import torch
    with pytest.raises(_lib.ODError):
        _lib.quant_rows(torch.zeros(4, 8, dtype=torch.bfloat16))
