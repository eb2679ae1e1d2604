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


def test_attention_split_plan_is_host_only():
    """od_prefix_attn_plan is host arithmetic (no GPU): a launch with fewer query tiles than SMs splits the state
    prefix and gets a workspace of nsplit x R x t x Hq x (D + 1) floats; a full launch or no prefix does not."""
    lib = _lib.load()

    def plan(R, t, S, T, Hq=32, Hkv=8, D=128, G=0, mg=1, sms=148):
        dims = _lib.AttnDims(R, t, S, T, 0, 0, Hq, Hkv, D, _lib.OD_BF16, D ** -0.5, G or R, mg, 0, 0)
        n, b = ctypes.c_int(0), ctypes.c_int64(-1)
        assert lib.od_prefix_attn_plan(ctypes.byref(dims), sms, ctypes.byref(n), ctypes.byref(b)) == 0
        return n.value, b.value

    n, b = plan(R=1, t=2, S=1, T=4096)                       # 8 query tiles on 148 SMs
    assert n > 1 and b == 4 * n * 1 * 2 * 32 * 129
    assert plan(R=64 * 64, t=16, S=64, T=4096, G=64 * 16, mg=4) == (1, 0)   # thousands of tiles
    assert plan(R=8, t=2, S=0, T=0) == (1, 0)                 # no state prefix
