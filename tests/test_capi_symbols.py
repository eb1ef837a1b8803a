"""The C-ABI library loads without a GPU and exports exactly the functions include/one_b200.h
declares (no compute call is made here)."""
import os
import re
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "one_b200.h")
LIB = os.path.join(REPO, "medit-one_b200", "one", "libone_b200.so")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(one_[a-z0-9_]+)\s*\(", src))


def test_header_declares_entry_points():
    names = declared()
    for must in ("one_engine_create", "one_engine_step", "one_engine_prefill", "one_linear_moe", "one_flash_attention",
                 "one_rotary_embedding", "one_cumsum_and_normalize", "one_combined_rope_attention", "one_moe_routing"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import ctypes
    lib = ctypes.CDLL(LIB)
    for name in declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T one_" in ln}
    assert exported == declared(), (exported ^ declared())


def test_binding_matches_header():
    from one import _capi
    assert set(_capi.SIGNATURES) == declared()
    assert _capi.LIB.one_abi_version() == _capi.ABI_VERSION == 2
