"""The C-ABI library builds for sm_100a, loads, and exports every entry point that
include/b200moe.h declares (no compute calls: no GPU needed)."""
from __future__ import annotations

import ctypes
import os
import re

from easyinfra_b200 import _lib, build

HEADER = os.path.join(build.REPO_DIR, "include", "b200moe.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"B200MOE_API\s+[\w\s\*]+?\b(b200moe_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "b200moe_router" in syms and "b200moe_grouped_swiglu" in syms
    assert set(syms) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_builds_and_exports_all_symbols():
    path = build.build()
    lib = ctypes.CDLL(path)
    for s in declared_symbols():
        assert hasattr(lib, s), s


def test_abi_version_and_host_only_queries():
    lib = _lib.load()
    assert lib.b200moe_abi_version() == 1
    assert lib.b200moe_tokens_per_block(64) in (8, 16, 32)
    ws = lib.b200moe_router_workspace_bytes(16384, 129, 160)
    assert ws >= 256 + 16384 * 129 * 4


def test_argument_errors_are_reported_without_a_gpu():
    """Validation happens before any device call: bad sizes return B200MOE_E* codes."""
    lib = _lib.load()
    rc = lib.b200moe_router(None, 0, 0, None, None, 0, 1, 64, 0, 1, 0, 1.0, None, None, 0, 8,
                            None, None, None, None, None, None, None, None, 0, None, None)
    assert rc != 0
    assert b"E=" in lib.b200moe_last_error()


def test_no_cluster_shared_loads_in_sources():
    """Code that runs on several GPUs must never issue a TMA/bulk load that fans out
    to a whole cluster: no bulk-copy instruction in the sources carries the cluster
    fan-out qualifier.  (The pair GEMM's tcgen05.commit, a completion signal and not a
    load, is the one instruction that names it.)"""
    needle = "multi" + "cast"
    csrc = os.path.join(build.PKG_DIR, "csrc")
    for f in os.listdir(csrc):
        for i, line in enumerate(open(os.path.join(csrc, f)), 1):
            if needle in line:
                assert "tcgen05.commit" in line, f"{f}:{i}"
                assert "cp.async" not in line and "bulk" not in line, f"{f}:{i}"


def test_exchange_descriptor_and_layout_without_a_gpu():
    """The ctypes mirror of b200moe_ep_desc has the C layout, and the exchange buffer
    layout (flags, per-source counts, receive rows, combine rows) is what the header
    describes."""
    assert ctypes.sizeof(_lib.EpDesc) == 8 * 8 + 4 * 4 + 2 * 8 + 2 * 8 + 8
    from easyinfra_b200.peer_exchange import layout
    G, P, cap, comb, row = 2, 4, 128, 128, 1024
    recv, comb_off, total = layout(G, P, cap, comb, row)
    assert recv == 256 + 256                      # flags, then G*(P+1) ints rounded to 256 B
    assert comb_off == recv + G * cap * row
    assert total == comb_off + comb * row
    recv8, _, _ = layout(8, 64, 16, 16, 4096)
    assert recv8 == 256 + ((8 * 65 * 4 + 255) // 256) * 256
    lib = _lib.load()
    bad = ctypes.c_int64()
    assert lib.b200moe_ep_layout(9, 4, 1, 1, 1024, None, None, ctypes.byref(bad)) != 0   # > 8 ranks
    assert lib.b200moe_ep_layout(2, 4, 1, 1, 1000, None, None, ctypes.byref(bad)) != 0   # rows not 16-B multiples


def _declared_signatures():
    """{name: [parameter type strings]} for every B200MOE_API declaration."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"B200MOE_API\s+([\w\s\*]+?)\b(b200moe_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(3).split(",") if p.strip()]
        if params == ["void"]:
            params = []
        out[m.group(2)] = (m.group(1).strip(), params)
    return out


def _ctype_of(decl: str):
    """The ctypes type a C parameter declaration should map to."""
    d = " ".join(decl.replace("*", " * ").split())
    if "*" in d:
        return "ptr"
    base = d.rsplit(" ", 1)[0] if " " in d else d
    base = base.replace("const ", "").strip()
    return {"int": "int", "int64_t": "int64", "size_t": "size", "float": "float", "uint64_t": "uint64",
            "uint32_t": "uint32"}.get(base, base)


def test_ctypes_signatures_match_the_header():
    """Every entry point's ctypes argument list has the header's arity and kinds
    (pointer / int / int64 / size_t / float) and the same return kind, so a changed
    C signature cannot be called with a stale Python table."""
    kinds = {ctypes.c_void_p: "ptr", ctypes.c_char_p: "ptr", ctypes.c_int: "int", ctypes.c_int64: "int64",
             ctypes.c_size_t: "size", ctypes.c_float: "float", ctypes.c_uint64: "uint64",
             ctypes.c_uint32: "uint32"}
    decl = _declared_signatures()
    assert set(decl) == set(_lib.SIGNATURES)
    for name, (ret, params) in decl.items():
        restype, argtypes = _lib.SIGNATURES[name]
        want = [_ctype_of(p) for p in params]
        got = [kinds.get(a, "ptr" if a is not None and issubclass(a, ctypes._Pointer) else str(a))
               for a in argtypes]
        # size_t and uint64 are the same width on this platform's ABI; int64 likewise
        norm = {"size": "u64", "uint64": "u64", "int64": "i64"}
        assert [norm.get(k, k) for k in got] == [norm.get(k, k) for k in want], (name, got, want)
        ret_kind = _ctype_of(ret + " x")
        got_ret = "ptr" if restype in (ctypes.c_char_p, ctypes.c_void_p) else kinds.get(restype, str(restype))
        assert norm.get(got_ret, got_ret) == norm.get(ret_kind, ret_kind), (name, got_ret, ret_kind)
