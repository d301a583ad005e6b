"""The C ABI library loads on a CPU-only host and exports every entry point
that include/specverify.h declares (no compute calls: there is no GPU here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "specverify.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)   # drop comments
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(tv_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    import sys
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    import build
    path = build.build()        # incremental: compiles only what changed
    return ctypes.CDLL(str(path))


def test_header_declares_the_path_entry_points():
    names = _declared()
    for expected in ("tv_verify_attn", "tv_attn_workspace_size", "tv_merge_partials", "tv_pack_mask", "tv_accept",
                     "tv_accept_workspace_size", "tv_compact_contig", "tv_copy_pages", "tv_compact_paged",
                     "tv_arena_gather", "tv_gather_page_table", "tv_status_string", "tv_version"):
        assert expected in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"declared in specverify.h but not exported: {missing}"


def test_python_binding_covers_the_header(lib):
    from specverify import _lib
    assert set(_lib.EXPORTED) >= set(_declared())


def test_no_undeclared_debug_entry_points(lib):
    """The shipped library exports no profiling hooks beyond the header."""
    assert not hasattr(lib, "tv_debug_set_trace")


def test_host_only_calls(lib):
    lib.tv_version.restype = ctypes.c_char_p
    lib.tv_status_string.restype = ctypes.c_char_p
    assert lib.tv_version().decode()
    for code in range(0, -9, -1):
        assert lib.tv_status_string(code).decode()
    # shape / null validation happens on the host, before any device work
    lib.tv_attn_workspace_size.restype = ctypes.c_int32
    assert lib.tv_attn_workspace_size(None, None) != 0


def test_sharded_exchange_buffer_size(lib):
    """tv_sharded_exchange_bytes (host arithmetic): two slots, each of W
    partials' O and LSE plus the final rows as 8-byte words (256-byte aligned
    sections), then one int32 step count per exchange-kernel block (up to
    4 x 148), and the argument checks."""
    f = lib.tv_sharded_exchange_bytes
    f.restype = ctypes.c_int32
    f.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.POINTER(ctypes.c_int64)]
    a = lambda x: (x + 255) // 256 * 256
    for world, rows, d in ((1, 2048, 128), (2, 2048, 128), (8, 8192, 64), (3, 7, 32)):
        n = ctypes.c_int64(-1)
        assert f(world, rows, d, ctypes.byref(n)) == 0
        slot = a(world * rows * d * 8) + a(world * rows * 8) + a(rows * d * 8) + a(rows * 8)
        assert n.value == 2 * slot + a(4 * 4 * 148), (world, rows, d)
    n = ctypes.c_int64(0)
    assert f(0, 16, 128, ctypes.byref(n)) != 0           # no ranks
    assert f(9, 16, 128, ctypes.byref(n)) != 0           # more than 8 ranks
    assert f(2, 16, 96, ctypes.byref(n)) != 0            # head_dim not 32 / 64 / 128
    assert f(2, 16, 128, None) != 0


def test_ctypes_structs_match_the_header(tmp_path):
    """The ctypes mirrors have the C structs' size and every field offset
    (compiled against include/specverify.h with the host C compiler)."""
    import shutil
    import subprocess
    import sys
    if shutil.which("gcc") is None:
        pytest.skip("no host C compiler")
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    from specverify import _lib
    mirrors = {"tv_attn_args": _lib.AttnArgs, "tv_accept_args": _lib.AcceptArgs, "tv_rope_args": _lib.RopeArgs,
               "tv_lmhead_args": _lib.LmheadArgs}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "specverify.h"', "int main(void) {"]
    for cname, py in mirrors.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for line in filter(None, out):
        cname, field, value = line.split()
        got[(cname, field)] = int(value)
    for cname, py in mirrors.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, f"{cname}.{fname}"


def test_sharded_entry_rejects_a_mismatched_exchange_buffer(lib):
    """tv_verify_attn_sharded checks the exchange buffer's size against the
    layout of this request's (world, rows, head_dim) on the host and returns
    TV_ERR_WORKSPACE before any launch (the pointers here are never used)."""
    import sys
    sys.path.insert(0, str(ROOT / "specdiff-ae_b200"))
    from specverify import _lib
    a = _lib.AttnArgs()
    a.dtype = 0                       # TV_BF16
    a.batch, a.rows, a.heads, a.kv_heads, a.head_dim = 1, 64, 32, 8, 128
    a.scale = 128 ** -0.5
    fake = 1 << 20                    # 16-byte aligned stand-ins, never dereferenced
    a.q, a.k, a.v, a.out = fake, fake, fake, fake
    a.q_sb, a.q_sm, a.q_sh = 64 * 32 * 128, 32 * 128, 128
    a.k_sb, a.k_sn, a.k_sh = 8 * 16 * 128, 128, 16 * 128
    a.v_sb, a.v_sn, a.v_sh = a.k_sb, a.k_sn, a.k_sh
    a.page_table, a.pt_sb, a.page_size, a.num_pages = fake, 4096, 16, 4096
    a.num_keys = 32768
    a.o_sb, a.o_sm, a.o_sh = a.q_sb, a.q_sm, a.q_sh
    f = lib.tv_verify_attn_sharded
    f.restype = ctypes.c_int32
    f.argtypes = [ctypes.POINTER(_lib.AttnArgs), ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                  ctypes.c_int64, ctypes.c_void_p]
    n = ctypes.c_int64(0)
    lib.tv_sharded_exchange_bytes.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_int64)]
    assert lib.tv_sharded_exchange_bytes(2, 64 * 32, 128, ctypes.byref(n)) == 0
    bases = (ctypes.c_void_p * 2)(fake, fake + (1 << 16))
    for wrong in (n.value - 256, n.value + 256, 0):
        assert f(ctypes.byref(a), 2, 0, bases, wrong, None) == -5, wrong      # TV_ERR_WORKSPACE
    # a buffer sized for another world size or row count is rejected too
    other = ctypes.c_int64(0)
    assert lib.tv_sharded_exchange_bytes(4, 64 * 32, 128, ctypes.byref(other)) == 0
    assert f(ctypes.byref(a), 2, 0, bases, other.value, None) == -5
    assert lib.tv_sharded_exchange_bytes(2, 65 * 32, 128, ctypes.byref(other)) == 0
    assert f(ctypes.byref(a), 2, 0, bases, other.value, None) == -5
