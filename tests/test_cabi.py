"""The C ABI library loads and exports every entry point include/*.h declares,
and the ctypes mirrors have the C structs' exact layout (no GPU calls)."""

import ctypes
import glob
import os
import re
import subprocess
import tempfile

import pytest

from intent_attention import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = glob.glob(os.path.join(ROOT, "include", "*.h"))


def _declared():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"^\s*(?:int|const char\*)\s+(iak_\w+)\s*\(", src, flags=re.M))
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert {"iak_version", "iak_last_error", "iak_decode", "iak_decode_workspace_size", "iak_merge_partials",
            "iak_pack_metadata", "iak_quantize_pages"} <= names


def test_library_exports_all_declared_symbols():
    assert N.available(), "libiak_b200.so missing: run intent-attention-kernel_b200/build.py"
    lib = ctypes.CDLL(N.LIB_PATH)
    for name in sorted(_declared()):
        assert hasattr(lib, name), name
        assert name in N.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_query():
    L = N.lib()
    assert L.iak_version() == 2
    # a pure host-side validation error: no device call is made
    st = L.iak_merge_partials(None, None, None, 4, 0, 64, None, 0, 64, None)
    assert st == N.IAK_ERR_INVALID_ARG
    assert b"merge" in L.iak_last_error()


_STRUCTS = {"iak_page_pools": N.PagePools, "iak_decode_args": N.DecodeArgs, "iak_pack_args": N.PackArgs,
            "iak_quant_args": N.QuantArgs, "iak_mla_args": N.MlaArgs, "iak_peer_exchange": N.PeerExchange,
            "iak_route_args": N.RouteArgs, "iak_append_args": N.AppendArgs, "iak_convert_args": N.ConvertArgs,
            "iak_prefill_args": N.PrefillArgs}


def test_struct_layout_matches_header():
    """sizeof and every field offset of each ctypes mirror equal the C compiler's."""
    lines = []
    for cname, ct in _STRUCTS.items():
        lines.append(f'  printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in ct._fields_:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    prog = ("#include <stdio.h>\n#include <stddef.h>\n#include \"intent_attention_b200.h\"\n"
            "int main(void) {\n" + "\n".join(lines) + "\n  return 0;\n}\n")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        r = subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], capture_output=True, text=True)
        if r.returncode:
            pytest.skip("gcc unavailable: " + r.stderr[:200])
        out = subprocess.run([exe], capture_output=True, text=True).stdout
    got = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    assert len(got) == sum(1 + len(ct._fields_) for ct in _STRUCTS.values())
    for k, v in got.items():
        if "." in k:
            t, f = k.split(".")
            assert getattr(_STRUCTS[t], f).offset == int(v), k
        else:
            assert ctypes.sizeof(_STRUCTS[k]) == int(v), k


def test_route_args_rejected_on_the_host():
    """iak_route_pages validates its scalars before any device call
    (memory_pressure outside [0, 1] is a ValueError in IntentQuantizer)."""
    L = N.lib()
    a = N.RouteArgs()
    a.batch, a.num_table_heads, a.page_size, a.num_blocks = 1, 1, 16, 4
    a.memory_pressure = 1.5
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG
    assert b"memory_pressure" in L.iak_last_error()
    a.memory_pressure = float("nan")
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG
    a.memory_pressure = 0.5
    a.page_size = 0
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG
    a.page_size = 16
    a.num_blocks = N.ROUTE_MAX_BLOCKS + 1
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_UNSUPPORTED
    a.num_blocks = 4
    a.layout_stride = 2
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG
    a.layout_stride = 0
    a.page_tags = 1
    a.prec_to_tag[3] = 16
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG
    a.page_tags = None
    # batch 0 is a no-op; missing outputs are an argument error
    a.batch = 0
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_OK
    a.batch = 2
    assert L.iak_route_pages(ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG


def test_prefill_and_kv_write_args_rejected_on_the_host():
    """iak_prefill / iak_append_tokens / iak_convert_pages validate their
    scalars and pointers before any device call."""
    L = N.lib()
    pools = N.PagePools()
    pools.num_pages, pools.page_size, pools.head_dim, pools.scale_mode = 4, 16, 128, 0
    a = N.PrefillArgs()
    a.batch, a.num_q_heads, a.num_table_heads, a.num_queries, a.table_width = 1, 4, 3, 8, 4
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG   # 4 % 3 != 0
    assert b"multiple" in L.iak_last_error()
    a.num_table_heads = 2
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG   # null q / out
    a.num_queries = 0
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_OK               # nothing to do
    a.num_queries = 8
    a.q, a.out, a.page_table, a.page_tags, a.tag_bytes = 16, 16, 16, 16, 2
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_INVALID_ARG   # tag_bytes
    a.tag_bytes = 1
    pools.page_size, a.row_masks = 128, 16
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_UNSUPPORTED   # masks, PS > 64
    pools.page_size, pools.head_dim = 16, 40
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_UNSUPPORTED   # head_dim
    pools.head_dim = 128
    # the tensor-core kernel takes a positive scale only; asked for by name, it refuses others
    a.kernel, a.sm_scale = N.KERNEL_TENSOR, -0.1
    assert L.iak_prefill(ctypes.byref(pools), ctypes.byref(a), None) == N.IAK_ERR_UNSUPPORTED
    assert b"positive sm_scale" in L.iak_last_error()
    a.kernel = N.KERNEL_AUTO
    ap = N.AppendArgs()
    ap.batch, ap.num_table_heads, ap.num_new = 2, 1, 1
    assert L.iak_append_tokens(ctypes.byref(pools), ctypes.byref(ap), None) == N.IAK_ERR_INVALID_ARG
    ap.num_new = 0
    assert L.iak_append_tokens(ctypes.byref(pools), ctypes.byref(ap), None) == N.IAK_OK
    cv = N.ConvertArgs()
    cv.num_ids = 3
    assert L.iak_convert_pages(ctypes.byref(pools), ctypes.byref(cv), None) == N.IAK_ERR_INVALID_ARG
    pools.page_size = 256
    cv.page_ids, cv.new_formats, cv.page_tags, cv.tag_bytes = 16, 16, 16, 1
    assert L.iak_convert_pages(ctypes.byref(pools), ctypes.byref(cv), None) == N.IAK_ERR_UNSUPPORTED   # PS*D too big
