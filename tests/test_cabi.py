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
    assert L.iak_version() == 1
    # a pure host-side validation error: no device call is made
    st = L.iak_merge_partials(None, None, None, 4, 0, 64, None, 0, 64, None)
    assert st == N.IAK_ERR_INVALID_ARG
    assert b"merge" in L.iak_last_error()


def test_struct_layout_matches_header():
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "intent_attention_b200.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("iak_page_pools %zu\n", sizeof(iak_page_pools));
  printf("iak_decode_args %zu\n", sizeof(iak_decode_args));
  printf("iak_pack_args %zu\n", sizeof(iak_pack_args));
  printf("iak_quant_args %zu\n", sizeof(iak_quant_args));
  printf("iak_mla_args %zu\n", sizeof(iak_mla_args));
  printf("iak_peer_exchange %zu\n", sizeof(iak_peer_exchange));
  P(iak_peer_exchange, rank) P(iak_peer_exchange, rows) P(iak_peer_exchange, head_dim)
  P(iak_page_pools, num_pages) P(iak_page_pools, scale_mode)
  P(iak_decode_args, tag_map) P(iak_decode_args, sm_scale) P(iak_decode_args, partial_acc) P(iak_decode_args, num_splits) P(iak_decode_args, kernel)
  P(iak_pack_args, pad_value) P(iak_quant_args, scale_mode) P(iak_quant_args, num_pages)
  P(iak_mla_args, dense_pages) P(iak_mla_args, num_pages) P(iak_mla_args, page_table) P(iak_mla_args, tag_map)
  P(iak_mla_args, sm_scale) P(iak_mla_args, partial_acc) P(iak_mla_args, kernel)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        r = subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], capture_output=True, text=True)
        if r.returncode:
            pytest.skip("gcc unavailable: " + r.stderr[:200])
        out = subprocess.run([exe], capture_output=True, text=True).stdout
    got = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    types = {"iak_page_pools": N.PagePools, "iak_decode_args": N.DecodeArgs, "iak_pack_args": N.PackArgs,
             "iak_quant_args": N.QuantArgs, "iak_mla_args": N.MlaArgs,
             "iak_peer_exchange": N.PeerExchange}
    for k, v in got.items():
        if "." in k:
            t, f = k.split(".")
            assert getattr(types[t], f).offset == int(v), k
        else:
            assert ctypes.sizeof(types[k]) == int(v), k
