"""The C-ABI library loads without a GPU and exports every entry point include/mfd_b200.h declares."""
import ctypes
import os
import re

from mfd_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "mfd_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mfd_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_what_the_binding_binds():
    assert declared_symbols() == sorted(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.mfd_abi_version() == 1


def test_error_path_without_gpu_reports_status():
    lib = _lib.load()
    # invalid sizes are rejected on the host before any CUDA call
    rc = lib.mfd_topk_logz(None, 0, 1, 10, 10, 0, None, None, 3, None, None, 0, None, 0, None)
    assert rc == 1
    assert b"invalid sizes" in lib.mfd_last_error()
    rc = lib.mfd_build_trees(None, None, 2, None, 1, 32, 4, 4, 4, 0, None, None, None, None, None, None)
    assert rc == 2 and b"limits" in lib.mfd_last_error()
    ws = lib.mfd_topk_logz_workspace(128, 151936, 64)
    assert ws > 0


def test_attention_ticket_words_cover_the_merge_counters():
    """mfd_tree_attention_tickets: three counters (arrived, claimed, finished) per (request, KV head, M-tile) of
    128 packed rows (node x query head of the KV head's group), a host-only computation."""
    lib = _lib.load()
    for bs, n, H, Hkv in [(1, 65, 32, 8), (256, 65, 32, 8), (3, 17, 16, 16), (2, 129, 8, 2)]:
        G = H // Hkv
        mtiles = (n * G + 127) // 128
        assert lib.mfd_tree_attention_tickets(bs, n, H, Hkv) == 3 * bs * Hkv * mtiles
