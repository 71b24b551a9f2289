"""The C-ABI library loads (no GPU needed) and exports every function that
include/hanns_gpu.h declares."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "hanns_gpu.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", src)
    return sorted({n for n in names if n.startswith(("knowhere_", "hanns_gpu_"))})


def test_header_declares_reference_entry_points():
    names = declared_functions()
    for n in ["knowhere_create_index", "knowhere_search", "knowhere_search_with_bitset",
              "knowhere_free_result", "knowhere_set_nprobe", "knowhere_ivf_exrabitq_batch_search"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    from hanns_b200 import _lib
    L = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_cpu_only_calls_fail_cleanly():
    """Without a usable GPU the library reports errors instead of crashing."""
    import ctypes as C
    from hanns_b200 import _lib
    L = _lib.lib()
    assert L.knowhere_search(None, None, 0, 0, 0) is None or not L.knowhere_search(None, None, 0, 0, 0)
    cfg = _lib.CIndexConfig.default()
    cfg.index_type = 0  # Flat: not built by this library
    cfg.dim = 8
    assert not L.knowhere_create_index(cfg)
    b = L.knowhere_bitset_create(130)
    L.knowhere_bitset_set(b, 5, True)
    L.knowhere_bitset_set(b, 129, True)
    assert L.knowhere_bitset_get(b, 5) and L.knowhere_bitset_get(b, 129) and not L.knowhere_bitset_get(b, 6)
    assert L.knowhere_bitset_count(b) == 2 and L.knowhere_bitset_size(b) == 130
    L.knowhere_bitset_free(b)
