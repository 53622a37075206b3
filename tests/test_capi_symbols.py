"""The C ABI library loads without a GPU and exports every function that
include/*.h declares; the oracle library loads too."""
import ctypes
import glob
import os
import re

from conftest import REPO


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        # a declaration: <type> <name>(...);  (typedef'd struct/enum bodies excluded)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", src, re.M):
            if not m.group(0).lstrip().startswith("typedef"):
                names.add(m.group(1))
    return sorted(names)


def test_header_declares_the_boundary():
    names = _declared_functions()
    for required in ("gaje_cuda_load", "gaje_cuda_forward", "gaje_cuda_generate", "gaje_cuda_free",
                     "gaje_cuda_clear_cache", "gaje_cuda_set_k_wta_ratio", "gaje_cuda_last_error",
                     "gaje_flat_inspect", "gaje_quantize_q4_0", "gaje_cuda_q4_0_gemv"):
        assert required in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(g):
    lib = ctypes.CDLL(os.path.join(REPO, "gaje-semantic-compression_b200", "libgaje_cuda.so"))
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared in include/ but not exported: {missing}"


def test_last_error_is_empty_string_initially(g):
    assert isinstance(g.last_error(), str)


def test_oracle_library_loads(O):
    L = O.lib()
    assert L.or_max_threads() >= 1
