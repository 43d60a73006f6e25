"""The C ABI library loads, exports every entry point declared in include/ssparse.h, and rejects
bad arguments on the host (none of these calls reaches a CUDA API)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ssparse.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^int\s+(ss_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from streaming_sparse_b200 import build
    build.build()
    from streaming_sparse_b200._lib import lib as load
    return load()


def test_every_declared_symbol_is_exported(lib):
    from streaming_sparse_b200._lib import SIGNATURES
    names = declared()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
        assert name in SIGNATURES, f"{name} has no ctypes signature"


def _declarations():
    """{name: [parameter declarations]} of every entry point in include/ssparse.h."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"^int\s+(ss_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
        params = [p.strip() for p in m.group(2).replace("\n", " ").split(",") if p.strip() and p.strip() != "void"]
        out[m.group(1)] = params
    return out


def test_ctypes_signatures_match_the_header():
    """Every ctypes argtype has the kind of the header's parameter: pointers as pointers, and
    int / int64_t / size_t / float as those widths."""
    import ctypes
    from streaming_sparse_b200._lib import SIGNATURES
    decls = _declarations()
    assert set(decls) == set(SIGNATURES)
    scalar = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t, "float": ctypes.c_float}
    for name, params in decls.items():
        args, _ = SIGNATURES[name]
        assert len(args) == len(params), f"{name}: {len(args)} argtypes for {len(params)} parameters"
        for i, (decl, a) in enumerate(zip(params, args)):
            if "*" in decl:
                assert a is ctypes.c_void_p or hasattr(a, "_type_") and issubclass(a, ctypes._Pointer), \
                    f"{name} parameter {i} ({decl}) is a pointer, argtype {a}"
            else:
                typ = decl.rsplit(" ", 1)[0].replace("const ", "").strip()
                assert a is scalar[typ], f"{name} parameter {i} ({decl}): argtype {a}, want {scalar[typ]}"


def test_version(lib):
    assert lib.ss_version() >= 100


def test_workspace_and_capacity_queries(lib):
    n = ctypes.c_size_t()
    assert lib.ss_router_workspace_bytes(12, 4680, 32760, 64, 64, ctypes.byref(n)) == 0
    # 64-wide fp32 projections of the 74 query and 512 key blocks of every head
    assert n.value >= 4 * 12 * (74 + 512) * 64
    m = ctypes.c_int()
    assert lib.ss_attention_max_ids(32760, 64, ctypes.byref(m)) == 0
    assert m.value == 512          # config 2 fits with every block listed
    assert lib.ss_attention_max_ids(98280, 64, ctypes.byref(m)) == 0
    assert m.value >= 768          # config 5 at 50% density
    assert lib.ss_attention_max_ids(100, 96, ctypes.byref(m)) == 1001


def test_host_argument_errors(lib):
    fake = ctypes.c_void_p(0x100000)  # never dereferenced: every call below fails its host checks first
    # null pointers
    assert lib.ss_attention(None, fake, fake, fake, 12, 64, 64, 64, 1, 0.1, fake, 0, None, None, None) == 1002
    # unsupported block size / empty sizes
    assert lib.ss_attention(fake, fake, fake, fake, 12, 64, 64, 96, 1, 0.1, fake, 0, None, None, None) == 1001
    assert lib.ss_attention(fake, fake, fake, fake, 0, 64, 64, 64, 1, 0.1, fake, 0, None, None, None) == 1001
    # misaligned base pointer (TMA needs 16-byte alignment)
    odd = ctypes.c_void_p(0x100002)
    assert lib.ss_attention(odd, fake, fake, fake, 12, 64, 64, 64, 1, 0.1, fake, 0, None, None, None) == 1002
    # out 16-byte but not 32-byte aligned (the output rows leave in 32-byte stores)
    out16 = ctypes.c_void_p(0x100010)
    assert lib.ss_attention(fake, fake, fake, fake, 12, 64, 64, 64, 1, 0.1, out16, 0, None, None, None) == 1002
    # router: budget larger than the unforced blocks, n_ids inconsistent, workspace too small
    ws = ctypes.c_size_t(1 << 30)
    assert lib.ss_router(fake, fake, fake, fake, 12, 1560, 6240, 64, 64, 0, 74, fake, 99, None, None, fake, ws,
                         None, None) == 1004
    assert lib.ss_router(fake, fake, fake, fake, 12, 1560, 6240, 64, 64, 0, 24, fake, 48, None, None, fake, ws,
                         None, None) == 1001
    assert lib.ss_router(fake, fake, fake, fake, 12, 1560, 6240, 64, 64, 0, 24, fake, 49, None, None, fake,
                         ctypes.c_size_t(16), None, None) == 1003
    # commit-time key pooling and the cached route: ranges and table sizes
    assert lib.ss_router_pool_keys(fake, fake, 12, 32760, 64, 64, 0, 513, fake, 512, None, None) == 1001
    assert lib.ss_router_pool_keys(fake, fake, 12, 32760, 64, 64, 10, 5, fake, 512, None, None) == 1001
    assert lib.ss_router_pool_keys(fake, fake, 12, 32760, 64, 64, 0, 438, fake, 511, None, None) == 1001
    assert lib.ss_router_pool_keys(fake, None, 12, 32760, 64, 64, 0, 438, fake, 512, None, None) == 1002
    assert lib.ss_router_cached(fake, fake, 0, fake, fake, 12, 4680, 32760, 64, 64, 0, 54, fake, 511, 438, fake, 128,
                                None, None, fake, ws, None, None) == 1001
    assert lib.ss_router_cached(fake, fake, 0, fake, fake, 12, 4680, 32760, 64, 64, 0, 54, fake, 512, 513, fake, 128,
                                None, None, fake, ws, None, None) == 1001
    assert lib.ss_router_cached(fake, fake, 0, fake, fake, 12, 4680, 32760, 64, 64, 0, 54, None, 512, 438, fake, 128,
                                None, None, fake, ws, None, None) == 1002
    # merge / cache shape checks
    assert lib.ss_lse_merge(fake, fake, 0, 12, 10, fake, 0, None, None) == 1001
    end = ctypes.c_int64()
    assert lib.ss_cache_append(fake, fake, 24, 1, fake, fake, 128, 30, 1, 0, 0, 0, 4, ctypes.byref(end), None) == 1001
    assert lib.ss_cache_append(fake, fake, 24, 1, fake, fake, 100, 12, 1, 0, 0, 0, 4, ctypes.byref(end), None) == 1001
    # INT8-QK path: page ranges past the window, null and misaligned pointers, more pages than the
    # kernel's page list holds (4096), unsupported block size and output type
    assert lib.ss_quant_k_pages(fake, 12, 32760, 0, 513, fake, fake, None) == 1001
    assert lib.ss_quant_k_pages(fake, 12, 32760, 10, 5, fake, fake, None) == 1001
    assert lib.ss_quant_k_pages(None, 12, 32760, 0, 512, fake, fake, None) == 1002
    assert lib.ss_quant_k_pages(odd, 12, 32760, 0, 512, fake, fake, None) == 1002
    assert lib.ss_quant_k_pages(fake, 12, 32760, 7, 7, fake, fake, None) == 0        # empty range: nothing launched
    sz = ctypes.c_size_t(0)
    assert lib.ss_attention_i8(fake, fake, fake, fake, fake, 12, 4680, 4096 * 64 + 1, 64, 4, 0.1, fake, 0, None, None,
                               None, sz, None) == 1001
    assert lib.ss_attention_i8(fake, fake, fake, fake, fake, 12, 4680, 32760, 96, 4, 0.1, fake, 0, None, None,
                               None, sz, None) == 1001
    assert lib.ss_attention_i8(fake, fake, fake, fake, fake, 12, 4680, 32760, 64, 4, 0.1, fake, 2, None, None,
                               None, sz, None) == 1001
    assert lib.ss_attention_i8(fake, fake, fake, fake, fake, 12, 4680, 32760, 64, 4, 0.1, odd, 0, None, None,
                               None, sz, None) == 1002
    assert lib.ss_attention_i8(fake, None, fake, fake, fake, 12, 4680, 32760, 64, 4, 0.1, fake, 0, None, None,
                               None, sz, None) == 1002
