"""CPU: the C-ABI library loads, exports every symbol include/bread_b200.h
declares (plus the C++-linkage drop-ins under the reference's mangled names),
and its host-only entry points behave (argument checks, synthetic data).
No GPU compute is issued here."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bread_b200.h")


def _c_decls():
    src = open(HEADER).read()
    start = src.index('extern "C" {')
    body = src[start:]
    return sorted(set(re.findall(r"^(?:const\s+)?\w+\s*\*?\s*(bread_\w+)\s*\(", body, re.M)))


@pytest.fixture(scope="module")
def L():
    from breadv2_b200 import _lib

    return _lib


def test_library_loads(L):
    assert os.path.exists(L.LIB_PATH)
    L.lib()


def test_every_declared_symbol_exported(L):
    names = _c_decls()
    assert len(names) >= 25
    lib = L.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert set(names) <= set(L.SIGNATURES), set(names) - set(L.SIGNATURES)


def test_cxx_dropins_exported_with_reference_mangling(L):
    lib = L.lib()
    for name, mangled in L.MANGLED.items():
        assert hasattr(lib, mangled), name


def test_status_strings(L):
    assert L.status_string(0) == "ok"
    assert "qtype" in L.status_string(2)


def test_argument_errors_without_gpu(L):
    lib = L.lib()
    st = lib.bread_matvec_f32(None, None, None, 16, 256, 12, None)
    assert st == 1 and "NULL" in L.last_error()
    st = lib.bread_matvec_f32(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 16, 100, 12, None)
    assert st == 1  # cols not a multiple of 256
    st = lib.bread_matvec_f32(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 16, 256, 13, None)
    assert st == 2  # Q5_K: unsupported
    st = lib.bread_dequant(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 99, None)
    assert st == 2


def test_moe_shape_limits(L):
    lib = L.lib()
    ws = ctypes.c_void_p(256)
    # T beyond the limit, E < top_k, H not a multiple of 256
    for T, H, E, K in ((65, 2048, 256, 8), (1, 2048, 4, 8), (1, 1000, 256, 8)):
        st = lib.bread_moe_route(ctypes.c_void_p(256), ctypes.c_void_p(256), None, T, H, E, K, ctypes.c_void_p(256),
                                 ctypes.c_void_p(256), None, ws, 1 << 30, None)
        assert st == 1, (T, H, E, K)
    # workspace too small
    st = lib.bread_moe_route(ctypes.c_void_p(256), ctypes.c_void_p(256), None, 1, 2048, 256, 8, ctypes.c_void_p(256),
                             ctypes.c_void_p(256), None, ws, 16, None)
    assert st == 5


def test_workspace_bytes_monotone(L):
    f = L.lib().bread_moe_workspace_bytes
    a, b = f(1, 2048, 512, 256, 8), f(64, 2048, 512, 256, 8)
    assert 0 < a < b and a % 256 == 0


def test_synth_host_deterministic_and_distributed():
    import breadv2_b200 as bb

    a = bb.synth_blocks_host(4096, 12, 1234, 7)
    b = bb.synth_blocks_host(4096, 12, 1234, 7)
    c = bb.synth_blocks_host(4096, 12, 1235, 7)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    blk = a.reshape(4096, 144)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    # |N(0,1)| * 1e-3: mean sqrt(2/pi)*1e-3 ~ 0.80e-3
    assert 0.7e-3 < d.mean() < 0.9e-3 and d.min() >= 0
    q = blk[:, 16:]
    assert abs(q.mean() - 127.5) < 2
    b6 = bb.synth_blocks_host(4096, 14, 1234, 8).reshape(4096, 210)
    sc = b6[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31
    x = bb.synth_normal_host(1 << 16, 1.0, 1, 2)
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1.0) < 0.02


@pytest.mark.parametrize("qt", [12, 14, 8])
def test_oracle_synth_equals_library_synth(orc, qt):
    """The oracle's host restatement of the seeded generator (used by the
    bench's CPU legs so that they load no product code) gives the library's
    bytes."""
    import breadv2_b200 as bb

    assert np.array_equal(orc.synth_blocks(3001, qt, 7, 3), bb.synth_blocks_host(3001, qt, 7, 3))
    a = orc.synth_normal(10007, 0.02, 5, 6)
    assert np.array_equal(a.view(np.uint32), bb.synth_normal_host(10007, 0.02, 5, 6).view(np.uint32))
    assert np.array_equal(orc.synth_normal(4099, 0.02, 5, 6, half=True),
                          bb.synth_normal_host(4099, 0.02, 5, 6, half=True))
