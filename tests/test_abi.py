"""The C-ABI library without a GPU: it loads, exports every symbol include/yah_qgemm.h declares, reports format
traits, and refuses bad arguments with the documented status codes before touching CUDA."""
import ctypes

import numpy as np
import pytest


def test_library_exports_every_header_symbol(pkg):
    L = pkg._lib
    declared = set(L.header_symbols())
    assert declared, "no declarations parsed from the header"
    assert declared == set(L.SYMBOLS)
    lib = L.lib()
    for name in declared:
        assert hasattr(lib, name), name


def test_version_and_traits(pkg):
    lib = pkg.lib()
    assert b"sm_100a" in lib.yah_version()
    # engine/core/gguf.cpp:27-35
    assert (lib.yah_block_elements(8), lib.yah_block_bytes(8)) == (32, 34)
    assert (lib.yah_block_elements(12), lib.yah_block_bytes(12)) == (256, 144)
    assert (lib.yah_block_elements(14), lib.yah_block_bytes(14)) == (256, 210)
    assert lib.yah_block_elements(2) == 0
    assert lib.yah_row_bytes(12, 4096) == 16 * 144
    assert lib.yah_row_bytes(8, 4096) == 128 * 34
    assert lib.yah_row_bytes(14, 100) == -1


def test_footprint(pkg):
    w, x, y = pkg.ops.footprint("q4_k", 10, 512, 2 * 144, 0, 3, 520, "f32", 12)
    assert w == 9 * 288 + 288
    assert x == (2 * 520 + 512) * 2
    assert y == (2 * 12 + 10) * 4


def _call(lib, **kw):
    a = dict(w=16, t=12, N=128, K=256, rs=144, kb=0, x=16, M=4, ldx=256, y=16, yd=0, ldy=128, epi=0, aux=None,
             ldaux=0)
    a.update(kw)
    return lib.yah_qgemm(a["w"], a["t"], a["N"], a["K"], a["rs"], a["kb"], a["x"], a["M"], a["ldx"], a["y"], a["yd"],
                         a["ldy"], a["epi"], a["aux"], a["ldaux"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(w=None), 1), (dict(x=None), 1), (dict(y=None), 1),
    (dict(t=2), 2),               # Q4_0 is not a supported format
    (dict(K=300), 1),             # K not a multiple of 256
    (dict(N=0), 1), (dict(M=0), 1),
    (dict(rs=100), 1),            # row stride shorter than the row
    (dict(w=24), 2),              # weights not 16-byte aligned
    (dict(x=24), 1),              # activations not 16-byte aligned
    (dict(ldx=260), 1),           # ldx not a multiple of 8
    (dict(ldy=64), 1),            # ldy < N
    (dict(epi=1), 1),             # resid without aux
    (dict(epi=1, aux=16, ldaux=128, yd=1), 2),  # resid writes f32
    (dict(epi=2, aux=16, ldaux=128, yd=0), 2),  # swiglu writes f16
    (dict(epi=7), 2),
])
def test_qgemm_argument_checks(pkg, kw, code):
    lib = pkg.lib()
    assert _call(lib, **kw) == code
    assert lib.yah_last_error()


def test_qgemv_rejects_more_than_32_tokens(pkg):
    lib = pkg.lib()
    rc = lib.yah_qgemv(16, 12, 128, 256, 144, 0, 16, 33, 256, 16, 0, 128, 0, None, 0, None)
    assert rc == 1 and b"32" in lib.yah_last_error()


def test_dequant_argument_checks(pkg):
    lib = pkg.lib()
    assert lib.yah_dequant(None, 12, 1, 256, 144, 0, 16, 256, None) == 1
    assert lib.yah_dequant(16, 12, 1, 256, 144, 0, 16, 250, None) == 1
    assert lib.yah_dequant(17, 12, 1, 256, 144, 0, 16, 256, None) == 1


def test_ops_footprint_refusal(pkg):
    """The numpy helper refuses a weight buffer smaller than the call's footprint (hal_run.cc:107-111)."""
    class Fake:
        nbytes = 10
    with pytest.raises(ValueError):
        pkg.ops._check_size(Fake(), 11, "weight")
