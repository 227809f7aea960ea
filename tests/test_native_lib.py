"""CPU-side checks of the C ABI library: it loads without a GPU and exports every declared symbol."""
import ctypes

from jaxml_b200 import _native as N


def test_library_exports_every_header_symbol():
    lib = N.load()
    syms = N.header_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert lib.jx_version().startswith(b"jxb200")


def test_struct_layouts_match_the_header():
    # sizes compiled from include/jxb200.h with the host compiler (x86-64 LP64)
    assert ctypes.sizeof(N.JxEpilogue) == 80
    assert ctypes.sizeof(N.JxNormArgs) == 192
    assert ctypes.sizeof(N.JxQkvArgs) == 128
    assert ctypes.sizeof(N.JxAttnArgs) == 104
    assert ctypes.sizeof(N.JxSampleArgs) == 168


def test_argument_errors_are_reported_without_a_gpu():
    lib = N.load()
    rc = lib.jx_pack_k128(None, N.JX_F32, 1, 1, 1, 0, None, 8, 128, None)
    assert rc == N.JX_ERR_ARG
    assert b"null" in lib.jx_last_error()
    out = N.LL()
    assert lib.jx_linear_decode_workspace(148, 65, out) == N.JX_ERR_SHAPE
    # two partial-tile slots per CTA of 16 rows x 128 columns
    assert lib.jx_linear_decode_workspace(148, 16, out) == N.JX_OK and out.value == 148 * 2 * 16 * 128
