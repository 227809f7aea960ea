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
    assert ctypes.sizeof(N.JxEpilogue) == 264
    assert ctypes.sizeof(N.JxNormArgs) == 232
    assert ctypes.sizeof(N.JxQkvArgs) == 128
    assert ctypes.sizeof(N.JxAttnArgs) == 120
    assert ctypes.sizeof(N.JxFilterArgs) == 56
    assert ctypes.sizeof(N.JxSampleArgs) == 168


def test_struct_field_offsets_match_the_c_compiler(tmp_path):
    """Every ctypes field sits at the offset the C compiler gives the header's field of the same name."""
    import os
    import shutil
    import subprocess

    import pytest

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    pairs = [(N.JxEpilogue, "jx_epilogue"), (N.JxNormArgs, "jx_norm_args"), (N.JxQkvArgs, "jx_qkv_args"),
             (N.JxAttnArgs, "jx_attn_args"), (N.JxDAttnArgs, "jx_dattn_args"), (N.JxPAttnArgs, "jx_pattn_args"),
             (N.JxSampleArgs, "jx_sample_args"), (N.JxRopeArgs, "jx_rope_args"), (N.JxFilterArgs, "jx_filter_args")]
    inc = os.path.join(os.path.dirname(N.__file__), os.pardir, "include")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "jxb200.h"', "int main(void) {"]
    for cls, cname in pairs:
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for f, _ in cls._fields_:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        c, f, v = ln.split()
        got[(c, f)] = int(v)
    for cls, cname in pairs:
        assert got[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert got[(cname, f)] == getattr(cls, f).offset, (cname, f)


def test_argument_errors_are_reported_without_a_gpu():
    lib = N.load()
    rc = lib.jx_pack_k128(None, N.JX_F32, 1, 1, 1, 0, None, 8, 128, None)
    assert rc == N.JX_ERR_ARG
    assert b"null" in lib.jx_last_error()
    out = N.LL()
    assert lib.jx_linear_decode_workspace(148, 65, out) == N.JX_ERR_SHAPE
    # two partial-tile slots per CTA of 16 rows x 128 columns
    assert lib.jx_linear_decode_workspace(148, 16, out) == N.JX_OK and out.value == 148 * 2 * 16 * 128


def test_decode_attention_rejects_an_output_too_small_for_the_batch():
    """The K128 attention output must hold every batch row (out_rp >= B, a multiple of 8); the check runs
    on the host before any device work, so it needs no GPU."""
    lib = N.load()
    a = N.JxDAttnArgs()
    a.B, a.Hq, a.Hkv, a.hd, a.T, a.window, a.cache_rows, a.layer_row0 = 20, 32, 8, 128, 768, 0, 20 * 768, 0
    fake = 1 << 20   # never dereferenced: the call fails before touching memory
    a.q = a.k_base = a.v_base = a.out = a.ws = a.counters = a.len_ptr = fake
    a.len_add, a.scale, a.ws_bytes = 2, 128 ** -0.5, 1 << 30
    for rp in (16, 20):
        a.out_rp = rp
        assert lib.jx_decode_attention(a, 0, None) == N.JX_ERR_ARG
        assert b"out_rp" in lib.jx_last_error()
    for impl in (0, 1, 2, 3, 4, 5, 6):
        assert lib.jx_set_decode_attention_impl(impl) == (N.JX_OK if impl <= 5 else N.JX_ERR_ARG)
        assert lib.jx_set_prefill_linear_impl(impl) == (N.JX_OK if impl <= 2 else N.JX_ERR_ARG)
        assert lib.jx_set_prefill_attention_impl(impl) == (N.JX_OK if impl <= 2 else N.JX_ERR_ARG)
    lib.jx_set_decode_attention_impl(0)
    lib.jx_set_prefill_linear_impl(0)
    lib.jx_set_prefill_attention_impl(0)


def test_comm_layout_regions_do_not_overlap():
    """jx_comm_layout (host only): every part of a rank's peer region (header with the all-reduce flags,
    counters, push epoch, bases table and push flags; two pull buffers; 2 x world push receive slots) is
    16-byte aligned, large enough and disjoint, for each world size and message size."""
    lib = N.load()
    for world in (1, 2, 4, 8):
        for max_floats in (4, 1000, 64 * 8192):
            out = (N.LL * 10)()
            assert lib.jx_comm_layout(max_floats, world, out) == N.JX_OK
            size, b0, b1, recv, stride, flags, flag_set, seq, bases, units = list(out)
            assert units == 256 and flag_set == 256 * 8 * 4 and stride >= 4 * max_floats
            parts = [(seq, 8), (bases, 8 * world), (flags, 2 * flag_set), (b0, 4 * max_floats), (b1, 4 * max_floats)]
            parts += [(recv + i * stride, 4 * max_floats) for i in range(2 * world)]
            for off, n in parts:
                assert off % 16 == 0 and off + n <= size
            spans = sorted(parts)
            for (o1, n1), (o2, _) in zip(spans, spans[1:]):
                assert o1 + n1 <= o2, (world, max_floats, spans)
    bad = (N.LL * 10)()
    assert lib.jx_comm_layout(0, 2, bad) == N.JX_ERR_ARG
    assert lib.jx_comm_layout(16, 9, bad) == N.JX_ERR_ARG


def test_filter_logits_checks_its_arguments_before_any_launch():
    """jx_filter_logits refuses null pointers, unsupported sizes and dtypes on the host (no GPU needed)."""
    lib = N.load()
    a = N.JxFilterArgs()
    a.B, a.V, a.ld_in, a.ld_out, a.dtype, a.top_k, a.top_p, a.min_p = 4, 1000, 1000, 1000, N.JX_BF16, 5, 0.9, 0.0
    assert lib.jx_filter_logits(a, None) == N.JX_ERR_ARG            # null logits / out
    a.logits = a.out = 1 << 20                                        # never dereferenced
    for field, value, code in (("V", 0, N.JX_ERR_SHAPE), ("V", 8 * 49152 + 1, N.JX_ERR_SHAPE),
                               ("ld_in", 999, N.JX_ERR_SHAPE), ("ld_out", 10, N.JX_ERR_SHAPE),
                               ("B", 65535, N.JX_ERR_SHAPE), ("dtype", 7, N.JX_ERR_DTYPE)):
        b = N.JxFilterArgs.from_buffer_copy(a)
        setattr(b, field, value)
        if field == "V" and value > 1000:
            b.ld_in = b.ld_out = value
        assert lib.jx_filter_logits(b, None) == code, (field, value)
    b = N.JxFilterArgs.from_buffer_copy(a)
    b.B = 0
    assert lib.jx_filter_logits(b, None) == N.JX_OK                   # nothing to do


def test_tensor_core_prefill_attention_refuses_unsupported_shapes_before_any_launch():
    """With the tcgen05 prefill attention selected, head sizes other than 64 / 128 / 256, a row-major output,
    S > T or Hq % Hkv != 0 fail with JX_ERR_SHAPE before any device work (the pointers are never
    dereferenced)."""
    lib = N.load()
    fake = 1 << 20
    a = N.JxPAttnArgs()
    a.B, a.S, a.Hq, a.Hkv, a.hd, a.T, a.window = 2, 64, 8, 2, 128, 128, 0
    a.cache_rows, a.layer_row0 = 2 * 128, 0
    a.q = a.k_base = a.v_base = a.out = a.len_ptr = fake
    a.len_add, a.scale, a.out_rp = 1, 128 ** -0.5, 128
    assert lib.jx_set_prefill_attention_impl(2) == N.JX_OK
    try:
        for field, value in (("hd", 32), ("hd", 96), ("out_rp", 0), ("S", 200), ("Hkv", 3)):
            saved = getattr(a, field)
            setattr(a, field, value)
            assert lib.jx_prefill_attention(a, 0, None) == N.JX_ERR_SHAPE, field
            setattr(a, field, saved)
    finally:
        lib.jx_set_prefill_attention_impl(0)
