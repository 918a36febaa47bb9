"""The C-ABI library: loads without a GPU, exports every header symbol, and
rejects bad arguments before touching the device. CPU only (no compute calls)."""
import ctypes
import os

import pytest
import torch

from swiglu_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_exports_every_header_symbol(lib):
    syms = _lib.header_symbols()
    assert len(syms) >= 13
    for s in syms:
        assert hasattr(lib, s), s
    # Every declared symbol has a binding signature (no unbound entry points).
    assert set(syms) == set(_lib._SIGNATURES)


def test_abi_version_and_status_strings(lib):
    assert lib.swiglu_b200_abi_version() == 1
    assert lib.swiglu_b200_status_string(0) == b"SWIGLU_OK"
    assert lib.swiglu_b200_status_string(1) == b"SWIGLU_ERR_INVALID_ARGUMENT"
    assert lib.swiglu_b200_status_string(5) == b"SWIGLU_ERR_DEVICE_TIMEOUT"
    assert lib.swiglu_b200_status_string(99) == b"SWIGLU_ERR_UNKNOWN"


def _p(v):
    return ctypes.c_void_p(v)


@pytest.mark.parametrize("args,fragment", [
    # unknown dtype
    ((_p(16), _p(16), _p(16), 8, 8, 8, 0, 0, 7, 1, 16, _p(0)), b"dtype"),
    # bad layout flag
    ((_p(16), _p(16), _p(16), 8, 8, 8, 2, 0, 1, 1, 16, _p(0)), b"layout"),
    # null pointer
    ((_p(0), _p(16), _p(16), 8, 8, 8, 0, 0, 1, 1, 16, _p(0)), b"null"),
    # K = 0
    ((_p(16), _p(16), _p(16), 8, 8, 0, 0, 0, 1, 1, 16, _p(0)), b"K must be positive"),
    # f32 GEMM cannot write bf16
    ((_p(16), _p(16), _p(16), 8, 8, 8, 0, 0, 0, 1, 16, _p(0)), b"f32"),
    # negative size
    ((_p(16), _p(16), _p(16), -1, 8, 8, 0, 0, 1, 1, 16, _p(0)), b"dimensions"),
])
def test_matmul_rejects_bad_arguments(lib, args, fragment):
    rc = lib.swiglu_b200_matmul(*args)
    assert rc == 1
    assert fragment in lib.swiglu_b200_last_error_message()


def test_swiglu_forward_argument_checks(lib):
    f = lib.swiglu_b200_fused_matmul_swiglu_save_preact
    # packed layout needs H % 128 == 0
    assert f(_p(16), _p(16), _p(16), _p(0), 128, 64, 96, 1, 1, 1, 0, 16, _p(0)) == 1
    assert b"128" in lib.swiglu_b200_last_error_message()
    # packed layout only with the [D, 2H] weight form
    assert f(_p(16), _p(16), _p(16), _p(0), 128, 64, 128, 1, 0, 1, 0, 16, _p(0)) == 1
    # group size must be positive
    assert f(_p(16), _p(16), _p(16), _p(0), 128, 64, 128, 1, 1, 0, 0, 0, _p(0)) == 1


def test_pack_rejects_alias_and_bad_block(lib):
    f = lib.swiglu_b200_pack_weight_chunked
    assert f(_p(16), _p(16), 4, 256, 128, 1, 0, _p(0)) == 1
    assert f(_p(16), _p(32), 4, 250, 128, 1, 0, _p(0)) == 1


def test_check_raises_with_detail(lib):
    rc = lib.swiglu_b200_bwd_dw2(_p(0), _p(16), _p(16), 8, 8, 8, 1, 0, _p(0))
    with pytest.raises(_lib.SwigluError, match="SWIGLU_ERR_INVALID_ARGUMENT: null pointer"):
        _lib.check(rc)


def test_synthetic_inputs_match_the_oracle_draw():
    """bench.py and the TP bench draw their inputs with swiglu_b200.synthetic,
    the tests with the oracle's copy: same seed, same bits."""
    from oracle import swiglu_oracle as O
    from swiglu_b200.synthetic import make_inputs

    for shape, seed, dtype in [((64, 48, 40, 24), 0, torch.float32), ((33, 16, 8, 8), 7, torch.bfloat16)]:
        for a, b in zip(make_inputs(*shape, seed=seed, dtype=dtype), O.make_inputs(*shape, seed=seed, dtype=dtype)):
            assert torch.equal(a, b)


def test_device_drawn_inputs_have_the_configured_distributions():
    """The large-shape draw (on the device; here on the CPU generator): same
    shapes, dtype and scales as make_inputs, reproducible for a seed."""
    from swiglu_b200.synthetic import make_inputs_on_device

    M, D, H, Dout = 512, 256, 384, 128
    a = make_inputs_on_device(M, D, H, Dout, "cpu", seed=3)
    b = make_inputs_on_device(M, D, H, Dout, "cpu", seed=3)
    assert [t.shape for t in a] == [(M, D), (2 * H, D), (Dout, H), (M, Dout)]
    assert all(t.dtype == torch.bfloat16 for t in a)
    assert all(torch.equal(u, v) for u, v in zip(a, b))
    for t, std in zip(a, (1.0, D ** -0.5, H ** -0.5, 1.0)):
        assert abs(t.float().std().item() / std - 1.0) < 0.05
        assert abs(t.float().mean().item()) < 0.05 * std


@pytest.mark.parametrize("M,N,tile_n,family", [
    (11136, 3584, 0, 2),     # config 2 y = h . W2^T: 4 waves of 256 x 512 tiles -> 256 x 256
    (3584, 14336, 0, 2),     # config 2 dW2: 5 waves -> 256 x 256
    (28672, 3584, 0, 3),     # config 2 dW1 shape: 10.6 waves -> 256 x 512 even without the hint
    (11136, 3584, 512, 3),   # config 2 dx with the backward's hint
    (65536, 8192, 0, 3),     # config 5 y: 55 waves
    (8192, 28672, 0, 3),     # config 5 dW2: 24 waves
    (65536, 8192, 256, 2),   # an explicit 256 keeps the narrow tiles
    (65536, 2048, 0, 3),     # the GPU size-rule tests' shapes
    (4096, 20480, 0, 3),
    (2560, 4096, 0, 2),      # the stream-K test shape
    (256, 512, 0, 1),        # less than a wave of pairs -> single-SM kernel
])
def test_gemm_plan_size_rule(M, N, tile_n, family):
    """The kernel-family choice of the plain GEMM, host-only, on a 148-SM B200."""
    assert _lib.gemm_plan(M, N, tile_n, 148) == family


def test_gemm_plan_honours_forced_path_and_rejects_bad_widths():
    try:
        for mode in (1, 2, 3):
            _lib.set_gemm_path(mode)
            assert _lib.gemm_plan(65536, 8192) == mode
    finally:
        _lib.set_gemm_path(0)
    with pytest.raises(_lib.SwigluError, match="tile_n"):
        _lib.gemm_plan(1024, 1024, 384)


@pytest.mark.parametrize("M,K,H,family", [
    (11136, 3584, 14336, 2),    # config 2 GEMM1: K below 8192 -> 256 x 256
    (65536, 8192, 28672, 3),    # config 5 GEMM1: K = 8192, 98 waves -> 256 x 512
    (65536, 8192, 28672 // 8, 3),  # config 5 per rank at 8-way tensor parallel: 12 waves
    (4096, 8192, 2048, 2),      # a wave of pairs but under 8 waves of 256 x 512 tiles
    (256, 8192, 256, 1),        # less than a wave of pairs
    (8192, 8192, 8192, 3),      # the GPU test's shape
])
def test_swiglu_fwd_plan_size_rule(M, K, H, family):
    """GEMM1 + SwiGLU takes 256 x 512 tiles by size only from K >= 8192."""
    assert _lib.swiglu_fwd_plan(M, K, H, 148) == family


def test_swiglu_fwd_plan_honours_forced_path_and_rejects_bad_arguments():
    try:
        for mode in (1, 2, 3):
            _lib.set_gemm_path(mode)
            assert _lib.swiglu_fwd_plan(11136, 3584, 14336) == mode
    finally:
        _lib.set_gemm_path(0)
    with pytest.raises(_lib.SwigluError, match="num_sms"):
        _lib.swiglu_fwd_plan(11136, 3584, 14336, 1)
    with pytest.raises(_lib.SwigluError):
        _lib.swiglu_fwd_plan(-1, 3584, 14336)
    rc = _lib.load().swiglu_b200_swiglu_fwd_plan(1024, 1024, 1024, 148, None)   # null result pointer
    assert rc != _lib.OK
    assert b"null" in _lib.load().swiglu_b200_last_error_message()


C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "swiglu_b200.h"

int main(void) {
  int fam = 0;
  if (swiglu_b200_abi_version() <= 0) return 10;
  if (swiglu_b200_gemm_plan(65536, 8192, 0, 148, &fam) != SWIGLU_OK || fam != 3) return 11;
  if (swiglu_b200_gemm_plan(11136, 3584, 0, 148, &fam) != SWIGLU_OK || fam != 2) return 12;
  if (swiglu_b200_gemm_plan(1024, 1024, 384, 148, &fam) != SWIGLU_ERR_INVALID_ARGUMENT) return 13;
  if (!strstr(swiglu_b200_last_error_message(), "tile_n")) return 14;
  if (strcmp(swiglu_b200_status_string(SWIGLU_OK), "SWIGLU_OK") != 0) return 15;
  /* a null device pointer is rejected before any device work */
  if (swiglu_b200_matmul(NULL, NULL, NULL, 256, 256, 64, 0, 0, SWIGLU_BF16, SWIGLU_BF16, 8, NULL)
      != SWIGLU_ERR_INVALID_ARGUMENT) return 16;
  printf("ok %d\n", swiglu_b200_abi_version());
  return 0;
}
"""


def test_header_compiles_as_c99_and_a_c_caller_links(tmp_path):
    """The boundary as a C caller sees it: the header is plain C99, the
    library links with -lswiglu_b200, and the host-only calls and argument
    checks behave as documented (no GPU needed)."""
    import shutil
    import subprocess

    from swiglu_b200.build import INCLUDE_DIR, LIB_PATH

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    libdir = os.path.dirname(LIB_PATH)
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-pedantic", f"-I{INCLUDE_DIR}", str(src),
                    f"-L{libdir}", "-lswiglu_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.startswith("ok ")


def _header_prototypes():
    import re
    with open(_lib.HEADER) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    protos = {}
    for ret, name, params in re.findall(r"\b(int|const char\s*\*)\s*(swiglu_b200_\w+)\s*\(([^)]*)\)\s*;", text):
        params = " ".join(params.split())
        protos[name] = ([] if params in ("", "void") else [p.strip() for p in params.split(",")], ret)
    return protos


_SCALARS = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t,
            "uint32_t": ctypes.c_uint32}


def test_binding_signatures_match_the_header_prototypes():
    """Every ctypes argument list has the header's arity, integer widths and
    pointer positions, so a Python (or INTEGRATION-style) caller cannot pass
    an int where the library reads an int64 or a pointer."""
    protos = _header_prototypes()
    assert set(protos) == set(_lib._SIGNATURES)
    for name, (params, ret) in protos.items():
        argtypes = _lib._SIGNATURES[name]
        assert len(params) == len(argtypes), name
        for decl, at in zip(params, argtypes):
            ctype = decl.rsplit(" ", 1)[0] if not decl.endswith("*") else decl
            if "*" in decl:
                assert at is ctypes.c_void_p or issubclass(at, ctypes._Pointer), (name, decl)
                if issubclass(at, ctypes._Pointer):
                    # pointee: a pointer (T* const* = an array of pointers) or a scalar
                    base = ctype.replace("const", "").replace("*", "").split()[0]
                    pointee_is_ptr = decl.count("*") >= 2
                    want = ctypes.c_void_p if pointee_is_ptr or base == "void" else _SCALARS[base]
                    assert at._type_ is want, (name, decl)
            else:
                assert at is _SCALARS[ctype.replace("const", "").strip()], (name, decl)
        want_ret = ctypes.c_char_p if "char" in ret else ctypes.c_int
        assert _lib._RESTYPES.get(name, ctypes.c_int) is want_ret, name


def test_sm_reserve_range(lib):
    assert lib.swiglu_b200_set_sm_reserve(-1) == 1
    assert lib.swiglu_b200_set_sm_reserve(65) == 1
    assert b"SM reserve" in lib.swiglu_b200_last_error_message()
    assert lib.swiglu_b200_set_sm_reserve(8) == 0
    assert lib.swiglu_b200_set_sm_reserve(0) == 0
