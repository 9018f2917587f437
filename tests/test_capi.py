"""CPU tests of the C ABI: the library loads, exports every entry point include/duo_mixer.h declares, and rejects
bad arguments with a status and a message before touching a GPU (the reference throws on shape limits,
engine/model.js:52, 406, 418)."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "duo_mixer.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(duo_\w+)\s*\(", text)) - {"duo_config", "duo_q8_view"})


@pytest.fixture(scope="module")
def L():
    from duo import lib as dl
    return dl


def test_library_exports_every_declared_symbol(L):
    lib = L.lib()
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding knows every one of them
    assert sorted(set(names) - set(L.SIGNATURES)) == []


def test_abi_version(L):
    assert L.lib().duo_abi_version() >= 1


def test_bad_arguments_return_status_and_message(L):
    lib = L.lib()
    st = lib.duo_q8_quantize(None, L.DUO_F32, 4, 100, 128, None, None, None)  # k not a multiple of the group
    assert st == L.DUO_EINVAL
    assert b"multiple" in lib.duo_last_error()
    st = lib.duo_q8_gemv(None, L.DUO_F32, 9, 128, None, None, 128, 4, None, L.DUO_F32, 0, None)
    assert st == L.DUO_EINVAL
    st = lib.duo_gemm_bf16(None, 4, 100, None, 4, None, None, L.DUO_F32, 4, 0, None)
    assert st == L.DUO_EINVAL and b"64" in lib.duo_last_error()
    st = lib.duo_gdn_recurrent_fwd(None, None, None, L.DUO_F32, None, None, None, None, L.DUO_F32, 1, 1, 1, 64, 128,
                                   1, None)
    assert st == L.DUO_EINVAL and b"128" in lib.duo_last_error()
    st = lib.duo_attention(None, None, None, None, None, 0, None, 7, 1, 1, 8, 2, 256, 16, 1.0, None)
    assert st == L.DUO_EINVAL


def test_projection_and_scan_arguments_are_checked_first(L):
    """Shape, dtype and table checks of the projection and scan entry points return a status before any device work."""
    lib = L.lib()
    # fused gate|up + SwiGLU: inter a multiple of 64, ldo >= inter, a push table when there are pushes, rows in it
    st = lib.duo_gemm_swiglu(None, 4, 64, None, 100, L.DUO_BF16, None, None, 100, None, None, None, 0, 0, 1, 0, None)
    assert st == L.DUO_EINVAL and b"64" in lib.duo_last_error()
    st = lib.duo_gemm_swiglu(None, 4, 64, None, 128, L.DUO_F32, None, None, 128, None, None, None, 0, 0, 1, 0, None)
    assert st == L.DUO_EINVAL and b"bf16 or f16" in lib.duo_last_error()
    st = lib.duo_gemm_swiglu(None, 4, 64, None, 128, L.DUO_BF16, None, None, 128, None, None, None, 0, 0, 1, 0, None)
    assert st == L.DUO_EINVAL and b"null" in lib.duo_last_error()
    sentinel = C.c_void_p(16)  # never dereferenced: the checks fail first
    st = lib.duo_gemm_swiglu(sentinel, 4, 64, sentinel, 128, L.DUO_BF16, None, sentinel, 64, None, None, None, 0, 0,
                             1, 0, None)
    assert st == L.DUO_EINVAL and b"ldo" in lib.duo_last_error()
    st = lib.duo_gemm_swiglu(sentinel, 4, 64, sentinel, 128, L.DUO_BF16, None, sentinel, 128, None, None, None, 2, 4,
                             1, 0, None)
    assert st == L.DUO_EINVAL and b"push table" in lib.duo_last_error()
    st = lib.duo_gemm_swiglu(sentinel, 4, 64, sentinel, 128, L.DUO_BF16, None, sentinel, 128, sentinel, sentinel,
                             sentinel, 1, 2, 1, 0, None)  # 4 rows of A, 2 rows in the push table
    assert st == L.DUO_EINVAL and b"push table" in lib.duo_last_error()
    # int8 decode GEMM: at most 256 rows, the group a multiple of 64 dividing k, x 16-bit, SwiGLU n a multiple of 128
    st = lib.duo_q8_gemm(sentinel, L.DUO_BF16, 300, 128, sentinel, sentinel, 128, 128, 0, sentinel, L.DUO_F32, 128, 0,
                         None)
    assert st == L.DUO_EINVAL and b"256" in lib.duo_last_error()
    st = lib.duo_q8_gemm(sentinel, L.DUO_BF16, 4, 128, sentinel, sentinel, 32, 128, 0, sentinel, L.DUO_F32, 128, 0,
                         None)
    assert st == L.DUO_EINVAL and b"group" in lib.duo_last_error()
    st = lib.duo_q8_gemm(sentinel, L.DUO_F32, 4, 128, sentinel, sentinel, 128, 128, 0, sentinel, L.DUO_F32, 128, 0,
                         None)
    assert st == L.DUO_EINVAL and b"bf16 or f16" in lib.duo_last_error()
    st = lib.duo_q8_gemm(sentinel, L.DUO_BF16, 4, 128, sentinel, sentinel, 128, 192, 1, sentinel, L.DUO_BF16, 96, 0,
                         None)
    assert st == L.DUO_EINVAL and b"SwiGLU" in lib.duo_last_error()
    # the residual-add GEMM accumulates into f32 only
    st = lib.duo_gemm_bf16(sentinel, 4, 64, sentinel, 4, None, sentinel, L.DUO_BF16, 4, 1, None)
    assert st == L.DUO_EINVAL and b"f32" in lib.duo_last_error()
    # chunked scan: head dims 128, one dtype for q/k/v/o
    st = lib.duo_gdn_chunk_fwd(None, None, None, L.DUO_BF16, None, None, None, None, L.DUO_BF16, 1, 64, 1, 64, 128, 1,
                               None)
    assert st == L.DUO_EINVAL and b"128" in lib.duo_last_error()
    st = lib.duo_gdn_chunk_fwd(None, None, None, L.DUO_BF16, None, None, None, None, L.DUO_F32, 1, 64, 1, 128, 128, 1,
                               None)
    assert st == L.DUO_EINVAL and b"dtype" in lib.duo_last_error()


def test_engine_rejects_bad_config_and_null_handle(L):
    lib = L.lib()
    full = (C.c_uint8 * 4)(0, 0, 0, 1)
    cfg = L.duo_config(hidden=1024, inter=3584, vocab=1000, layers=4, nh=8, nkv=2, hd=128, rot=64, theta=1e7,
                       eps=1e-6, hk=16, hv=16, dk=128, dv=128, ks=4, full_attention_host=C.cast(full, C.c_void_p),
                       group=128, act_dtype=L.DUO_BF16)
    h = C.c_void_p()
    assert lib.duo_engine_create(C.byref(cfg), C.byref(h)) == L.DUO_EINVAL  # hd must be 256
    assert b"hd" in lib.duo_last_error()
    cfg.hd, cfg.dk = 256, 64
    assert lib.duo_engine_create(C.byref(cfg), C.byref(h)) == L.DUO_EINVAL
    assert lib.duo_engine_alloc(None, 3, 64, 64) == L.DUO_EINVAL
    assert lib.duo_engine_forward(None, None, 0, 1, 1, -1, None) == L.DUO_EINVAL
    assert lib.duo_engine_row_len(None, 0) == L.DUO_EINVAL


def test_python_errors_raise(L):
    with pytest.raises(L.DuoError):
        L.call("duo_q8_quantize", None, L.DUO_F32, 4, 100, 128, None, None, None)


def test_engine_calls_refuse_work_after_a_fault(L):
    """A bounded wait that gave up inside a kernel reaches the host through a mirrored fault word; every engine call
    reads it before anything else and returns DUO_ECUDA without launching a kernel, until duo_fault_status reads and
    clears it.  Here the word is set from the host (duo_fault_raise), the way a mirrored device fault would appear:
    no device fault is involved."""
    lib = L.lib()
    n0 = lib.duo_launch_count()
    assert lib.duo_fault_raise(16) == L.DUO_OK
    calls = {
        "forward": lambda: lib.duo_engine_forward(None, None, 0, 1, 1, -1, None),
        "forward_device": lambda: lib.duo_engine_forward_device(None, None, 0, 1, 1, -1, None),
        "logits": lambda: lib.duo_engine_logits(None, 0, 1, None, None),
        "argmax": lambda: lib.duo_engine_argmax(None, 0, 1, None, None),
        "generate": lambda: lib.duo_engine_generate(None, 4, -1, None, None),
    }
    for name, call in calls.items():
        assert call() == L.DUO_ECUDA, name
        msg = lib.duo_last_error()
        assert b"gave up" in msg and b"fault code 16" in msg, (name, msg)
    assert lib.duo_launch_count() == n0  # nothing was launched
    code = C.c_uint(0)
    assert lib.duo_fault_status(C.byref(code)) == L.DUO_OK
    assert code.value == 16
    assert lib.duo_fault_status(C.byref(code)) == L.DUO_OK and code.value == 0  # read and cleared
    # the gate is open again: what fails now is the null handle
    assert lib.duo_engine_forward(None, None, 0, 1, 1, -1, None) == L.DUO_EINVAL
