"""ctypes binding of libduo_mixer.so (the C ABI declared in include/duo_mixer.h).

The library is built in-tree by duo-mech-interp_b200/build.py.  There is no fallback: if it is missing or fails to
load, every call raises.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libduo_mixer.so")

DUO_OK, DUO_EINVAL, DUO_ECUDA, DUO_ESTATE, DUO_ENOMEM = 0, -1, -2, -3, -4
DUO_F32, DUO_BF16, DUO_F16, DUO_I8, DUO_I32 = 0, 1, 2, 3, 4
DUO_PUSH_ADD, DUO_PUSH_MUL = 0, 1
DUO_ALL_NEURONS = -1
DUO_CAP_RESID, DUO_CAP_RESID_ATTN, DUO_CAP_ACT = 0, 1, 2
DUO_STATS_COLS = 6

# every symbol the header declares, with (restype, argtypes)
_vp, _i, _f, _u = C.c_void_p, C.c_int, C.c_float, C.c_uint


class duo_config(C.Structure):
    _fields_ = [("hidden", _i), ("inter", _i), ("vocab", _i), ("layers", _i), ("nh", _i), ("nkv", _i), ("hd", _i),
                ("rot", _i), ("theta", _f), ("eps", _f), ("hk", _i), ("hv", _i), ("dk", _i), ("dv", _i), ("ks", _i),
                ("full_attention_host", _vp), ("group", _i), ("act_dtype", _i)]


class duo_q8_view(C.Structure):
    _fields_ = [("q", _vp), ("s", _vp)]


class duo_layer_view(C.Structure):
    _fields_ = [("in_norm", _vp), ("post_norm", _vp), ("proj", duo_q8_view), ("out", duo_q8_view),
                ("gu", duo_q8_view), ("down", duo_q8_view), ("conv", _vp), ("a_log", _vp), ("dt_bias", _vp),
                ("gnorm", _vp), ("q_norm", _vp), ("k_norm", _vp)]


class duo_weights_view(C.Structure):
    _fields_ = [("embed", duo_q8_view), ("final_norm", _vp), ("layers_host", _vp)]


SIGNATURES = {
    "duo_last_error": (C.c_char_p, []),
    "duo_abi_version": (_i, []),
    "duo_q8_quantize": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    "duo_q8_dequantize": (_i, [_vp, _vp, _i, _i, _i, _vp, _i, _vp]),
    "duo_q8_gemv": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp]),
    "duo_q8_gather": (_i, [_vp, _i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "duo_gemm_bf16": (_i, [_vp, _i, _i, _vp, _i, _vp, _vp, _i, _i, _i, _vp]),
    "duo_q8_gemm": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _i, _i, _vp, _i, _i, _i, _vp]),
    "duo_gemm_swiglu": (_i, [_vp, _i, _i, _vp, _i, _i, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "duo_rmsnorm": (_i, [_vp, _i, _i, _vp, _f, _i, _vp, _i, _vp]),
    "duo_gdn_conv_fwd": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "duo_gdn_recurrent_fwd": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "duo_gdn_chunk_fwd": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "duo_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
    "duo_attention_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _vp]),
    "duo_token_extremes": (_i, [_vp, _i, _i, _i, _i, _vp, _vp]),
    "duo_engine_set_capture": (_i, [_vp, _i, _i, _vp, _vp, _i]),
    "duo_engine_set_capture_t0": (_i, [_vp, _i, _i]),
    "duo_engine_set_stop_after": (_i, [_vp, _i]),
    "duo_push_stats": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "duo_fault_status": (_i, [C.POINTER(_u)]),
    "duo_fault_raise": (_i, [_u]),
    "duo_engine_create": (_i, [C.POINTER(duo_config), C.POINTER(_vp)]),
    "duo_engine_destroy": (None, [_vp]),
    "duo_engine_load": (_i, [_vp, C.POINTER(duo_weights_view), _vp]),
    "duo_engine_alloc": (_i, [_vp, _i, _i, _i]),
    "duo_engine_reset": (_i, [_vp, _i, _vp]),
    "duo_engine_set_vectors": (_i, [_vp, _vp, _i, _vp]),
    "duo_engine_set_head_scales": (_i, [_vp, _i, _vp, _vp]),
    "duo_engine_set_pushes": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "duo_engine_forward": (_i, [_vp, _vp, _i, _i, _i, _i, _vp]),
    "duo_engine_forward_device": (_i, [_vp, _vp, _i, _i, _i, _i, _vp]),
    "duo_engine_logits": (_i, [_vp, _i, _i, _vp, _vp]),
    "duo_engine_argmax": (_i, [_vp, _i, _i, _vp, _vp]),
    "duo_engine_generate": (_i, [_vp, _i, _i, _vp, _vp]),
    "duo_engine_row_len": (_i, [_vp, _i]),
    "duo_launch_count": (C.c_ulonglong, []),
    "duo_engine_reset_all": (_i, [_vp, _vp]),
    "duo_engine_capture_resid": (_i, [_vp, _i, _vp]),
    "duo_engine_profile": (_i, [_vp, _u]),
    "duo_engine_profile_read": (_i, [_vp, C.POINTER(C.c_double), C.POINTER(C.c_longlong)]),
}

# profiling classes of duo_engine_profile (enum duo_prof_kind)
PROF_KINDS = ["gather", "rmsnorm", "gemv", "gemm", "gdn_conv", "gdn_scan", "attn_prep", "attn", "swiglu", "other"]


class DuoError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"duo error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Load the library once (raises if it is absent: there is no CPU or PyTorch fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with duo-mech-interp_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status is not None and status < 0:
        raise DuoError(status, lib().duo_last_error().decode(errors="replace"))
    return status


def call(name, *args):
    return check(getattr(lib(), name)(*args))


def ptr(t):
    """Device (or host) address of a tensor, None for None."""
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def dtype_code(dt):
    import torch
    return {torch.float32: DUO_F32, torch.bfloat16: DUO_BF16, torch.float16: DUO_F16, torch.int8: DUO_I8,
            torch.int32: DUO_I32}[dt]
