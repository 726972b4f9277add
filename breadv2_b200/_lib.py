"""ctypes binding of libbread_b200.so (the C ABI in include/bread_b200.h).

The library is built in-tree by ``breadv2_b200.build``.  Loading fails loudly
when it is missing: there is no CPU or PyTorch fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbread_b200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_LL = ctypes.c_longlong
_U64 = ctypes.c_uint64

# entry point -> (restype, argtypes); every symbol declared extern "C" in the header
SIGNATURES = {
    "bread_status_string": (ctypes.c_char_p, [_I]),
    "bread_last_error": (ctypes.c_char_p, []),
    "bread_device_error": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "bread_matvec_f16": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "bread_matvec_f32": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "bread_matvec_batch_f32": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "bread_dequant": (_I, [_P, _P, _LL, _I, _P]),
    "bread_lm_head_argmax": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "bread_rmsnorm_half_c": (_I, [_P, _P, _I, _F, _P]),
    "bread_silu_mul_c": (_I, [_P, _P, _I, _P]),
    "bread_scale_accum_c": (_I, [_P, _P, _F, _I, _P]),
    "bread_copy_half_c": (_I, [_P, _P, _I, _P]),
    "bread_moe_route": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "bread_moe_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "bread_moe_ffn": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "bread_moe_ffn_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "bread_gguf_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "bread_gguf_close": (_I, [_P]),
    "bread_gguf_info": (_I, [_P, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(_U64), ctypes.POINTER(ctypes.c_uint32),
                             ctypes.POINTER(_U64)]),
    "bread_gguf_tensor": (_I, [_P, _U64, _P]),
    "bread_gguf_find": (_I, [_P, ctypes.c_char_p, _P]),
    "bread_gguf_read": (_I, [_P, _U64, _P, _U64]),
    "bread_stack_create": (_I, [ctypes.POINTER(_P), _P]),
    "bread_stack_create_gguf": (_I, [ctypes.POINTER(_P), ctypes.c_char_p, _P]),
    "bread_stack_destroy": (_I, [_P]),
    "bread_stack_device_bytes": (_SZ, [_P]),
    "bread_stack_get_config": (_I, [_P, _P]),
    "bread_stack_layer": (_I, [_P, _I] + [ctypes.POINTER(_P)] * 8 + [ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "bread_stack_norm_weight": (_I, [_P, _I, _P, ctypes.POINTER(_I)]),
    "bread_stack_mailbox": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_SZ)]),
    "bread_stack_set_peers": (_I, [_P, ctypes.POINTER(_P), _I]),
    "bread_stack_set_peer_timeout": (_I, [_P, ctypes.c_double]),
    "bread_ipc_get_handle": (_I, [_P, _P]),
    "bread_ipc_open_handle": (_I, [_P, ctypes.POINTER(_P)]),
    "bread_ipc_close_handle": (_I, [_P]),
    "bread_stack_step": (_I, [_P, _P, _I, _P]),
    "bread_stack_step_host": (_I, [_P, _P, _P, _I, _P]),
    "bread_stack_launches_per_step": (_I, [_P, _I]),
    "bread_stack_profile_step": (_I, [_P, _P, _I, _P, _P]),
    "bread_stack_profile_stamps": (_I, [_P, _P, _SZ, ctypes.POINTER(_I)]),
    "bread_stack_routing_stats": (_I, [_P, _P, _P]),
    "bread_stack_routing": (_I, [_P, _P, _P, _P, ctypes.POINTER(_I)]),
    "bread_synth_blocks": (_I, [_P, _LL, _I, _U64, _U64, _P]),
    "bread_synth_normal_f32": (_I, [_P, _LL, _F, _U64, _U64, _P]),
    "bread_synth_normal_f16": (_I, [_P, _LL, _F, _U64, _U64, _P]),
    "bread_synth_blocks_host": (_I, [_P, _LL, _I, _U64, _U64]),
    "bread_synth_normal_f32_host": (_I, [_P, _LL, _F, _U64, _U64]),
    "bread_synth_normal_f16_host": (_I, [_P, _LL, _F, _U64, _U64]),
}

# C++-linkage drop-ins (reference kernels.cu:289, layer_logic.cu:28-31)
MANGLED = {
    "bread_matvec": "_Z12bread_matvecPvP6__halfS1_iiiP11CUstream_st",
    "bread_rmsnorm_half": "_Z18bread_rmsnorm_halfP6__halfPKfifP11CUstream_st",
    "bread_silu_mul": "_Z14bread_silu_mulP6__halfPKS_iP11CUstream_st",
    "bread_scale_accum": "_Z17bread_scale_accumP6__halfPKS_fiP11CUstream_st",
    "bread_copy_half": "_Z15bread_copy_halfP6__halfPKS_iP11CUstream_st",
}


class BreadError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({last_error()})")


class GgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
                ("dims", _U64 * 4), ("offset", _U64), ("size", _U64), ("n_elems", _U64)]


class StackConfig(ctypes.Structure):
    _fields_ = [("n_layers", _I), ("hidden", _I), ("inter", _I), ("n_experts", _I), ("top_k", _I),
                ("max_tokens", _I), ("shared_expert", _I), ("norm_eps", _F), ("seed", _U64), ("rank", _I),
                ("world", _I), ("norm_weight", _I)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m breadv2_b200.build` (there is no fallback path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_string(st: int) -> str:
    return lib().bread_status_string(st).decode()


def last_error() -> str:
    return lib().bread_last_error().decode()


def check(st: int, what: str) -> None:
    if st != 0:
        raise BreadError(st, what)


def device_error(clear: bool = True) -> int:
    w = ctypes.c_uint(0)
    check(lib().bread_device_error(ctypes.byref(w), int(clear)), "bread_device_error")
    return w.value
