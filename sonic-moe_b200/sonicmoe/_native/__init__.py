"""ctypes binding of libsonic_b200.so (the C ABI in include/sonic_b200.h).

The library is the only compute path of this package: if it is missing, importing the ops raises
instead of falling back to anything else.  Build it with ``python sonic-moe_b200/build.py``.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsonic_b200.so")

SM_OK = 0
SM_EIO = -5
SM_EINVAL = -22
SM_ENOTSUP = -95

DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2

ERR_NAMES = {
    101: "TMA producer wait timed out",
    102: "MMA issuer wait timed out",
    103: "epilogue wait timed out",
    104: "drain wait timed out",
    201: "expert index outside [0, E)",
    202: "up-projection row without a valid home row (home-down expert parallel)",
    203: "exchange count outside the expert-parallel buffers (device-side counts)",
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "sm_last_error": (ctypes.c_char_p, []),
    "sm_version": (ctypes.c_char_p, []),
    "sm_router_topk": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "sm_router_fused_workspace": (_SZ, [_I, _I]),
    "sm_router_fused": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P, _P]),
    "sm_moe_forward_fused_router": (
        _I,
        [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_route_metadata_workspace": (_SZ, [_I, _I, _I]),
    "sm_route_metadata": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "sm_general_route_metadata": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "sm_route_metadata_noalloc": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "sm_quant_1x128": (_I, [_P, _I, _I, _P, _P, _P]),
    "sm_weight_sf_bytes": (_SZ, [_I, _I, _I]),
    "sm_weight_prep": (_I, [_P, _I, _I, _I, _I, _P, _P, _P]),
    "sm_moe_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "sm_moe_forward": (
        _I,
        [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_moe_general_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "sm_moe_general_forward": (
        _I,
        [_P, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_max_padded_blocks": (_I, [_LL, _I]),
    "sm_moe_down_slices": (_I, [_I, _I]),
    "sm_ep_record_bytes": (_I, [_I, _I]),
    "sm_ep_dispatch_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "sm_ep_dispatch_prepare": (
        _I,
        [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_ep_expert_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "sm_ep_expert_forward": (
        _I,
        [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_ep_combine": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "sm_set_gemm_sm_reserve": (_I, [_I]),
    "sm_selftest_bounded_wait": (_I, [_P, _P]),
    "sm_ep_expert_forward_p2p": (
        _I,
        [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_ep_combine_p2p": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "sm_ep_dispatch_records": (
        _I,
        [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P],
    ),
    "sm_ep_expert_up_p2p": (
        _I,
        [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _LL, _P, _P, _SZ, _P, _P],
    ),
    "sm_ep_expert_up_home": (
        _I,
        [_P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _LL, _P, _P, _SZ, _P, _P],
    ),
    "sm_ipc_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    "sm_ipc_open": (_I, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "sm_ipc_close": (_I, [_P]),
    "sm_ipc_free": (_I, [_P]),
    "sm_copy_d2d_async": (_I, [_P, _P, _SZ, _P]),
    "sm_route_plan": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "sm_quant_pack": (_I, [_P, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P]),
    "sm_general_route_plan": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P, _P]),
    "sm_quant_pack_general": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "sm_moe_up": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "sm_moe_up_preact": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "sm_weight_prep_t": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "sm_weight_prep_with_t": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "sm_moe_dact": (
        _I,
        [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P],
    ),
    "sm_tq_pack": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "sm_tq_pack_dual": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P]),
    "sm_moe_wgrad": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "sm_router_bwd": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "sm_moe_down_combine": (
        _I,
        [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    ),
}

_lib = None


class SonicError(RuntimeError):
    """A non-zero return from libsonic_b200 (message from sm_last_error)."""

    def __init__(self, code, message):
        super().__init__(f"libsonic_b200 error {code}: {message}")
        self.code = code


def load():
    """Load the library (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with `python sonic-moe_b200/build.py` "
            "(this package has no CPU or non-CUDA fallback)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int):
    if rc != SM_OK:
        msg = load().sm_last_error().decode(errors="replace")
        if rc == SM_EINVAL:
            raise ValueError(msg)
        if rc == SM_ENOTSUP:
            raise NotImplementedError(msg)
        raise SonicError(rc, msg)


def call(name: str, *args):
    check(getattr(load(), name)(*args))
