"""ctypes binding of libinferno_b200.so (C ABI in include/inferno_b200.h).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinferno_b200.so")

IFR_OK, IFR_ERR_ARG, IFR_ERR_CUDA, IFR_ERR_NOMEM, IFR_ERR_TIMEOUT, IFR_ERR_UNSUPPORTED = range(6)
ERR_NAMES = {1: "IFR_ERR_ARG", 2: "IFR_ERR_CUDA", 3: "IFR_ERR_NOMEM", 4: "IFR_ERR_TIMEOUT",
             5: "IFR_ERR_UNSUPPORTED"}
TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 1, 8, 12, 13, 14
MAX_VERIFY_COLS = 8

# every symbol the header declares, with (restype, argtypes)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f = ctypes.c_float
SIGNATURES = {
    "ifr_last_error": (ctypes.c_char_p, []),
    "ifr_version": (_i, []),
    "ifr_ctx_create": (_i, [_i, ctypes.POINTER(_vp)]),
    "ifr_ctx_destroy": (_i, [_vp]),
    "ifr_ctx_set_stream": (_i, [_vp, _vp]),
    "ifr_ctx_get_stream": (_i, [_vp, ctypes.POINTER(_vp)]),
    "ifr_ctx_reserve_accept": (_i, [_vp, _i, _i, _i]),
    "ifr_sync": (_i, [_vp]),
    "ifr_weights_upload": (_i, [_vp, _i, _vp, _i64, _i64, ctypes.POINTER(_vp)]),
    "ifr_weights_from_device": (_i, [_vp, _i, _vp, _i64, _i64, ctypes.POINTER(_vp)]),
    "ifr_tensor_free": (_i, [_vp]),
    "ifr_tensor_info": (_i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                             ctypes.POINTER(_i64)]),
    "ifr_dequant": (_i, [_vp, _vp, _vp]),
    "ifr_qgemm": (_i, [_vp, _vp, _vp, _i, _vp]),
    "ifr_ctx_set_dense_min_cols": (_i, [_vp, _i]),
    "ifr_ctx_set_prefill_dense": (_i, [_vp, _i]),
    "ifr_ctx_set_fused_layers": (_i, [_vp, _i]),
    "ifr_test_fused_timeout": (_i, [_vp]),
    "ifr_ctx_set_dense_f16_weights": (_i, [_vp, _i]),
    "ifr_ctx_set_kv_bf16": (_i, [_vp, _i]),
    "ifr_tensor_prepare_dense": (_i, [_vp, _vp]),
    "ifr_state_read_request": (_i, [_vp, _i, _vp, _i, _vp, _vp]),
    "ifr_prefill_batch": (_i, [_vp, _vp, _i, _vp]),
    "ifr_state_create_batch": (_i, [_vp, _i, _i, ctypes.POINTER(_vp)]),
    "ifr_qgemm_dense": (_i, [_vp, _vp, _vp, _i, _vp]),
    "ifr_qgemm_rmsnorm": (_i, [_vp, _vp, _vp, _i, _vp, _f, _vp]),
    "ifr_ctx_reserve_dense": (_i, [_vp, _vp, _i]),
    "ifr_quantize": (_i, [_i, _vp, _i64, _i64, _vp]),
    "ifr_accept": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp, _vp, _vp]),
    "ifr_ctx_set_activation": (_i, [_vp, _i]),
    "ifr_accept_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp, _vp, _vp]),
    "ifr_accept_filtered": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _f, _f, _vp, _vp, _vp]),
    "ifr_accept_greedy": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "ifr_sample": (_i, [_vp, _vp, _i, _i, _f, _i, _f, _f, _vp, _vp]),
    "ifr_draft_mtp": (_i, [_vp, _i, _vp]),
    "ifr_verify_step": (_i, [_vp, _i, _vp, _vp]),
    "ifr_rollback": (_i, [_vp, _vp, _vp]),
    "ifr_apply_penalties": (_i, [_vp, _vp, _i, _i, _vp, _i, _f, _f]),
    "ifr_model_load_gguf": (_i, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "ifr_model_load_gguf_tp": (_i, [_vp, ctypes.c_char_p, _vp, ctypes.POINTER(_vp)]),
    "ifr_comm_available": (_i, []),
    "ifr_spec_step_draft": (_i, [_vp, _vp, _i]),
    "ifr_spec_graph_draft": (_i, [_vp, _vp, _i, _i]),
    "ifr_model_get_shard": (_i, [_vp, _vp]),
    "ifr_comm_unique_id": (_i, [_vp]),
    "ifr_comm_create": (_i, [_vp, _i, _i, _vp, ctypes.POINTER(_vp)]),
    "ifr_comm_destroy": (_i, [_vp]),
    "ifr_model_free": (_i, [_vp]),
    "ifr_model_get_info": (_i, [_vp, _vp]),
    "ifr_state_create": (_i, [_vp, _i, ctypes.POINTER(_vp)]),
    "ifr_state_free": (_i, [_vp]),
    "ifr_state_reset": (_i, [_vp]),
    "ifr_prefill": (_i, [_vp, _vp, _i, _vp]),
    "ifr_spec_step": (_i, [_vp, _i, _vp]),
    "ifr_spec_graph": (_i, [_vp, _i, _i]),
    "ifr_spec_graph_launch": (_i, [_vp]),
    "ifr_state_profile": (_i, [_vp, _i]),
    "ifr_state_profile_read": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "ifr_state_fused_trace": (_i, [_vp, _i, _vp, _vp, _vp]),
    "ifr_gemv_pass": (_i, [_vp, _i]),
    "ifr_state_read": (_i, [_vp, _vp, _i, _vp, _vp]),
    "ifr_state_last_verify": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "q4_k_gemv": (None, [_vp, _vp, _vp, _vp, _i, _i]),
    "q5_k_gemv": (None, [_vp, _vp, _vp, _vp, _i, _i]),
    "q6_k_gemv": (None, [_vp, _vp, _vp, _vp, _i, _i]),
    "q8_0_gemv": (None, [_vp, _vp, _vp, _i, _i]),
}

_lib = None


class IfrError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


def load(path=None):
    """Load the shared library (building it first if absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        from . import build as _build
        _build.build()
    L = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc):
    if rc != IFR_OK:
        raise IfrError(rc, load().ifr_last_error().decode())
    return rc
