"""ctypes bindings of libfreeml_cuda.so (the C ABI in include/freeml_cuda.h).

The library is the only compute path: if it is missing this module raises --
there is no CPU fallback.  Every call's status is checked; a non-zero status
raises FmlError with the library's message.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfreeml_cuda.so")

FML_OK = 0
STATUS_NAMES = {1: "FML_ERR_INVALID", 2: "FML_ERR_CUDA", 3: "FML_ERR_NOMEM", 4: "FML_ERR_UNSUPPORTED",
                5: "FML_ERR_STATE"}

FML_MATH_FP32, FML_MATH_TF32X3, FML_MATH_TF32 = 0, 1, 2
FML_WEIGHTS_FP32, FML_WEIGHTS_BF16 = 0, 1
FML_LM_NCLASS = 10
PROFILE_CLASSES = ["embed", "layernorm", "qkv", "attention", "proj", "fc", "mlp", "lm_head", "finalize",
                   "allreduce"]


class FmlError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class LMConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_uint32), ("context", ctypes.c_uint32), ("d_model", ctypes.c_uint32),
                ("n_head", ctypes.c_uint32), ("n_layer", ctypes.c_uint32), ("max_batch", ctypes.c_uint32)]


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_F = ctypes.c_float
_I = ctypes.c_int

# name -> (restype, argtypes); the status-returning functions are checked.
SIGNATURES = {
    "fml_last_error": (ctypes.c_char_p, []),
    "fml_version": (ctypes.c_char_p, []),
    "fml_device_check": (_I, [_P, _P, _P]),
    "fml_kernel_launch_count": (_U64, []),
    "fml_device_error_count": (_I, [_P]),
    "fml_device_alloc": (_I, [ctypes.POINTER(_P), ctypes.c_size_t]),
    "fml_device_free": (_I, [_P]),
    "fml_memcpy_to_device": (_I, [_P, _P, ctypes.c_size_t]),
    "fml_memcpy_to_host": (_I, [_P, _P, ctypes.c_size_t]),
    "fml_synchronize": (_I, []),
    "fml_gather_rows": (_I, [_P, _P, _P, _U32, _U32, _U32, _P]),
    "fml_add": (_I, [_P, _P, _P, _U64, _P]),
    "fml_broadcast_add": (_I, [_P, _P, _P, _U64, _U32, _P]),
    "fml_mul_elementwise": (_I, [_P, _P, _P, _U64, _P]),
    "fml_scale": (_I, [_P, _P, _F, _P, _U64, _P]),
    "fml_scale_add": (_I, [_P, _P, _P, _P, _U64, _P]),
    "fml_fill": (_I, [_P, _F, _P, _U64, _P]),
    "fml_copy": (_I, [_P, _P, _U64, _P]),
    "fml_layernorm": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _F, _P]),
    "fml_gelu": (_I, [_P, _P, _U64, _P]),
    "fml_softmax": (_I, [_P, _P, _U32, _U32, _P]),
    "fml_split_qkv": (_I, [_P, _P, _P, _P, _U32, _U32, _P]),
    "fml_matmul": (_I, [_P, _P, _P, _U32, _U32, _U32, _I, _P]),
    "fml_matmul_strided": (_I, [_P, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _I, _U32, _U64, _U64, _U64, _P]),
    "fml_attention_workspace_bytes": (ctypes.c_size_t, [_U32, _U32, _U32, _U32]),
    "fml_attention_decode": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _F, _P, ctypes.c_size_t, _P]),
    "fml_attention_decode_noalloc": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _F, _P]),
    "fml_attention_prefill": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _I, _P]),
    "fml_set_math_mode": (_I, [_I]),
    "fml_get_math_mode": (_I, []),
    "fml_lm_create": (_I, [ctypes.POINTER(LMConfig), _I, ctypes.POINTER(_P)]),
    "fml_lm_destroy": (_I, [_P]),
    "fml_lm_bind_weights": (_I, [_P, _P, _P]),
    "fml_lm_bind_packed": (_I, [_P, _P, _I, _P]),
    "fml_lm_param_count": (_U64, [ctypes.POINTER(LMConfig)]),
    "fml_lm_get_config": (_I, [_P, ctypes.POINTER(LMConfig)]),
    "fml_matmul_left": (_I, [_P, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _U32, _U64, _U64, _U64, _P]),
    "fml_merge_qkv": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _P]),
    "fml_gelu_derivative": (_I, [_P, _P, _U64, _P]),
    "fml_softmax_backward": (_I, [_P, _P, _P, _U32, _U32, _P]),
    "fml_scatter_add_rows": (_I, [_P, _P, _P, _U32, _U32, _U32, _U32, _U32, _P]),
    "fml_layernorm_backward": (_I, [_P, _P, _P, _P, _P, _P, _P, _U32, _U32, ctypes.c_float, _P, _P]),
    "fml_adamw_update": (_I, [_P, _P, _P, _P, _U64] + [ctypes.c_float] * 7 + [_P]),
    "fml_xent_with_logits": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _I, _P, _P]),
    "fml_capture_begin": (_I, [ctypes.POINTER(_P)]),
    "fml_capture_end": (_I, [_P, ctypes.POINTER(_P)]),
    "fml_graph_launch": (_I, [_P, _P]),
    "fml_graph_destroy": (_I, [_P]),
    "fml_checkpoint_config": (_I, [ctypes.c_char_p, ctypes.POINTER(LMConfig)]),
    "fml_checkpoint_pack": (_I, [ctypes.c_char_p, _P, _U64]),
    "fml_lm_load_checkpoint": (_I, [_P, ctypes.c_char_p, _P]),
    "fml_lm_prefill": (_I, [_P, _P, _U32, _U32, _P]),
    "fml_lm_step": (_I, [_P, _P, _P, _P]),
    "fml_lm_steps": (_I, [_P, _U32, _P]),
    "fml_lm_set_weight_format": (_I, [_P, _I]),
    "fml_lm_step_host": (_I, [_P, _P, _P, _P]),
    "fml_lm_generate_host": (_I, [_P, _U32, _P, _P, _P]),
    "fml_lm_set_graph": (_I, [_P, _I]),
    "fml_lm_set_prefill_math": (_I, [_P, _I]),
    "fml_lm_set_stamps": (_I, [_P, _P, _U32, ctypes.POINTER(_U32)]),
    "fml_lm_stamp_classes": (_I, [_P, _P, _U32, ctypes.POINTER(_U32)]),
    "fml_nccl_unique_id": (_I, [_P]),
    "fml_lm_set_tensor_parallel": (_I, [_P, _I, _I, _P]),
    "fml_lm_tp_ipc_handles": (_I, [_P, _P]),
    "fml_lm_tp_connect": (_I, [_P, _P]),
    "fml_lm_tp_error_count": (_I, [_P]),
    "fml_tp_flag_check": (_I, [_U32, _U32, _U32, _U32, ctypes.POINTER(_I)]),
    "fml_lm_pending": (_I, [_P, _P, _P]),
    "fml_lm_get_position": (_I, [_P, _U32, ctypes.POINTER(_U32)]),
    "fml_lm_rewind": (_I, [_P, _U32, _P, _I, _P]),
    "fml_lm_step_bytes": (_U64, [_P]),
    "fml_lm_attention_bytes": (_U64, [_P]),
    "fml_lm_set_profiling": (_I, [_P, _I]),
    "fml_lm_get_profile": (_I, [_P, _P, _P, _I]),
}
CHECKED_RESTYPE = _I
UNCHECKED = {"fml_get_math_mode"}

_lib = None


def load(path: str | None = None):
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    # torch first: the library links NCCL, and torch's own NCCL build must be
    # the one the process resolves (loading ours first binds an older system
    # copy that torch's CUDA library cannot use)
    import torch  # noqa: F401
    if not os.path.exists(path):
        raise FmlError(2, "load", f"{path} not found -- build it with `python -m freeml_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args):
    """Call a status-returning entry point and raise on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if SIGNATURES[name][0] is CHECKED_RESTYPE and name not in UNCHECKED and rc != FML_OK:
        raise FmlError(rc, name, lib.fml_last_error().decode(errors="replace"))
    return rc


def launch_count() -> int:
    return int(load().fml_kernel_launch_count())
