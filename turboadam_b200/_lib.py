"""ctypes binding of libturboadam_b200.so (include/turboadam_b200.h).

The library is the only compute path: every entry point below launches the
sm_100a kernels. There is no CPU fallback; importing works without a GPU
(so the optimizer can be constructed and inspected), but any call that would
launch a kernel raises ``TurboAdamBackendError`` when the library or a CUDA
device is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libturboadam_b200.so")

TA_OK = 0
TA_F32, TA_BF16 = 0, 1
TA_M_COSTATE = 1 << 0
TA_V_ONEQ = 1 << 1
TA_M_HAS_STATE = 1 << 2
TA_NO_PARAM = 1 << 3
TA_M_SPANNING = 1 << 4
TA_EXACT_PARAM = 1 << 5
TA_M_EF = 1 << 6
TA_M_EF_STATE = 1 << 7
TA_PHASE_PASS1, TA_PHASE_PASS2, TA_PHASE_SEL1, TA_PHASE_SEL2, TA_PHASE_LABELS = range(5)
TA_SHARD_ALIGN_BLOCKS = 4096
TA_STATUS_NONFINITE_GRAD = 1 << 0
TA_STATUS_WAIT_TIMEOUT = 1 << 1
TA_STATUS_BIAS_TABLE_SHORT = 1 << 2

STATUS_NAMES = {
    1: "TA_ERR_INVALID",
    2: "TA_ERR_ALIGN",
    3: "TA_ERR_UNSUPPORTED",
    4: "TA_ERR_WORKSPACE",
    5: "TA_ERR_CUDA",
}

# Every symbol declared in include/turboadam_b200.h.
EXPORTED = (
    "ta_abi_version",
    "ta_last_error",
    "ta_state_padded_blocks",
    "ta_workspace_size",
    "ta_step",
    "ta_step_profiled",
    "ta_read_status",
    "ta_v_update",
    "ta_v_update_noalloc",
    "ta_v_update_noalloc_status",
    "ta_v_init",
    "ta_v_decode",
    "ta_costate_decode",
    "ta_costate_encode",
    "ta_thresholds",
    "ta_aux_workspace_size",
    "ta_exchange_layout",
    "ta_step_phase",
    "ta_plan_prepare",
    "ta_step_prepared",
    "ta_selftest_fast_math",
    "ta_selftest_wait_timeout",
)


class TurboAdamBackendError(RuntimeError):
    pass


class TaTensor(ctypes.Structure):
    _fields_ = [
        ("param_dev", ctypes.c_void_p),
        ("grad_dev", ctypes.c_void_p),
        ("numel", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("group", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("tensor_id", ctypes.c_uint32),
        ("step", ctypes.c_uint32),
        ("reserved0", ctypes.c_int32),
        ("v_idx_dev", ctypes.c_void_p),
        ("v_hdr_dev", ctypes.c_void_p),
        ("exp_avg_sq_dev", ctypes.c_void_p),
        ("m_labels_dev", ctypes.c_void_p),
        ("m_signs_dev", ctypes.c_void_p),
        ("m_norms_dev", ctypes.c_void_p),
        ("m_amp_dev", ctypes.c_void_p),
        ("m_alpha_dev", ctypes.c_void_p),
        ("exp_avg_dev", ctypes.c_void_p),
        ("sr_uniforms_dev", ctypes.c_void_p),
        ("alpha_inject_dev", ctypes.c_void_p),
        ("m_out_dev", ctypes.c_void_p),
        ("v_out_dev", ctypes.c_void_p),
        ("block_offset", ctypes.c_int64),
        ("global_blocks", ctypes.c_int64),
        ("exch_chunk_off", ctypes.c_int64),
        ("exch_hist_off", ctypes.c_int64),
        ("m_ef_dev", ctypes.c_void_p),
    ]


class TaGroup(ctypes.Structure):
    _fields_ = [
        ("lr", ctypes.c_double),
        ("beta1", ctypes.c_double),
        ("beta2", ctypes.c_double),
        ("eps", ctypes.c_double),
        ("weight_decay", ctypes.c_double),
        ("null_pct", ctypes.c_double),
        ("amp_pct", ctypes.c_double),
        ("bc1", ctypes.c_float),
        ("bc2", ctypes.c_float),
        ("block_size", ctypes.c_int32),
        ("v_bits", ctypes.c_int32),
    ]


class TaDynamic(ctypes.Structure):
    _fields_ = [
        ("steps_dev", ctypes.c_void_p),
        ("bias_table_dev", ctypes.c_void_p),
        ("table_steps", ctypes.c_int64),
        ("lr_dev", ctypes.c_void_p),
        ("grad_scale_dev", ctypes.c_void_p),
        ("found_inf_dev", ctypes.c_void_p),
    ]


# numpy views of the same layouts, for vectorised per-step updates
TENSOR_DTYPE = np.dtype(
    {
        "names": [f[0] for f in TaTensor._fields_],
        "formats": [
            {ctypes.c_void_p: np.uint64, ctypes.c_int64: np.int64, ctypes.c_int32: np.int32,
             ctypes.c_uint32: np.uint32}[f[1]]
            for f in TaTensor._fields_
        ],
        "offsets": [getattr(TaTensor, f[0]).offset for f in TaTensor._fields_],
        "itemsize": ctypes.sizeof(TaTensor),
    }
)
GROUP_DTYPE = np.dtype(
    {
        "names": [f[0] for f in TaGroup._fields_],
        "formats": [
            {ctypes.c_double: np.float64, ctypes.c_float: np.float32, ctypes.c_int32: np.int32}[f[1]]
            for f in TaGroup._fields_
        ],
        "offsets": [getattr(TaGroup, f[0]).offset for f in TaGroup._fields_],
        "itemsize": ctypes.sizeof(TaGroup),
    }
)

_P = ctypes.c_void_p
_SIG = {
    "ta_abi_version": (ctypes.c_int, []),
    "ta_last_error": (ctypes.c_char_p, []),
    "ta_state_padded_blocks": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int32]),
    "ta_workspace_size": (ctypes.c_size_t, [_P, ctypes.c_int32]),
    "ta_step": (ctypes.c_int, [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_uint64, _P,
                               ctypes.c_size_t, _P]),
    "ta_step_profiled": (ctypes.c_int, [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_uint64,
                                        _P, ctypes.c_size_t, _P, _P]),
    "ta_read_status": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32), _P]),
    "ta_v_update": (ctypes.c_int, [_P, _P, _P, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_int32, ctypes.c_double, _P, ctypes.c_uint64,
                                   ctypes.c_uint32, ctypes.c_uint32, _P, _P, _P, _P,
                                   ctypes.c_size_t, _P]),
    "ta_v_update_noalloc": (ctypes.c_int, [_P, _P, _P, ctypes.c_int32, ctypes.c_int64,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_double, _P,
                                           ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                           _P, _P, _P, _P]),
    "ta_v_update_noalloc_status": (ctypes.c_int, [ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_uint32), _P]),
    "ta_v_init": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, _P, _P, _P]),
    "ta_v_decode": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _P,
                                   _P]),
    "ta_costate_decode": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_int32, _P, _P]),
    "ta_costate_encode": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P]),
    "ta_thresholds": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_double, ctypes.c_double, _P,
                                     _P, _P, ctypes.c_size_t, _P]),
    "ta_aux_workspace_size": (ctypes.c_size_t, [ctypes.c_int64]),
    "ta_exchange_layout": (ctypes.c_int, [_P, ctypes.c_int32, _P, _P,
                                          ctypes.POINTER(ctypes.c_size_t),
                                          ctypes.POINTER(ctypes.c_size_t)]),
    "ta_step_phase": (ctypes.c_int, [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_uint64, _P,
                                     ctypes.c_size_t, _P, ctypes.c_size_t, ctypes.c_size_t,
                                     ctypes.c_int32, _P]),
    "ta_plan_prepare": (ctypes.c_int, [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_uint64, _P,
                                       ctypes.c_size_t, _P]),
    "ta_step_prepared": (ctypes.c_int, [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_uint64,
                                        _P, ctypes.c_size_t, ctypes.POINTER(TaDynamic), _P]),
    "ta_selftest_fast_math": (ctypes.c_int, [_P, _P]),
    "ta_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _P, _P, _P]),
}

_lib = None


def load():
    """Load the library (no CUDA needed to load; kernels need a GPU)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise TurboAdamBackendError(
            f"{LIB_PATH} is missing: build it with `python -m turboadam_b200.csrc.build` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIG.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int, what: str):
    if code != TA_OK:
        msg = load().ta_last_error().decode(errors="replace")
        raise TurboAdamBackendError(f"{what} failed: {STATUS_NAMES.get(code, code)}: {msg}")


def require_cuda(t) -> None:
    import torch

    if not torch.cuda.is_available():
        raise TurboAdamBackendError(
            "turboadam_b200 runs only on CUDA (sm_100a) devices; no CUDA device is visible")
    if not (hasattr(t, "is_cuda") and t.is_cuda):
        raise TurboAdamBackendError(
            "turboadam_b200 updates CUDA tensors only (got a tensor on "
            f"{getattr(t, 'device', '?')}); there is no CPU fallback")


def stream_ptr(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
