"""ctypes bindings of libgotensor_cuda.so (include/gt_cuda.h) and
libgotensor_host.so (include/gt_host.h).

Loading fails loudly when the libraries are missing: there is no CPU
fallback. Build them with ``python go-tensor_b200/build.py`` (or
``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIBDIR = os.path.join(os.path.dirname(HERE), "lib")
CUDA_LIB_PATH = os.path.join(LIBDIR, "libgotensor_cuda.so")
HOST_LIB_PATH = os.path.join(LIBDIR, "libgotensor_host.so")

MAX_DIMS = 8
FLOAT32, FLOAT64 = 0, 1
ACT_NONE, ACT_RELU, ACT_TANH, ACT_SIGMOID = 0, 1, 2, 3


class GtView(ctypes.Structure):
    _fields_ = [("ndim", ctypes.c_int32), ("_pad", ctypes.c_int32), ("offset", ctypes.c_int64),
                ("shape", ctypes.c_int64 * MAX_DIMS), ("strides", ctypes.c_int64 * MAX_DIMS)]


class GtGeom(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int64) for f in ("N", "C", "H", "W", "KH", "KW", "OH", "OW", "stride", "pad")]


class SgdCfg(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_double), ("momentum", ctypes.c_double), ("weight_decay", ctypes.c_double)]


class AdamCfg(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_double), ("beta1", ctypes.c_double), ("beta2", ctypes.c_double),
                ("eps", ctypes.c_double), ("weight_decay", ctypes.c_double)]


class Layer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("_pad", ctypes.c_int32), ("in_", ctypes.c_int64),
                ("out", ctypes.c_int64), ("kernel", ctypes.c_int64), ("stride", ctypes.c_int64),
                ("padding", ctypes.c_int64), ("p", ctypes.c_double)]


class GTError(RuntimeError):
    """An error returned by the native library (the Go backend panics with it)."""


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_D = ctypes.c_double

# name: (restype, argtypes); restype "err" = char* error convention.
CUDA_API = {
    "gt_init": ("err", [_INT, ctypes.POINTER(_P)]),
    "gt_destroy": ("err", [_P]),
    "gt_free_error": (None, [_P]),
    "gt_device_name": (ctypes.c_char_p, [_P]),
    "gt_device_index": (_INT, [_P]),
    "gt_sm_count": (_INT, [_P]),
    "gt_stream": (_P, [_P]),
    "gt_sync": ("err", [_P]),
    "gt_alloc": ("err", [_P, ctypes.c_size_t, ctypes.POINTER(_P)]),
    "gt_release": ("err", [_P, _P]),
    "gt_zero": ("err", [_P, _P, ctypes.c_size_t]),
    "gt_pool_usage": ("err", [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "gt_upload": ("err", [_P, _P, _P, ctypes.c_size_t]),
    "gt_download": ("err", [_P, _P, _P, ctypes.c_size_t]),
    "gt_upload_async": ("err", [_P, _P, _P, ctypes.c_size_t]),
    "gt_download_async": ("err", [_P, _P, _P, ctypes.c_size_t]),
    "gt_write": ("err", [_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t]),
    "gt_cast": ("err", [_P, _P, _INT, _P, _INT, _I64]),
    "gt_unary": ("err", [_P, _INT, _INT, _D, _P, _P, _I64]),
    "gt_binary": ("err", [_P, _INT, _INT, _P, ctypes.POINTER(GtView), _P, ctypes.POINTER(GtView), _P]),
    "gt_copy": ("err", [_P, _INT, _P, ctypes.POINTER(GtView), _P]),
    "gt_reduce": ("err", [_P, _INT, _INT, _P, _P, _I64, _I64, _I64]),
    "gt_matmul": ("err", [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _INT, _INT]),
    "gt_im2col": ("err", [_P, _INT, _P, _P, ctypes.POINTER(GtGeom)]),
    "gt_col2im": ("err", [_P, _INT, _P, _P, ctypes.POINTER(GtGeom)]),
    "gt_maxpool_fwd": ("err", [_P, _INT, _P, _P, ctypes.POINTER(GtGeom)]),
    "gt_maxpool_bwd": ("err", [_P, _INT, _P, _P, _P, ctypes.POINTER(GtGeom)]),
    "gt_linear_fwd": ("err", [_P, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _INT]),
    "gt_linear_bwd_data": ("err", [_P, _INT, _P, _P, _P, _INT, _P, _I64, _I64, _I64]),
    "gt_relu_bits": ("err", [_P, _INT, _P, _P, _I64, _I64]),
    "gt_mse_fwd_bwd": ("err", [_P, _INT, _P, _P, _I64, _P, _P]),
    "gt_bce_fwd_bwd": ("err", [_P, _INT, _P, _P, _I64, _P, _P]),
    "gt_linear_fwd_bits": ("err", [_P, _INT, _P, _P, _P, _P, _P, _I64, _I64, _I64]),
    "gt_linear_bwd_data_bits": ("err", [_P, _INT, _P, _P, _P, _P, _I64, _I64, _I64]),
    "gt_linear_bwd_data_db": ("err", [_P, _INT, _P, _P, _P, _INT, _P, _P, _I64, _I64, _I64]),
    "gt_linear_bwd_data_bits_db": ("err", [_P, _INT, _P, _P, _P, _P, _P, _I64, _I64, _I64]),
    "gt_linear_bwd_weight": ("err", [_P, _INT, _P, _P, _P, _P, _I64, _I64, _I64]),
    "gt_act_bwd": ("err", [_P, _INT, _INT, _P, _P, _P, _I64]),
    "gt_bias_act": ("err", [_P, _INT, _P, _P, _I64, _I64, _I64, _INT]),
    "gt_conv_fwd": ("err", [_P, _INT, _P, _P, _P, _P, ctypes.POINTER(GtGeom), _I64, _INT]),
    "gt_conv_bwd_data": ("err", [_P, _INT, _P, _P, _P, ctypes.POINTER(GtGeom), _I64]),
    "gt_conv_bwd_weight": ("err", [_P, _INT, _P, _P, _P, _P, ctypes.POINTER(GtGeom), _I64]),
    "gt_linear_bwd_weight_rows": ("err", [_P, _INT, _P, _P, _P, _I64, _I64, _I64, _I64, _I64]),
    "gt_conv_fwd_cols": ("err", [_P, _INT, _P, _P, _P, _P, _P, ctypes.POINTER(GtGeom), _I64, _INT]),
    "gt_conv_bwd": ("err", [_P, _INT, _P, _P, _P, _P, _P, _P, ctypes.POINTER(GtGeom), _I64]),
    "gt_maxpool_fwd_idx": ("err", [_P, _INT, _P, _P, _P, ctypes.POINTER(GtGeom)]),
    "gt_maxpool_bwd_idx": ("err", [_P, _INT, _P, _P, _P, _INT, _P, ctypes.POINTER(GtGeom)]),
    "gt_conv_fwd_pool": ("err", [_P, _INT, _P, _P, _P, _P, _P, ctypes.POINTER(GtGeom), ctypes.POINTER(GtGeom),
                                 _I64, _INT]),
    "gt_conv_bwd_weight_pool": ("err", [_P, _INT, _P, _P, _P, _P, _INT, _P, _P, ctypes.POINTER(GtGeom),
                                        ctypes.POINTER(GtGeom), _I64]),
    "gt_argmax_rows": ("err", [_P, _INT, _P, _I64, _I64, _P]),
    "gt_count_equal": ("err", [_P, _P, _P, _I64, _P]),
    "gt_xent_fwd_bwd": ("err", [_P, _INT, _P, _P, _I64, _I64, _P, _P, _P]),
    "gt_xent_fwd_bwd_db": ("err", [_P, _INT, _P, _P, _I64, _I64, _P, _P, _P, _P]),
    "gt_xent_fwd_bwd_noalloc": ("err", [_P, _INT, _P, _P, _I64, _I64, _P, _P, _P]),
    "gt_sgd_step": ("err", [_P, _INT, _P, _P, _P, _I64, ctypes.POINTER(SgdCfg), _INT]),
    "gt_adam_step": ("err", [_P, _INT, _P, _P, _P, _P, _I64, ctypes.POINTER(AdamCfg), _I64]),
    "gt_adam_step_dev": ("err", [_P, _INT, _P, _P, _P, _P, _I64, ctypes.POINTER(AdamCfg), _P]),
    "gt_comm_unique_id": ("err", [ctypes.c_char_p]),
    "gt_comm_init": ("err", [_P, _INT, _INT, ctypes.c_char_p, _INT]),
    "gt_allreduce_avg": ("err", [_P, _INT, _P, _I64]),
    "gt_allreduce_avg_async": ("err", [_P, _INT, _P, _I64]),
    "gt_comm_wait": ("err", [_P]),
    "gt_comm_destroy": ("err", [_P, _INT]),
    "gt_capture_begin": ("err", [_P]),
    "gt_capture_end": ("err", [_P, ctypes.POINTER(_P)]),
    "gt_graph_launch": ("err", [_P, _P]),
    "gt_graph_free": (None, [_P]),
    "gt_mark": ("err", [_P, _INT]),
    "gt_elapsed_ms": ("err", [_P, _INT, _INT, ctypes.POINTER(ctypes.c_float)]),
    "gt_event_new": ("err", [_P, ctypes.POINTER(_P)]),
    "gt_event_free": (None, [_P]),
    "gt_event_record": ("err", [_P, _P, _INT]),
    "gt_stream_wait_event": ("err", [_P, _INT, _P]),
    "gt_upload_on": ("err", [_P, _INT, _P, _P, ctypes.c_size_t]),
    "gt_host_alloc": ("err", [ctypes.c_size_t, ctypes.POINTER(_P)]),
    "gt_host_free": (None, [_P]),
    "gt_launch_count": (_I64, []),
    "gt_gemm_timer_start": ("err", [_P, _I64]),
    "gt_gemm_timer_stop": ("err", [_P]),
    "gt_gemm_timer_count": ("err", [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "gt_gemm_timer_read": ("err", [_P, _I64, ctypes.POINTER(_I64), ctypes.POINTER(_INT), ctypes.POINTER(ctypes.c_float)]),
    "gt_set_gemm_sm_reserve": ("err", [_P, _INT]),
    "gt_debug_set_gemm_path": (None, [_INT]),
    "gt_debug_set_gemm_splits": (None, [_INT]),
    "gt_debug_set_tc_wait_limit_us": (None, [_I64]),
    "gt_debug_tc_withhold_arrive": (None, []),
    "gt_gemm_path_taken": (_INT, []),
}

HOST_API = {
    "gth_model_new": ("err", [_P, _INT, ctypes.POINTER(Layer), _INT, ctypes.POINTER(_I64), _INT,
                              ctypes.POINTER(_P)]),
    "gth_model_free": (None, [_P]),
    "gth_num_tensors": (_INT, [_P]),
    "gth_num_params": (_I64, [_P]),
    "gth_param_info": ("err", [_P, _INT, ctypes.c_char_p, _INT, ctypes.POINTER(_I64), ctypes.POINTER(_INT),
                               ctypes.POINTER(_I64)]),
    "gth_set_params": ("err", [_P, _P]),
    "gth_get_params": ("err", [_P, _P]),
    "gth_get_grads": ("err", [_P, _P]),
    "gth_params_device": (_P, [_P]),
    "gth_grads_device": (_P, [_P]),
    "gth_set_sgd": ("err", [_P, ctypes.POINTER(SgdCfg)]),
    "gth_set_adam": ("err", [_P, ctypes.POINTER(AdamCfg)]),
    "gth_input_device": (_P, [_P]),
    "gth_labels_device": (_P, [_P]),
    "gth_loss_device": (_P, [_P]),
    "gth_stage_batch": ("err", [_P, _P, _P]),
    "gth_forward_backward": ("err", [_P]),
    "gth_optimizer_step": ("err", [_P]),
    "gth_train_step": ("err", [_P]),
    "gth_enable_graph": ("err", [_P, _INT]),
    "gth_loss": ("err", [_P, ctypes.POINTER(_D)]),
    "gth_forward": ("err", [_P, _P]),
    "gth_step_launches": (_INT, [_P]),
    "gth_predict": ("err", [_P, _P]),
    "gth_save_safetensors": ("err", [_P, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p),
                                     ctypes.POINTER(ctypes.c_char_p), _INT]),
    "gth_load_safetensors": ("err", [_P, ctypes.c_char_p, _INT]),
    "gth_save_gotn": ("err", [_P, ctypes.c_char_p]),
    "gth_load_gotn": ("err", [_P, ctypes.c_char_p]),
    "gth_safetensors_read": ("err", [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), _I64,
                                     ctypes.POINTER(_I64), _INT, ctypes.POINTER(_INT), ctypes.POINTER(_I64)]),
    "gth_safetensors_metadata": ("err", [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _INT,
                                         ctypes.POINTER(_INT)]),
    "gth_count_correct": ("err", [_P, ctypes.POINTER(_I64)]),
    "gth_dp_init": ("err", [_P, _INT, _INT, ctypes.c_char_p, _INT, _I64]),
    "gth_bucket_plan": (_INT, [ctypes.POINTER(_I64), _INT, _I64, ctypes.POINTER(_I64), _INT]),
    "gth_row_chunk_plan": (_INT, [ctypes.POINTER(_I64), _INT, _I64, _I64, _I64, _INT, ctypes.POINTER(_I64), _INT,
                                  ctypes.POINTER(_I64), _INT, ctypes.POINTER(_INT)]),
}

_cuda = None
_host = None


def _bind(lib, api):
    for name, (res, args) in api.items():
        f = getattr(lib, name)
        f.restype = _P if res == "err" else res
        f.argtypes = args


def cuda_lib() -> ctypes.CDLL:
    global _cuda
    if _cuda is None:
        if not os.path.exists(CUDA_LIB_PATH):
            raise GTError(f"{CUDA_LIB_PATH} is missing: build it with `python go-tensor_b200/build.py`")
        lib = ctypes.CDLL(CUDA_LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        _bind(lib, CUDA_API)
        _cuda = lib
    return _cuda


def host_lib() -> ctypes.CDLL:
    global _host
    if _host is None:
        cuda_lib()
        if not os.path.exists(HOST_LIB_PATH):
            raise GTError(f"{HOST_LIB_PATH} is missing: build it with `python go-tensor_b200/build.py`")
        lib = ctypes.CDLL(HOST_LIB_PATH)
        _bind(lib, HOST_API)
        _host = lib
    return _host


def check(err) -> None:
    """Raises GTError for a non-NULL char* error, freeing it."""
    if err:
        msg = ctypes.string_at(err).decode(errors="replace")
        cuda_lib().gt_free_error(err)
        raise GTError(msg)
