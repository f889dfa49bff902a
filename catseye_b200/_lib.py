"""Loads libcatsgpu.so (built in-tree by catseye_b200/csrc/Makefile) and
declares the C ABI of include/catsgpu.h for ctypes.

There is no CPU fallback: if the library is missing or no B200 is visible,
every entry point raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcatsgpu.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "catsgpu.h")

_vp, _fp, _ip = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int)
_i, _u64, _f, _ch, _sz = C.c_int, C.c_ulonglong, C.c_float, C.c_char, C.c_size_t


class LlmConfigC(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden", "n_layers", "n_heads", "n_kv_heads", "vocab",
                                       "seq_len", "wtype", "tp_rank", "tp_size")]


# name -> (restype, argtypes)
SIGNATURES = {
    "cats_gpu_init": (_i, [_i]),
    "cats_gpu_term": (None, []),
    "cats_gpu_last_error": (_i, []),
    "cats_gpu_clear_error": (None, []),
    "cats_gpu_error_string": (C.c_char_p, [_i]),
    "cats_gpu_device_error": (_i, []),
    "cats_gpu_register_weight": (_i, [_vp, _i, _i, _i]),
    "cats_gpu_unregister_weight": (None, [_vp]),
    "cats_gpu_weight_device_bytes": (_sz, [_vp]),
    "cats_gpu_matmul_f32": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_matmul_q4_0_q8": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_matmul_q8_0_q8": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_quantize_q8": (None, [_vp, _vp, _i]),
    "cats_gpu_dequantize_q4_0": (_vp, [_vp, _vp, _i, _i]),
    "cats_gpu_dequantize_q8_0": (_vp, [_vp, _vp, _i, _i]),
    "cats_gpu_matmul_q4_0_f32": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_matmul_q8_0_f32": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_matmul_q3_K_q8_K": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_matmul_q6_K_q8_K": (None, [_vp, _vp, _vp, _i, _i]),
    "cats_gpu_quantize_q8_K": (None, [_vp, _vp, _i]),
    "cats_gpu_dequantize_q3_K": (_vp, [_vp, _vp, _i, _i]),
    "cats_gpu_dequantize_q6_K": (_vp, [_vp, _vp, _i, _i]),
    "cats_gpu_matvec_dev": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cats_gpu_quantize_q8_dev": (_i, [_vp, _vp, _i, _i, _vp]),
    "cats_gpu_qgemm_dev": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cats_gpu_qgemm": (_i, [_vp, _vp, _vp, _i]),
    "cats_gpu_qgemm_plan": (_i, [_vp, _i, _vp]),
    "cats_gpu_qgemm_trace": (_i, [_vp, _vp, _vp, _i, _vp, _i]),
    "cats_gpu_dequantize_dev": (_i, [_i, _vp, _vp, _i, _i, _vp]),
    "cats_gpu_llm_create": (_vp, [C.POINTER(LlmConfigC)]),
    "cats_gpu_llm_destroy": (None, [_vp]),
    "cats_gpu_llm_set_weights": (_i, [_vp] + [_vp] * 12),
    "cats_gpu_llm_init_random": (_i, [_vp, _u64, _f]),
    "cats_gpu_llm_file_config": (_i, [C.c_char_p, C.POINTER(LlmConfigC)]),
    "cats_gpu_llm_load": (_vp, [C.c_char_p, _i, _i, _i]),
    "cats_gpu_llama2_transformer": (_vp, [_i, _i, _vp, _vp]),
    "cats_gpu_llm_generate": (_i, [_vp, _i, _i, _i, _vp]),
    "cats_gpu_llm_enqueue": (_i, [_vp, _i]),
    "cats_gpu_llm_batch_reserve": (_i, [_vp, _i, _i]),
    "cats_gpu_llm_forward_batch": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "cats_gpu_llm_generate_batch": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "cats_gpu_llm_batch_set": (_i, [_vp, _vp, _vp, _vp, _i]),
    "cats_gpu_llm_batch_enqueue": (_i, [_vp]),
    "cats_gpu_llm_batch_enqueue_decode": (_i, [_vp, _i]),
    "cats_gpu_llm_time_product": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "cats_gpu_llm_set_engine": (_i, [_vp, _i]),
    "cats_gpu_tp_unique_id_bytes": (_sz, []),
    "cats_gpu_tp_unique_id": (_i, [_vp, _sz]),
    "cats_gpu_llm_tp_connect": (_i, [_vp, _vp]),
    "cats_gpu_llm_tp_loopback": (_i, [_vp]),
    "cats_gpu_llm_trace_step": (_i, [_vp, _i, _i, _vp, _i, C.POINTER(C.c_int)]),
    "cats_gpu_llm_set_position": (_i, [_vp, _i, _i]),
    "cats_gpu_llm_synchronize": (_i, [_vp]),
    "cats_gpu_llm_stream": (_vp, [_vp]),
    "cats_gpu_llm_logits": (_i, [_vp, _vp]),
    "cats_gpu_llm_next_token": (_i, [_vp]),
    "cats_gpu_llm_weight_bytes": (_sz, [_vp]),
    "cats_gpu_llm_time_matvec": (_i, [_vp, _i, _i, C.POINTER(C.c_float), C.POINTER(C.c_double)]),
    "cats_gpu_synth_tensor": (_i, [_vp, _i, _i, _i, _u64, _i, _f, _f]),
    "cats_sgemm": (None, [_ch, _ch, _i, _i, _i, _f, _vp, _vp, _f, _vp]),
    "cats_gemm_rnn": (None, [_i, _i, _i, _f, _vp, _vp, _f, _vp]),
    "cats_gemm_rnt": (None, [_i, _i, _i, _f, _vp, _vp, _f, _vp]),
    "cats_gemm_rtn": (None, [_i, _i, _i, _f, _vp, _vp, _f, _vp]),
    "cats_sgemm_dev": (_i, [_ch, _ch, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i, _vp]),
    "cats_sgemm_dev_noalloc": (_i, [_ch, _ch, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i, _vp]),
    "cats_im2col": (None, [_vp] + [_i] * 9 + [_vp]),
    "cats_im2col_dev": (_i, [_vp] + [_i] * 9 + [_vp, _vp]),
    "cats_conv2d_forward": (None, [_vp, _vp, _vp] + [_i] * 8),
    "cats_conv2d_forward_dev": (_i, [_vp, _vp, _vp] + [_i] * 8 + [_vp]),
    "cats_linear_forward": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "cats_linear_forward_dev": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "cats_ocl_setup": (C.c_ulong, [_i]),
    "cats_ocl_alloc": (_vp, [_sz]),
    "cats_ocl_free": (None, [_vp]),
    "cats_ocl_write": (_i, [_vp, _sz, _sz, _vp]),
    "cats_ocl_read": (_i, [_vp, _sz, _sz, _vp]),
    "cats_ocl_run": (_i, [C.c_char_p, _vp, _vp, _vp]),
    "cats_col2im": (None, [_vp] + [_i] * 9 + [_vp]),
    "cats_col2im_dev": (_i, [_vp] + [_i] * 9 + [_vp, _vp]),
    "cats_conv2d_backward": (None, [_vp, _vp, _vp] + [_i] * 8),
    "cats_conv2d_backward_dev": (_i, [_vp, _vp, _vp] + [_i] * 8 + [_vp]),
    "cats_conv2d_update": (None, [_vp, _vp, _vp] + [_i] * 8),
    "cats_conv2d_update_dev": (_i, [_vp, _vp, _vp] + [_i] * 8 + [_vp]),
    "cats_linear_backward": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "cats_linear_backward_dev": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "cats_linear_update": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _f]),
    "cats_linear_update_dev": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp]),
}

_LIB = None


class CatsGpuError(RuntimeError):
    pass


def load(path=None):
    """Load and declare the library once (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = path or os.environ.get("CATS_GPU_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise CatsGpuError(f"{path} is missing: build it with `make -C catseye_b200/csrc` "
                           "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(rc, what="catsgpu"):
    """Raise on a non-zero status (or a sticky error after a void call)."""
    lib = load()
    if rc is None:
        rc = lib.cats_gpu_last_error()
        if rc:
            lib.cats_gpu_clear_error()
    if rc:
        lib.cats_gpu_clear_error()
        raise CatsGpuError(f"{what}: {lib.cats_gpu_error_string(rc).decode()} ({rc})")
    return rc


def call_void(fn, *args, what=None):
    """Call a void drop-in and raise if it recorded an error (the sticky
    status is cleared first, so only this call's outcome is reported)."""
    load().cats_gpu_clear_error()
    fn(*args)
    return check(None, what or fn.__name__)


def init(device=-1):
    lib = load()
    check(lib.cats_gpu_init(device), "cats_gpu_init")
    return lib
