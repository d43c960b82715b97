"""ctypes declarations of the C ABI in include/floyd_cuda.h.

The shared library is built in-tree (floyd_b200/build.py) for sm_100a.  There
is no Python or CPU implementation behind these names: if the library is
missing the import fails with an explicit error.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfloyd_cuda.so")

FMT_F32, FMT_Q8, FMT_Q4, FMT_MXFP4 = 0, 1, 2, 3
SCORE_SOFTMAX, SCORE_SIGMOID, SCORE_SQRT_SOFTPLUS = 0, 1, 2
EP_HANDLE_BYTES = 64    # FC_EP_HANDLE_BYTES
ACCEPT_GREEDY, ACCEPT_SAMPLE = 0, 1


class FcModelConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int), ("layer_count", ctypes.c_int),
        ("vocab_size", ctypes.c_int), ("head_count", ctypes.c_int),
        ("q_lora_rank", ctypes.c_int), ("kv_lora_rank", ctypes.c_int),
        ("qk_nope_dim", ctypes.c_int), ("qk_rope_dim", ctypes.c_int),
        ("value_dim", ctypes.c_int), ("expert_count", ctypes.c_int),
        ("experts_per_token", ctypes.c_int), ("moe_intermediate_size", ctypes.c_int),
        ("shared_expert_count", ctypes.c_int), ("first_dense_layer_count", ctypes.c_int),
        ("dense_intermediate_size", ctypes.c_int), ("hash_layer_count", ctypes.c_int),
        ("score_fn", ctypes.c_int), ("normalize_topk", ctypes.c_int),
        ("has_selection_bias", ctypes.c_int), ("routed_scale", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float), ("rms_norm_epsilon", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("dense_format", ctypes.c_int),
        ("expert_format", ctypes.c_int), ("mtp_layers", ctypes.c_int),
        ("embed_f32", ctypes.c_int), ("resident_bytes", ctypes.c_uint64),
    ]

    @classmethod
    def from_dict(cls, d):
        c = cls()
        for name, _ in cls._fields_:
            if name in d:
                setattr(c, name, d[name])
        return c

    def to_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class FcOptions(ctypes.Structure):
    _fields_ = [("context_size", ctypes.c_int), ("max_batch", ctypes.c_int)]


class FcBatchOptions(ctypes.Structure):
    _fields_ = [("context_size", ctypes.c_int), ("sequences", ctypes.c_int),
                ("rows_per_sequence", ctypes.c_int), ("shared_prefix", ctypes.c_int)]


class FcStats(ctypes.Structure):
    _fields_ = [
        ("command_buffers", ctypes.c_uint64), ("prefill_tokens", ctypes.c_uint64),
        ("decode_tokens", ctypes.c_uint64), ("cpu_fallbacks", ctypes.c_uint64),
        ("buffer_allocations", ctypes.c_uint64), ("resident_bytes", ctypes.c_uint64),
        ("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double),
        ("verify_calls", ctypes.c_uint64), ("proposed_tokens", ctypes.c_uint64),
        ("accepted_tokens", ctypes.c_uint64), ("graph_replays", ctypes.c_uint64),
        ("verify_ms", ctypes.c_double), ("gpu_ms", ctypes.c_double),
    ]


class FcAcceptConfig(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int), ("temperature", ctypes.c_float),
                ("seed", ctypes.c_uint64), ("counter", ctypes.c_uint64)]


class FcRuntime(ctypes.Structure):
    _fields_ = [("session", ctypes.c_void_p), ("logits", ctypes.POINTER(ctypes.c_float)),
                ("vocab_size", ctypes.c_int), ("max_context", ctypes.c_int),
                ("last_count", ctypes.c_int), ("last_start_position", ctypes.c_int),
                ("dspark_ready", ctypes.c_int)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_S = ctypes.c_size_t
_C = ctypes.c_char_p
_IP = ctypes.POINTER(ctypes.c_int)
_FP = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); every symbol include/floyd_cuda.h declares.
SIGNATURES = {
    "fc_model_create": (_I, [ctypes.POINTER(_P), ctypes.POINTER(FcModelConfig), _I, _C, _S]),
    "fc_model_create_ep": (_I, [ctypes.POINTER(_P), ctypes.POINTER(FcModelConfig), _I, _I, _I, _C, _S]),
    "fc_model_fill_synthetic": (_I, [_P, ctypes.c_uint64, _C, _S]),
    "fc_model_set_tensor": (_I, [_P, _C, _P, _S, _C, _S]),
    "fc_model_get_tensor": (_I, [_P, _C, _P, _S, _C, _S]),
    "fc_model_close": (None, [_P]),
    "fc_device_name": (_C, [_P]),
    "fc_model_info": (FcModelConfig, [_P]),
    "fc_session_create": (_I, [ctypes.POINTER(_P), _P, ctypes.POINTER(FcOptions), _C, _S]),
    "fc_session_create_batch": (_I, [ctypes.POINTER(_P), _P, ctypes.POINTER(FcBatchOptions), _C, _S]),
    "fc_session_batch_seed": (_I, [_P, _I, _I, _I, ctypes.c_uint64, _C, _S]),
    "fc_session_verify_batch": (_I, [_P, _IP, _I, ctypes.POINTER(FcAcceptConfig), _IP, _IP, _C, _S]),
    "fc_session_batch_position": (_I, [_P, _I]),
    "fc_session_batch_rollback": (_I, [_P, _I, _I, _C, _S]),
    "fc_session_destroy": (None, [_P]),
    "fc_session_reset": (None, [_P]),
    "fc_session_position": (_I, [_P]),
    "fc_session_stats": (FcStats, [_P]),
    "fc_session_prefill": (_I, [_P, _IP, _I, _FP, _C, _S]),
    "fc_session_append": (_I, [_P, _IP, _I, _FP, _C, _S]),
    "fc_session_decode": (_I, [_P, _I, _FP, _C, _S]),
    "fc_session_verify": (_I, [_P, _IP, _I, ctypes.POINTER(FcAcceptConfig), _IP, _IP, _IP, _FP, _C, _S]),
    "fc_session_rollback": (_I, [_P, _I, _C, _S]),
    "fc_session_copy_row_logits": (_I, [_P, _FP, _I]),
    "fc_session_seed_context": (_I, [_P, _I, ctypes.c_uint64, _C, _S]),
    "fc_session_ep_handle": (_I, [_P, ctypes.c_void_p, _S, _C, _S]),
    "fc_session_drafts": (_I, [_P, _IP, _I]),
    "fc_blocks_to_logical": (_I, [_I, ctypes.c_void_p, _S, _I, _I, ctypes.c_void_p, ctypes.c_void_p, _C, _S]),
    "fc_model_set_tensor_blocks": (_I, [_P, ctypes.c_char_p, _I, ctypes.c_void_p, _S, _C, _S]),
    "fc_model_set_tensor_rowscale": (_I, [_P, ctypes.c_char_p, ctypes.c_void_p, _S,
                                          ctypes.POINTER(ctypes.c_float), _I, _C, _S]),
    "fc_session_last_kernel_count": (_I, [_P]),
    "fc_session_exchange_wait_ms": (ctypes.c_double, [_P]),
    "fc_io_bytes": (None, [ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "fc_session_ep_connect": (_I, [_P, ctypes.c_char_p, _I, _C, _S]),
    "fc_session_set_profiling": (_I, [_P, _I]),
    "fc_session_profile": (_I, [_P, _I, _C, _S, ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_uint64)]),
    "fc_session_profile_reset": (None, [_P]),
    "fc_session_set_layer_trace": (_I, [_P, _I]),
    "fc_test_kv_length": (_I, [_P, _I]),
    "fc_test_embed": (_I, [_P, _IP, _I, _FP]),
    "fc_test_rmsnorm": (_I, [_P, _FP, ctypes.c_char_p, _I, _I, _FP]),
    "fc_test_matmul": (_I, [_P, ctypes.c_char_p, _FP, _I, _I, _I, _FP]),
    "fc_test_attention": (_I, [_P, _I, _FP, _I, _I, _FP]),
    "fc_test_moe": (_I, [_P, _I, _FP, _I, _IP, _FP, _FP, _FP, _FP, _FP]),
    "fc_test_dense_mlp": (_I, [_P, _I, _FP, _I, _FP]),
    "fc_test_prefill_layers": (_I, [_P, _IP, _I, _FP, _FP, _C, _S]),
    "fc_model_open": (_I, [ctypes.POINTER(_P), ctypes.c_char_p, _I, _C, _S]),
    "fm_init": (_I, []),
    "fm_device_name": (ctypes.c_char_p, []),
    "fm_matmul_q8": (None, [_FP, _FP, _P, _FP, _I, _I, _I, _I]),
    "fm_matmul_q4": (None, [_FP, _FP, _P, _FP, _I, _I, _I, _I]),
    "fm_matmul_deepseek_v4_fp8": (_I, [_FP, _FP, _P, _P, _I, _I, _I, _I]),
    "fm_matmul_deepseek_v4_fp4": (_I, [_FP, _FP, _P, _P, _I, _I, _I]),
    "fc_test_batch_page_table": (_I, [_I, _I, _I, _IP, _I]),
    "fc_test_copy_kv": (_I, [_P, _I, _FP, _FP, _I]),
    "fc_test_accept": (_I, [_FP, _I, _I, _IP, ctypes.POINTER(FcAcceptConfig), _I, _IP, _IP, _C, _S]),
    "fc_test_copy_routes": (_I, [_P, _I, _IP, _I]),
    "fc_test_copy_layer_outputs": (_I, [_P, _FP, _I]),
    "fc_runtime_init": (_I, [ctypes.POINTER(FcRuntime), _P, _I, _I]),
    "fc_runtime_forward": (_I, [ctypes.POINTER(FcRuntime), _IP, _I, ctypes.POINTER(_FP)]),
    "fc_runtime_argmax": (_I, [_FP, _I]),
    "fc_runtime_verify_token": (_I, [_FP, _I, ctypes.c_int64, _IP]),
    "fc_runtime_reset": (None, [ctypes.POINTER(FcRuntime)]),
    "fc_runtime_dspark_prefill": (_I, [ctypes.POINTER(FcRuntime)]),
    "fc_runtime_dspark_propose": (_I, [ctypes.POINTER(FcRuntime), _I, ctypes.POINTER(ctypes.c_int64), _FP]),
    "fc_runtime_free": (None, [ctypes.POINTER(FcRuntime)]),
    # include/floyd_kernels.h
    "fc_matmul": (_I, [_I, _FP, _FP, _P, _P, _I, _I, _I, _C, _S]),
    "fc_matmul_noalloc": (_I, [_I, _FP, _FP, _P, _P, _I, _I, _I, _C, _S]),
}

_lib = None


def load():
    """Loads libfloyd_cuda.so (building it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        try:
            from . import build
            build.build()
        except Exception as exc:  # no nvcc: the library must already exist
            raise RuntimeError(
                f"floyd_b200: {LIB_PATH} is missing and could not be built ({exc}); "
                "the backend has no CPU fallback") from exc
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
