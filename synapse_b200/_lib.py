"""ctypes binding of libsynapse_cuda.so (include/synapse_cuda.h).

The library is loaded from this package directory only; there is no fallback.
If it is missing, importing synapse_b200 raises ImportError with the build
command to run.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsynapse_cuda.so")

c_size = ctypes.c_size_t
c_vp = ctypes.c_void_p
c_st = ctypes.c_int32

# name -> (restype, argtypes). Every symbol declared in include/synapse_cuda.h.
SIGNATURES = {
    "syn_cuda_context_create": (c_st, [ctypes.c_int, ctypes.POINTER(c_vp)]),
    "syn_cuda_context_destroy": (c_st, [c_vp]),
    "syn_cuda_context_get_error": (c_st, [c_vp, ctypes.POINTER(ctypes.c_int32)]),
    "syn_cuda_capability_summary": (c_st, [c_vp]),
    "syn_cuda_status_string": (ctypes.c_char_p, [c_st]),
    "syn_cuda_last_error": (ctypes.c_char_p, []),
    "syn_cuda_quantize_per_channel_int8": (c_st, [c_vp, c_size, c_size, c_vp, c_vp, c_vp]),
    "syn_cuda_quantize_weights_int8": (c_st, [c_vp, c_size, c_size, c_vp, c_vp, c_vp]),
    "syn_cuda_qgemm_int8": (c_st, [c_size, c_size, c_size, c_vp, c_size, c_vp, c_size, c_vp,
                                   c_size, c_vp, c_vp, c_vp]),
    "syn_cuda_q4_0_gemv": (c_st, [c_size, c_size, c_vp, c_vp, c_vp, c_vp]),
    "syn_cuda_weight_upload": (c_st, [c_vp, ctypes.c_int, c_vp, c_size, c_size, c_vp,
                                      ctypes.POINTER(c_vp)]),
    "syn_cuda_weight_destroy": (c_st, [c_vp]),
    "syn_cuda_weight_bytes": (c_st, [c_vp, ctypes.POINTER(c_size)]),
    "syn_cuda_weight_dequant": (c_st, [c_vp, c_vp]),
    "syn_cuda_qmatmul": (c_st, [c_vp, c_vp, c_vp, c_size, c_vp, c_vp]),
    "syn_cuda_qmatmul_int8_prequant": (c_st, [c_vp, c_vp, c_vp, c_vp, c_size, c_vp, c_vp]),
    "syn_cuda_qmatmul_noalloc": (c_st, [c_vp, c_vp, c_size, c_vp, c_vp]),
    "syn_cuda_qmatmul_rmsnorm": (c_st, [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_float, c_vp,
                                        ctypes.c_int, c_vp, c_vp]),
    "syn_cuda_rope_tables": (c_st, [ctypes.c_double, c_size, c_size, c_vp, c_vp]),
    "syn_cuda_rmsnorm": (c_st, [c_vp, c_vp, c_size, c_size, ctypes.c_float, c_vp, c_vp]),
    "syn_cuda_add_rmsnorm": (c_st, [c_vp, c_vp, c_vp, c_size, c_size, ctypes.c_float, c_vp,
                                    c_vp]),
    "syn_cuda_embed_rmsnorm": (c_st, [c_vp, c_size, c_vp, c_size, c_size, c_vp, ctypes.c_float,
                                      c_vp, c_vp, c_vp]),
    "syn_cuda_kvcache_create": (c_st, [c_vp, c_size, c_size, c_size, c_size, c_size,
                                       ctypes.POINTER(c_vp)]),
    "syn_cuda_kvcache_destroy": (c_st, [c_vp]),
    "syn_cuda_kvcache_len": (c_st, [c_vp, c_size, ctypes.POINTER(c_size)]),
    "syn_cuda_kvcache_view": (c_st, [c_vp, c_size, c_size, ctypes.POINTER(c_vp),
                                     ctypes.POINTER(c_vp)]),
    "syn_cuda_kvcache_append": (c_st, [c_vp, c_size, c_size, c_vp, c_vp, c_size, c_vp]),
    "syn_cuda_kvcache_advance": (c_st, [c_vp, c_size, c_size, c_vp]),
    "syn_cuda_kvcache_truncate": (c_st, [c_vp, c_size, c_size, c_vp]),
    "syn_cuda_kvcache_reset": (c_st, [c_vp, c_size, c_vp]),
    "syn_cuda_attention_decode": (c_st, [c_vp, c_size, c_size, c_vp, c_vp, c_vp, c_size, c_size,
                                         c_vp, c_vp, ctypes.c_float, c_vp, c_vp, c_size, c_vp,
                                         c_size, c_vp]),
    "syn_cuda_qk_norm_rope_kv_append": (c_st, [c_vp, c_size, c_size, c_size, c_vp, c_vp, c_vp,
                                               c_size, c_size, c_vp, c_vp, ctypes.c_float, c_vp,
                                               c_vp, c_vp]),
    "syn_cuda_attention_prefill": (c_st, [c_vp, c_size, c_size, c_size, c_vp, c_vp, c_vp, c_size,
                                          c_size, c_vp, c_vp, ctypes.c_float, c_vp, c_vp, c_vp,
                                          c_size, c_vp]),
    "syn_cuda_attention_decode_flash": (c_st, [c_vp, c_size, c_size, c_vp, c_vp, c_vp, c_size,
                                               c_size, c_vp, c_vp, ctypes.c_float, c_vp, c_vp,
                                               c_size, c_vp, c_size, c_vp]),
    "syn_cuda_attention_prefill_flash": (c_st, [c_vp, c_size, c_size, c_size, c_vp, c_vp, c_vp,
                                                c_size, c_size, c_vp, c_vp, ctypes.c_float, c_vp,
                                                c_vp, c_vp, c_size, c_vp]),
    "syn_cuda_swiglu": (c_st, [c_vp, c_vp, c_size, c_size, c_size, ctypes.c_int, c_vp, c_size,
                               c_vp]),
    "syn_cuda_argmax": (c_st, [c_vp, c_size, c_size, c_vp, c_vp]),
    "syn_cuda_model_create": (c_st, [c_vp, ctypes.c_char_p, c_size, c_size,
                                     ctypes.POINTER(c_vp)]),
    "syn_cuda_model_set_tensor": (c_st, [c_vp, ctypes.c_char_p, c_vp, c_size]),
    "syn_cuda_model_set_linear": (c_st, [c_vp, ctypes.c_char_p, ctypes.c_int, c_vp, c_size,
                                         c_size, c_vp]),
    "syn_cuda_model_finalize": (c_st, [c_vp]),
    "syn_cuda_prefill": (c_st, [c_vp, c_size, c_vp, c_size, c_vp, c_vp]),
    "syn_cuda_decode_step": (c_st, [c_vp, c_size, c_vp, c_vp, c_vp]),
    "syn_cuda_generate": (c_st, [c_vp, c_size, c_size, c_vp]),
    "syn_cuda_kvcache_create_paged": (c_st, [c_vp, c_size, c_size, c_size, c_size, c_size, c_size,
                                             c_size, ctypes.POINTER(c_vp)]),
    "syn_cuda_kvcache_pages_free": (c_st, [c_vp, ctypes.POINTER(c_size)]),
    "syn_cuda_model_set_kv_paging": (c_st, [c_vp, c_size, c_size]),
    "syn_cuda_model_kv_pages_free": (c_st, [c_vp, ctypes.POINTER(c_size)]),
    "syn_cuda_decode_step_slots": (c_st, [c_vp, c_size, c_vp, c_vp, c_vp, c_vp]),
    "syn_cuda_decode_span": (c_st, [c_vp, c_size, c_vp, c_size, c_size, c_vp, c_vp]),
    "syn_cuda_generate_speculative": (c_st, [c_vp, c_size, ctypes.c_int32, c_size, c_size, c_size,
                                             c_vp, ctypes.POINTER(c_size), ctypes.POINTER(c_size)]),
    "syn_cuda_model_seq_len": (c_st, [c_vp, c_size, ctypes.POINTER(c_size)]),
    "syn_cuda_model_reset": (c_st, [c_vp, c_size]),
    "syn_cuda_model_truncate": (c_st, [c_vp, c_size, c_size]),
    "syn_cuda_model_destroy": (c_st, [c_vp]),
    "syn_cuda_tp_unique_id": (c_st, [c_vp]),
    "syn_cuda_tp_init": (c_st, [c_vp, ctypes.c_int, ctypes.c_int, c_vp]),
    "syn_cuda_tp_allreduce_sum": (c_st, [c_vp, c_vp, c_size, c_vp]),
    "syn_gguf_open": (c_st, [ctypes.c_char_p, ctypes.POINTER(c_vp)]),
    "syn_gguf_close": (c_st, [c_vp]),
    "syn_gguf_tensor_count": (c_st, [c_vp, ctypes.POINTER(c_size)]),
    "syn_gguf_tensor_info": (c_st, [c_vp, c_size, ctypes.POINTER(ctypes.c_char_p),
                                    ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(c_size),
                                    ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(c_vp),
                                    ctypes.POINTER(c_size)]),
    "syn_gguf_meta_num": (c_st, [c_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "syn_gguf_meta_str": (c_st, [c_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)]),
    "syn_gguf_runner_name": (c_st, [ctypes.c_char_p, ctypes.c_char_p, c_size]),
    "syn_gguf_config_json": (c_st, [c_vp, ctypes.c_char_p, c_size, ctypes.POINTER(c_size)]),
    "syn_safetensors_open": (c_st, [ctypes.c_char_p, ctypes.POINTER(c_vp)]),
    "syn_safetensors_close": (c_st, [c_vp]),
    "syn_safetensors_tensor_count": (c_st, [c_vp, ctypes.POINTER(c_size)]),
    "syn_safetensors_tensor_info": (c_st, [c_vp, c_size, ctypes.POINTER(ctypes.c_char_p),
                                           ctypes.POINTER(ctypes.c_int), ctypes.POINTER(c_size),
                                           ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(c_vp),
                                           ctypes.POINTER(c_size)]),
    "syn_convert_to_f32": (c_st, [ctypes.c_int, c_vp, c_size, c_vp]),
    "syn_cuda_quantize_weights_int8_half": (c_st, [c_vp, ctypes.c_int, c_size, c_size, c_vp, c_vp,
                                                   c_vp]),
    "syn_cuda_quantize_weights_int8_host": (c_st, [c_vp, ctypes.c_int, c_vp, c_size, c_size, c_vp,
                                                   c_vp]),
    "syn_cuda_weight_upload_cached": (c_st, [c_vp, ctypes.c_int, c_vp, c_size, c_size, c_vp,
                                             ctypes.c_char_p, ctypes.POINTER(c_vp),
                                             ctypes.POINTER(ctypes.c_int)]),
    "syn_cuda_model_load_gguf": (c_st, [c_vp, c_vp]),
    "syn_cuda_model_load_safetensors": (c_st, [c_vp, c_vp]),
    "syn_cuda_model_set_cache_dir": (c_st, [c_vp, ctypes.c_char_p]),
    "syn_cuda_model_cache_hits": (c_st, [c_vp, ctypes.POINTER(ctypes.c_int)]),
    "syn_cuda_tp_shard_linear": (c_st, [ctypes.c_int, c_vp, c_size, c_size, c_vp, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, c_vp, c_vp,
                                        ctypes.POINTER(c_size), ctypes.POINTER(c_size)]),
}


class CapabilitySummary(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_uint32), ("target_arch", ctypes.c_uint32),
                ("target_os", ctypes.c_uint32), ("simd_backend", ctypes.c_uint32),
                ("runtime_profile", ctypes.c_uint32), ("support_level", ctypes.c_uint32),
                ("feature_bits", ctypes.c_uint64)]


def load(path=LIB_PATH):
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python synapse_b200/build.py` "
            "(the CUDA backend has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib
