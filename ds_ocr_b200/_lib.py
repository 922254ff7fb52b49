"""ctypes binding of the C ABI in include/ds_cuda.h (libds_cuda.so, in-tree).

There is no CPU fallback: if the library is missing this module raises, and
if no sm_100 device is present ds_cuda_init returns NULL and `Context`
raises. Tests that need a GPU are marked `gpu`.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("DS_CUDA_LIB") or os.path.join(HERE, "libds_cuda.so")

c_int, c_float, c_size_t, c_void_p, c_uint64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint64
P = c_void_p  # all pointers are passed as raw addresses

# name -> (restype, argtypes); must match include/ds_cuda.h
SIGNATURES = {
    "ds_cuda_init": (c_void_p, [c_int]),
    "ds_cuda_free": (None, [P]),
    "ds_cuda_is_available": (c_int, [P]),
    "ds_cuda_last_error": (ctypes.c_char_p, [P]),
    "ds_cuda_stream": (c_void_p, [P]),
    "ds_cuda_synchronize": (c_int, [P]),
    "ds_cuda_set_numerics": (c_int, [P, c_int, c_int]),
    "ds_cuda_register_bf16": (c_int, [P, P, c_size_t]),
    "ds_cuda_register_f32": (c_int, [P, P, c_size_t]),
    "ds_cuda_register_expert_block": (c_int, [P, P, c_size_t]),
    "ds_cuda_register_int8_block": (c_int, [P, P]),
    "ds_cuda_unregister": (c_int, [P, P]),
    "ds_cuda_device_ptr": (c_void_p, [P, P]),
    "ds_cuda_registered_bytes": (c_size_t, [P]),
    "ds_cuda_moe_experts": (c_int, [P, P, P, P, P, c_int, c_int, c_int, P]),
    "ds_cuda_shared_experts": (c_int, [P, P, P, P, c_int, c_int, P]),
    "ds_cuda_expert_forward_fused": (c_int, [P, P, P, P, P, c_int, c_int]),
    "ds_cuda_expert_forward_fused_int4": (c_int, [P, P, P, P, P, c_int, c_int]),
    "ds_cuda_moe_layer": (c_int, [P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P]),
    "ds_cuda_moe_layer_int8": (c_int, [P, P, P, P] + [P] * 12 + [c_int] * 5 + [P, P]),
    "ds_cuda_lm_head_argmax": (c_int, [P, P, P, c_int, c_int]),
    "ds_cuda_argmax_matvec_bf16": (c_int, [P, P, P, c_int, c_int, P]),
    "ds_cuda_argmax_matvec_bf16_batch": (c_int, [P, P, P, c_int, c_int, c_int, P, P]),
    "ds_cuda_matvec_bf16": (c_int, [P, P, P, P, P, c_int, c_int]),
    "ds_cuda_int8_quantize_bf16": (c_int, [P, P, c_int, c_int, P, P, P]),
    "ds_cuda_argmax_matvec_bf16_dev": (c_int, [P, P, P, c_int, c_int, P, P, P]),
    "ds_cuda_argmax_matvec_bf16_batch_dev": (c_int, [P, P, P, c_int, c_int, c_int, P, P, P]),
    "ds_cuda_moe_layer_dev": (c_int, [P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P]),
    "ds_cuda_moe_layer_int8_dev": (c_int, [P] * 16 + [c_int] * 5 + [P, P, P]),
    "ds_cuda_ep_unique_id": (c_int, [P, P]),
    "ds_cuda_ep_init": (c_int, [P, c_int, c_int, P]),
    "ds_cuda_ep_free": (c_int, [P]),
    "ds_cuda_prefill_moe_ep": (c_int, [P, P, P, P, c_int, P, P, P, P]),
    "ds_cuda_moe_experts_noalloc": (c_int, [P, P, P, P, c_int, c_int, c_int, P, P]),
    "ds_cuda_decoder_create": (c_int, [P, P, P, P, P]),
    "ds_cuda_decoder_destroy": (c_int, [P, c_int]),
    "ds_cuda_decoder_load_kv": (c_int, [P, c_int, c_int, c_int, c_int, P, P]),
    "ds_cuda_decoder_set_len": (c_int, [P, c_int, c_int]),
    "ds_cuda_decoder_get_len": (c_int, [P, c_int]),
    "ds_cuda_decoder_forward": (c_int, [P, c_int, P, P, P]),
    "ds_cuda_decoder_generate": (c_int, [P, c_int, P, c_int, P]),
    "ds_cuda_decoder_generate_dev": (c_int, [P, c_int, c_int, P]),
    "ds_cuda_decoder_launches_per_step": (c_int, [P, c_int]),
    "ds_cuda_decoder_set_sampling": (c_int, [P, c_int, c_float, c_int, c_float]),
    "ds_cuda_decoder_set_history": (c_int, [P, c_int, P, c_int]),
    "ds_cuda_decoder_get_history": (c_int, [P, c_int, P, c_int]),
    "ds_cuda_decoder_set_uniforms": (c_int, [P, c_int, P, c_int]),
    "ds_cuda_decoder_set_window": (c_int, [P, c_int, c_int, c_int]),
    "ds_cuda_decoder_set_embeddings": (c_int, [P, c_int, P]),
    "ds_cuda_decoder_prefill": (c_int, [P, c_int, P, c_int, P, P]),
    "ds_cuda_decoder_prefill_dev": (c_int, [P, c_int, P, c_int, P]),
    "ds_cuda_decoder_get_kv": (c_int, [P, c_int, c_int, c_int, c_int, P, P]),
    "ds_cuda_decoder_create_from_safetensors": (c_int, [P, ctypes.c_char_p, P]),
    "ds_cuda_safetensors_count": (c_int, [ctypes.c_char_p]),
    "ds_cuda_safetensors_find": (c_int, [ctypes.c_char_p, ctypes.c_char_p, P, P, P, P, P]),
    "ds_cuda_safetensors_error": (ctypes.c_char_p, []),
    "ds_cuda_batch_decoder_create": (c_int, [P, P, P, P, P, c_int]),
    "ds_cuda_batch_decoder_destroy": (c_int, [P, c_int]),
    "ds_cuda_batch_decoder_load_kv": (c_int, [P, c_int, c_int, c_int, c_int, c_int, P, P]),
    "ds_cuda_batch_decoder_set_len": (c_int, [P, c_int, c_int, c_int]),
    "ds_cuda_batch_decoder_forward": (c_int, [P, c_int, P, P, P]),
    "ds_cuda_batch_decoder_generate": (c_int, [P, c_int, P, c_int, P]),
    "ds_cuda_batch_decoder_generate_dev": (c_int, [P, c_int, c_int, P]),
    "ds_cuda_batch_decoder_set_sampling": (c_int, [P, c_int, ctypes.c_float, c_int, ctypes.c_float]),
    "ds_cuda_batch_decoder_set_history": (c_int, [P, c_int, c_int, P, c_int]),
    "ds_cuda_batch_decoder_get_history": (c_int, [P, c_int, c_int, P, c_int]),
    "ds_cuda_batch_decoder_set_uniforms": (c_int, [P, c_int, P, c_int]),
    "ds_cuda_batch_decoder_set_window": (c_int, [P, c_int, c_int, P]),
    "ds_cuda_prefill_moe": (c_int, [P, P, P, P, c_int, P, P, P]),
    "ds_cuda_prefill_moe_dev": (c_int, [P, P, P, P, c_int, P, P, P, P]),
    "ds_cuda_prefill_check": (c_int, [P]),
    "ds_cuda_skinny_matmul_dev": (c_int, [P, P, c_int, c_int, P, c_int, P, P, P]),
    "ds_cuda_prefill_route_dev": (c_int, [P, P, P, P, c_int, P, P, P, P, P, P]),
    "ds_cuda_prefill_experts_dev": (c_int, [P, P, P, P, P, c_int, c_int, P, P, c_int, P, P, P, c_int, P, P]),
    "ds_cuda_prefill_combine_dev": (c_int, [P, P, P, c_int, P, P, P, P, P, P]),
    "ds_cuda_ep_dispatch_dev": (c_int, [P, c_int, c_int, c_int, c_int, P, P, P, c_int, P, P, P, P, P]),
    "ds_cuda_ep_pairs_dev": (c_int, [P, c_int, c_int, c_int, P, P, c_int, P, P, P, P]),
    "ds_cuda_prefill_timing": (c_int, [P, c_int]),
    "ds_cuda_prefill_stage_ms": (c_int, [P, P]),
    "ds_synth_normal_bf16": (None, [P, c_size_t, c_uint64, c_float, c_float]),
    "ds_synth_normal_f32": (None, [P, c_size_t, c_uint64, c_float, c_float]),
    "ds_synth_normal_f32_bf16exact": (None, [P, c_size_t, c_uint64, c_float, c_float]),
}

_lib = None


def load():
    """Load libds_cuda.so (building it first if only the sources are present)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        _build.build()
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_symbols():
    """Function names declared in include/ds_cuda.h (parsed from the header)."""
    import re
    hdr = os.path.join(os.path.dirname(HERE), "include", "ds_cuda.h")
    text = open(hdr).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ds_(?:cuda|synth)_\w+)\s*\(", text)))


class DsCudaError(RuntimeError):
    pass
