"""ctypes binding of ``libpopcorn_cuda.so`` (the C ABI in include/popcorn_cuda.h).

The library is the product; this module only declares its signatures. It
fails loudly when the library has not been built: there is no fallback.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libpopcorn_cuda.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "popcorn_cuda.h")

PC_MAX_RANK = 8


class pc_tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_int64 * PC_MAX_RANK)]


class pc_attention_mask(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("window", ctypes.c_int32)]


BORROW_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                             ctypes.POINTER(ctypes.c_int))
RELEASE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p)
HOOK_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p)


class pc_decode_stack_desc(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("num_layers", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("max_ctx", ctypes.c_int32), ("eps", ctypes.c_float),
                ("attn_scale", ctypes.c_float), ("activation", ctypes.c_int32), ("add_one_to_weight", ctypes.c_int32),
                ("layers", ctypes.c_void_p), ("x", ctypes.c_void_p), ("x2", ctypes.c_void_p), ("h", ctypes.c_void_p),
                ("q", ctypes.c_void_p), ("attn", ctypes.c_void_p), ("act", ctypes.c_void_p),
                ("position", ctypes.c_void_p), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
                ("qk_norm", ctypes.c_int32), ("norm_v", ctypes.c_int32), ("rope_rows", ctypes.c_int64)]


class pc_affine_quantized(ctypes.Structure):
    _fields_ = [("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("biases", ctypes.c_void_p),
                ("out_features", ctypes.c_int64), ("in_features", ctypes.c_int64), ("bits", ctypes.c_int32),
                ("group_size", ctypes.c_int32)]


class pc_scratch_allocator(ctypes.Structure):
    _fields_ = [("ctx", ctypes.c_void_p), ("borrow", BORROW_FN), ("release", RELEASE_FN)]


_lib = None


MAX_PEERS = 8


class pc_peer_group(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("partial", (ctypes.c_void_p * 2) * MAX_PEERS),
                ("control", ctypes.POINTER(ctypes.c_uint32) * MAX_PEERS)]


def lib():
    """Loads the CUDA library once; raises ImportError if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("popcorn_b200: %s is missing; build it with `python -c \"import __graft_entry__ as g; "
                              "g.build()\"` (nvcc, sm_100a)" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def _declare(L):
    P, I, I32, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
    T = ctypes.POINTER(pc_tensor)
    PP = ctypes.POINTER(ctypes.c_void_p)
    M = pc_attention_mask
    sig = {
        "pc_last_error_message": ([], ctypes.c_char_p),
        "pc_dtype_stride": ([I32], I),
        "pc_scratch_spec_byte_count": ([ctypes.POINTER(I64), I32, I32], I64),
        "pc_version": ([], I),
        "pc_device_count": ([ctypes.POINTER(I)], I),
        "pc_buffer_alloc": ([I, ctypes.c_size_t, PP], I),
        "pc_buffer_free": ([P], I),
        "pc_memcpy_htod_async": ([P, P, ctypes.c_size_t, P], I),
        "pc_memcpy_dtoh_async": ([P, P, ctypes.c_size_t, P], I),
        "pc_stream_synchronize": ([P], I),
        "pc_device_error_check": ([I, ctypes.POINTER(ctypes.c_uint32)], I),
        "pc_library_create": ([I, PP], I),
        "pc_library_destroy": ([P], None),
        "pc_library_device": ([P, ctypes.POINTER(I)], I),
        "pc_library_lookup": ([P, ctypes.c_char_p, PP], I),
        "pc_library_function_count": ([P], I),
        "pc_library_function_name": ([P, I], ctypes.c_char_p),
        "pc_encoder_create": ([P, P, ctypes.POINTER(pc_scratch_allocator), PP], I),
        "pc_encoder_destroy": ([P], None),
        "pc_encoder_encode": ([P, P], I),
        "pc_encoder_barrier": ([P], I),
        "pc_encoder_barrier_count": ([P], I64),
        "pc_encoder_dispatch_count": ([P], I64),
        "pc_encoder_set_dispatch_hook": ([P, HOOK_FN, P], I),
        "pc_encoder_stream": ([P, PP], I),
        "pc_kernel_destroy": ([P], None),
        "pc_kernel_name": ([P], ctypes.c_char_p),
        "pc_kernel_binding_count": ([P], I),
        "pc_kernel_binding": ([P, I, T, ctypes.POINTER(I)], I),
        "pc_kernel_function_names": ([P], ctypes.c_char_p),
        "pc_kernel_set_l2_prefetch": ([P, I32, P, ctypes.c_uint64], I),
        "pc_kernel_set_hint": ([P, I32, ctypes.c_int64], I),
        "pc_flash_attention_route": ([I64, I64, I32], I),
        "pc_kernel_flash_attention": ([T, T, T, T, F, M, PP], I),
        "pc_kernel_flash_attention_dims": ([T, T, T, T, I64, I64, I64, I64, I64, I64, F, M, PP], I),
        "pc_kernel_flash_decoding_ragged": ([T, T, T, T, T, F, M, PP], I),
        "pc_kernel_kv_cache_write": ([T, T, I64, PP], I),
        "pc_kernel_kv_cache_write_dims": ([T, T, I64, I64, I64, I64, I64, I64, PP], I),
        "pc_kernel_rmsnorm": ([T, T, T, I32, F, I32, PP], I),
        "pc_kernel_rmsnorm_dims": ([T, T, T, I64, I64, F, I32, PP], I),
        "pc_kernel_matmul": ([T, T, T, I32, PP], I),
        "pc_kernel_matmul_dims": ([T, T, T, I64, I64, I64, I32, PP], I),
        "pc_kernel_gelu_tanh": ([T, T, PP], I),
        "pc_kernel_mul": ([T, T, T, PP], I),
        "pc_kernel_add": ([T, T, T, PP], I),
        "pc_kernel_silu": ([T, T, PP], I),
        "pc_kernel_scalar_mul": ([T, F, T, PP], I),
        "pc_kernel_attention_mask_build": ([T, I32, PP], I),
        "pc_kernel_rmsnorm_matmul": ([T, T, F, I32, T, T, PP], I),
        "pc_kernel_gated_mlp": ([T, T, F, I32, T, T, I32, T, PP], I),
        "pc_kernel_matmul_residual": ([T, T, T, T, PP], I),
        "pc_kernel_qkv_projection": ([T, T, F, I32, T, T, T, T, I64, T, PP], I),
        "pc_kernel_qkv_scatter": ([T, T, T, T, I64, T, PP], I),
        "pc_kernel_argmax": ([T, T, I32, PP], I),
        "pc_kernel_rope_build_cos_sin": ([T, T, T, T, F, PP], I),
        "pc_kernel_matmul_affine_quantized": ([T, T, T, T, I64, I64, I32, I32, T, PP], I),
        "pc_kernel_embedding_gather": ([T, T, T, PP], I),
        "pc_kernel_aq_rmsnorm_matmul": ([T, T, F, I32, ctypes.POINTER(pc_affine_quantized), T, PP], I),
        "pc_kernel_aq_matmul_residual": ([T, ctypes.POINTER(pc_affine_quantized), T, T, PP], I),
        "pc_kernel_aq_gated_mlp": ([T, T, F, I32, ctypes.POINTER(pc_affine_quantized), I32, T, PP], I),
        "pc_kernel_aq_qkv_projection": ([T, T, F, I32, ctypes.POINTER(pc_affine_quantized), T, T, T, I64, T, PP],
                                        I),
        "pc_kernel_embedding_gather_affine_quantized": ([T, T, T, T, I64, I64, I32, I32, T, PP], I),
        "pc_kernel_rope_apply": ([T, T, T, T, PP], I),
        "pc_kernel_qk_norm_rope": ([T, T, T, T, T, T, T, F, I32, I32, I64, T, PP], I),
        "pc_ipc_get_handle": ([P, ctypes.POINTER(ctypes.c_uint8)], I),
        "pc_ipc_open_handle": ([ctypes.POINTER(ctypes.c_uint8), PP], I),
        "pc_ipc_close_handle": ([P], I),
        "pc_kernel_allreduce_add_rmsnorm": ([ctypes.POINTER(pc_peer_group), I32, T, T, F, I32, T, T, PP], I),
        "pc_kernel_matmul_allreduce_add_rmsnorm": ([T, T, ctypes.POINTER(pc_peer_group), I32, T, T, F, I32, T, T, PP],
                                                   I),
        "pc_kernel_gated_activation": ([T, I32, T, PP], I),
        "pc_kernel_add_rmsnorm": ([T, T, T, F, I32, T, T, PP], I),
        "pc_flash_decoding_noalloc": ([T, T, T, T, T, F, M, P], I),
        "pc_flash_decoding_noalloc_capacity": ([], ctypes.c_size_t),
        "pc_decode_stack_workspace_bytes": ([ctypes.POINTER(pc_decode_stack_desc), ctypes.POINTER(ctypes.c_uint64)], I),
        "pc_kernel_decode_stack": ([ctypes.POINTER(pc_decode_stack_desc), PP], I),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res


def header_symbols():
    """Names of every function include/popcorn_cuda.h declares (PC_API)."""
    import re
    text = open(HEADER_PATH).read()
    return sorted(set(re.findall(r"PC_API\s+[^;(]*?\b(pc_\w+)\s*\(", text)))
