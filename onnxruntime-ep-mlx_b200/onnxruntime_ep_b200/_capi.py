"""ctypes binding of ``include/b200_paged.h``, ``include/b200_ep.h`` and ``include/b200_shard.h``
(the library's C ABI).

The library is loaded from this package folder.  A missing or stale library raises at import
time: there is no CPU fallback for the claimed path.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libb200_paged.so"

B200_OK = 0
B200_ERR_INVALID_ARGUMENT = 1
B200_ERR_FAIL = 2
B200_ERR_CUDA = 3
B200_ERR_UNSUPPORTED = 4
B200_ERR_WORKSPACE = 5
B200_ERR_DEVICE = 6

DTYPE_FLOAT = 1
DTYPE_UINT8 = 2
DTYPE_INT8 = 3
DTYPE_INT32 = 6
DTYPE_INT64 = 7
DTYPE_FLOAT16 = 10
DTYPE_BFLOAT16 = 16
DTYPE_FLOAT8E4M3FN = 17

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class PagedAttentionParams(ctypes.Structure):
    """Mirror of ``B200PagedAttentionParams``."""

    _fields_ = [
        ("num_heads", _i32), ("kv_num_heads", _i32), ("head_size", _i32), ("scale", _f32),
        ("is_causal", _i32), ("local_window_size", _i32), ("softcap", _f32),
        ("do_rotary", _i32), ("rotary_interleaved", _i32), ("rotary_offset", _i32),
        ("rotary_dim", _i32), ("rotary_positions", _i32), ("qk_norm_epsilon", _f32),
        ("act_dtype", _i32), ("cache_dtype", _i32), ("k_quant_per_channel", _i32),
        ("v_quant_per_channel", _i32),
        ("num_tokens", _i32), ("batch", _i32), ("num_blocks", _i32), ("block_size", _i32),
        ("max_blocks_per_seq", _i32),
        ("query_row_stride", _i64), ("key_row_stride", _i64), ("value_row_stride", _i64),
        ("query", _vp), ("key", _vp), ("value", _vp), ("key_cache", _vp), ("value_cache", _vp),
        ("cumulative_sequence_length", _vp), ("past_seqlens", _vp), ("block_table", _vp),
        ("cos_cache", _vp), ("sin_cache", _vp), ("slot_mapping", _vp), ("head_sink", _vp),
        ("q_norm_weight", _vp), ("k_norm_weight", _vp), ("k_scale", _vp), ("v_scale", _vp),
        ("output", _vp),
        ("host_cumulative_sequence_length", _vp), ("host_past_seqlens", _vp),
        ("host_block_table", _vp), ("host_slot_mapping", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t), ("device_status", _vp),
        ("decode_min_tiles_per_warp", _i32), ("force_generic", _i32), ("num_sms", _i32),
        ("attention_event_begin", _vp), ("attention_event_end", _vp),
        ("kv_cache_latent", _i32), ("v_head_size", _i32),
    ]


MAX_RANK = 8


class TensorInfo(ctypes.Structure):
    _fields_ = [("present", _i32), ("dtype", _i32), ("rank", _i32), ("shape", _i64 * MAX_RANK)]


class NodeInfo(ctypes.Structure):
    """Mirror of ``B200NodeInfo`` (claim predicate input)."""

    _fields_ = [
        ("num_inputs", _i32), ("num_outputs", _i32),
        ("inputs", TensorInfo * 17), ("outputs", TensorInfo * 3),
        ("num_heads", _i64), ("kv_num_heads", _i64), ("is_causal", _i64),
        ("local_window_size", _i64), ("do_rotary", _i64), ("rotary_interleaved", _i64),
        ("rotary_offset", _i64), ("v_head_size", _i64),
        ("has_scale", _i32), ("scale", _f32), ("softcap", _f32), ("qk_norm_epsilon", _f32),
        ("kv_cache_layout", ctypes.c_char * 16), ("k_quant_type", ctypes.c_char * 16),
        ("v_quant_type", ctypes.c_char * 16), ("k_cache_dtype", ctypes.c_char * 16),
        ("v_cache_dtype", ctypes.c_char * 16),
    ]


class GqaParams(ctypes.Structure):
    """Mirror of ``B200GqaParams`` (GroupQueryAttention over a contiguous BNSH cache)."""

    _fields_ = [
        ("num_heads", _i32), ("kv_num_heads", _i32), ("head_size", _i32), ("scale", _f32),
        ("is_causal", _i32), ("local_window_size", _i32), ("softcap", _f32), ("smooth_softmax", _i32),
        ("dtype", _i32), ("batch", _i32), ("seq", _i32), ("new_seq", _i32), ("cap", _i32),
        ("present_cap", _i32), ("total_sequence_length", _i32),
        ("query_row_stride", _i64), ("key_row_stride", _i64), ("value_row_stride", _i64),
        ("query", _vp), ("key", _vp), ("value", _vp), ("past_key", _vp), ("past_value", _vp),
        ("present_key", _vp), ("present_value", _vp), ("seqlens_k", _vp), ("host_seqlens_k", _vp),
        ("head_sink", _vp), ("output", _vp), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("num_sms", _i32),
        ("do_rotary", _i32), ("rotary_interleaved", _i32), ("rotary_dim", _i32), ("rotary_positions", _i32),
        ("cos_cache", _vp), ("sin_cache", _vp), ("position_ids", _vp), ("host_position_ids", _vp),
        ("position_ids_width", _i32),
        ("attention_bias", _vp), ("bias_batch", _i32), ("bias_heads", _i32), ("bias_seq", _i32),
        ("bias_total", _i32), ("q_norm_weight", _vp), ("k_norm_weight", _vp), ("qk_norm_epsilon", _f32),
        ("qk_output", _i32), ("output_qk", _vp),
        ("cache_dtype", _i32), ("k_scale", _vp), ("v_scale", _vp), ("k_quant_per_channel", _i32),
        ("v_quant_per_channel", _i32), ("sliding_window_cache", _i32),
    ]


class GqaNodeInfo(ctypes.Structure):
    """Mirror of ``B200GqaNodeInfo`` (GroupQueryAttention claim predicate input)."""

    _fields_ = [
        ("num_inputs", _i32), ("num_outputs", _i32),
        ("inputs", TensorInfo * 16), ("outputs", TensorInfo * 4),
        ("num_heads", _i64), ("kv_num_heads", _i64), ("causal", _i64), ("local_window_size", _i64),
        ("do_rotary", _i64), ("rotary_interleaved", _i64), ("sliding_window_cache", _i64),
        ("smooth_softmax", _i64), ("qk_output", _i64), ("kv_cache_bit_width", _i64),
        ("has_causal", _i32), ("has_local_window_size", _i32), ("has_smooth_softmax", _i32),
        ("softcap", _f32), ("has_scale", _i32), ("scale", _f32), ("has_qk_norm_epsilon", _i32),
        ("qk_norm_epsilon", _f32), ("k_quant_type", ctypes.c_char * 16), ("v_quant_type", ctypes.c_char * 16),
    ]


class EpOptions(ctypes.Structure):
    """Mirror of ``B200EpOptions`` (include/b200_ep.h)."""

    _fields_ = [("kv_pool_bytes", ctypes.c_uint64), ("has_kv_pool_bytes", _i32), ("num_gpus", _i32),
                ("device_id", _i32), ("decode_min_tiles_per_warp", _i32), ("force_generic", _i32),
                ("check_status", _i32)]


class KvPoolDesc(ctypes.Structure):
    """Mirror of ``B200KvPoolDesc``."""

    _fields_ = [("device", _i32), ("block_size", _i32), ("kv_num_heads", _i32), ("head_size", _i32),
                ("cache_dtype", _i32), ("num_blocks", _i32), ("budget_bytes", ctypes.c_uint64),
                ("key_cache", _vp), ("value_cache", _vp), ("k_scale", _vp), ("v_scale", _vp)]


class KvPoolInfo(ctypes.Structure):
    """Mirror of ``B200KvPoolInfo``."""

    _fields_ = [("key_cache", _vp), ("value_cache", _vp), ("k_scale", _vp), ("v_scale", _vp),
                ("num_blocks", _i32), ("free_blocks", _i32), ("block_size", _i32), ("owns_memory", _i32),
                ("block_bytes", ctypes.c_uint64), ("allocated_bytes", ctypes.c_uint64)]


class PagedTensors(ctypes.Structure):
    """Mirror of ``B200PagedTensors`` (one PagedAttention Compute's inputs and sizes)."""

    _fields_ = [("query", _vp), ("key", _vp), ("value", _vp), ("key_cache", _vp), ("value_cache", _vp),
                ("cumulative_sequence_length", _vp), ("past_seqlens", _vp), ("block_table", _vp),
                ("cos_cache", _vp), ("sin_cache", _vp), ("slot_mapping", _vp), ("head_sink", _vp),
                ("q_norm_weight", _vp), ("k_norm_weight", _vp), ("k_scale", _vp), ("v_scale", _vp),
                ("output", _vp), ("host_cumulative_sequence_length", _vp), ("host_past_seqlens", _vp),
                ("host_block_table", _vp), ("host_slot_mapping", _vp),
                ("num_tokens", _i32), ("query_hidden", _i32), ("batch", _i32), ("num_blocks", _i32),
                ("block_size", _i32), ("max_blocks_per_seq", _i32), ("rotary_positions", _i32),
                ("rotary_half_dim", _i32), ("act_dtype", _i32), ("cache_dtype", _i32)]


B200_ORT_OK, B200_ORT_INVALID_ARGUMENT, B200_ORT_EP_FAIL = 0, 1, 2

SHARD_MAX_RANKS = 8


class ShardGatherParams(ctypes.Structure):
    """Mirror of ``B200ShardGatherParams`` (include/b200_shard.h)."""

    _fields_ = [("world", _i32), ("rank", _i32), ("rows", _i32), ("slice_bytes", _i32), ("local", _vp),
                ("outputs", _vp * SHARD_MAX_RANKS), ("flags", _vp * SHARD_MAX_RANKS), ("state", _vp),
                ("status", _vp), ("num_sms", _i32)]

# Every entry point the headers declare, with its ctypes signature.
SIGNATURES = {
    "b200_version": (ctypes.c_int, []),
    "b200_params_size": (ctypes.c_size_t, []),
    "b200_node_info_size": (ctypes.c_size_t, []),
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_launch_count": (ctypes.c_uint64, []),
    "b200_paged_attention_workspace_size": (
        ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), ctypes.POINTER(ctypes.c_size_t)]),
    "b200_paged_attention_validate_host": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams)]),
    "b200_paged_attention": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), _vp]),
    "b200_kv_append": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), _vp]),
    "b200_paged_attention_static_scratch": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), _vp]),
    "b200_read_status_static_scratch": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), _vp]),
    "b200_read_status": (ctypes.c_int, [ctypes.POINTER(PagedAttentionParams), _vp]),
    "b200_selftest_tcgen05": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_paged_attention_claim": (
        ctypes.c_int, [ctypes.POINTER(NodeInfo), ctypes.c_char_p, ctypes.c_size_t]),
    "b200_gqa_params_size": (ctypes.c_int, []),
    "b200_gqa_node_info_size": (ctypes.c_int, []),
    "b200_group_query_attention_workspace_size": (
        ctypes.c_int, [ctypes.POINTER(GqaParams), ctypes.POINTER(ctypes.c_size_t)]),
    "b200_group_query_attention": (ctypes.c_int, [ctypes.POINTER(GqaParams), _vp]),
    "b200_group_query_attention_read_status": (ctypes.c_int, [ctypes.POINTER(GqaParams), _vp]),
    "b200_group_query_attention_claim": (
        ctypes.c_int, [ctypes.POINTER(GqaNodeInfo), ctypes.c_char_p, ctypes.c_size_t]),
    # include/b200_ep.h
    "b200_ep_options_parse": (ctypes.c_int, [ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p),
                                             ctypes.c_size_t, ctypes.POINTER(EpOptions)]),
    "b200_ort_error_class": (ctypes.c_int, [ctypes.c_int]),
    "b200_ep_struct_size": (ctypes.c_size_t, [_i32]),
    "b200_kv_pool_block_bytes": (ctypes.c_int, [ctypes.POINTER(KvPoolDesc), ctypes.POINTER(ctypes.c_uint64)]),
    "b200_kv_pool_create": (ctypes.c_int, [ctypes.POINTER(KvPoolDesc), ctypes.POINTER(_vp)]),
    "b200_kv_pool_destroy": (ctypes.c_int, [_vp]),
    "b200_kv_pool_info": (ctypes.c_int, [_vp, ctypes.POINTER(KvPoolInfo)]),
    "b200_kv_pool_alloc": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_i32)]),
    "b200_kv_pool_free": (ctypes.c_int, [_vp, ctypes.POINTER(_i32), _i32]),
    "b200_kv_pool_blocks_for": (_i32, [_vp, _i64]),
    "b200_ep_node_create_paged": (ctypes.c_int, [ctypes.POINTER(NodeInfo), ctypes.POINTER(EpOptions),
                                                 ctypes.POINTER(_vp)]),
    "b200_ep_node_create_gqa": (ctypes.c_int, [ctypes.POINTER(GqaNodeInfo), ctypes.POINTER(EpOptions),
                                               ctypes.POINTER(_vp)]),
    "b200_ep_node_destroy": (ctypes.c_int, [_vp]),
    "b200_ep_node_compute_paged": (ctypes.c_int, [_vp, ctypes.POINTER(PagedTensors), _vp]),
    "b200_ep_node_compute_gqa": (ctypes.c_int, [_vp, ctypes.POINTER(GqaParams), _vp]),
    "b200_ep_node_stats": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "b200_ep_device_alloc": (ctypes.c_int, [_i32, ctypes.c_size_t, ctypes.POINTER(_vp)]),
    "b200_ep_device_free": (ctypes.c_int, [_i32, _vp]),
    "b200_ep_copy": (ctypes.c_int, [_i32, _vp, _vp, ctypes.c_size_t, _vp]),
    "b200_ep_is_device_pointer": (ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    "b200_ep_stream_create": (ctypes.c_int, [_i32, ctypes.POINTER(_vp)]),
    "b200_ep_stream_sync": (ctypes.c_int, [_vp]),
    "b200_ep_stream_destroy": (ctypes.c_int, [_i32, _vp]),
    # include/b200_shard.h
    "b200_shard_gather_params_size": (ctypes.c_int, []),
    "b200_shard_gather": (ctypes.c_int, [ctypes.POINTER(ShardGatherParams), _vp]),
    "b200_ipc_handle_size": (ctypes.c_int, []),
    "b200_ipc_get_handle": (ctypes.c_int, [_vp, _vp]),
    "b200_ipc_open_handle": (ctypes.c_int, [_i32, _vp, ctypes.POINTER(_vp)]),
    "b200_ipc_close_handle": (ctypes.c_int, [_i32, _vp]),
}


class B200Error(RuntimeError):
    """A failing library call; ``code`` is the B200_ERR_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def library_file() -> str:
    return os.path.join(HERE, LIB_NAME)


def load() -> ctypes.CDLL:
    path = library_file()
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `make -C onnxruntime-ep-mlx_b200/csrc` "
            "(the B200 path has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.b200_params_size() != ctypes.sizeof(PagedAttentionParams):
        raise ImportError("libb200_paged.so: B200PagedAttentionParams layout differs from the binding")
    if lib.b200_node_info_size() != ctypes.sizeof(NodeInfo):
        raise ImportError("libb200_paged.so: B200NodeInfo layout differs from the binding")
    if lib.b200_gqa_params_size() != ctypes.sizeof(GqaParams):
        raise ImportError("libb200_paged.so: B200GqaParams layout differs from the binding")
    if lib.b200_gqa_node_info_size() != ctypes.sizeof(GqaNodeInfo):
        raise ImportError("libb200_paged.so: B200GqaNodeInfo layout differs from the binding")
    if lib.b200_shard_gather_params_size() != ctypes.sizeof(ShardGatherParams):
        raise ImportError("libb200_paged.so: B200ShardGatherParams layout differs from the binding")
    for which, cls in enumerate((EpOptions, KvPoolDesc, KvPoolInfo, PagedTensors)):
        if lib.b200_ep_struct_size(which) != ctypes.sizeof(cls):
            raise ImportError(f"libb200_paged.so: {cls.__name__} layout differs from the binding")
    return lib


LIB = load()


def check(code: int) -> None:
    if code != B200_OK:
        raise B200Error(code, LIB.b200_last_error().decode() or f"B200 status {code}")
