"""ctypes binding of ``libmagpie_tts_rt_b200.so`` (declared in
``include/magpie_tts_rt_b200.h``).

There is no fallback: if the shared library is missing or does not export a
declared symbol, importing this module raises.  Build it with
``python -m magpie_tts_rt_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "libmagpie_tts_rt_b200.so")

P = ctypes.c_void_p
I32 = ctypes.c_int32
I64 = ctypes.c_int64
SZ = ctypes.c_size_t

MTT_PLUGIN_ABI_VERSION_1 = 1
MTT_PLUGIN_CREATOR_COUNT_V1 = 5
STATUS_OK = 0
STATUS_INVALID_ARGUMENT = -1
STATUS_CUDA_ERROR = -2


class PluginCreatorV1(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("name", ctypes.c_char * 64),
        ("version", ctypes.c_char * 16),
        ("plugin_namespace", ctypes.c_char * 64),
    ]


class PluginApiV1(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("abi_version", ctypes.c_uint32),
        ("creator_count", ctypes.c_uint32),
        ("reserved_0", ctypes.c_uint32),
        ("creators", PluginCreatorV1 * MTT_PLUGIN_CREATOR_COUNT_V1),
        ("register_plugins", ctypes.CFUNCTYPE(ctypes.c_int32)),
        ("reserved", ctypes.c_uint64 * 4),
    ]


class MainDevicePositionClassV1(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
        ("operation", ctypes.c_uint32), ("class_index", ctypes.c_uint32),
        ("parameter_transport", ctypes.c_uint32), ("block_x", ctypes.c_uint32),
        ("block_y", ctypes.c_uint32), ("block_z", ctypes.c_uint32),
        ("shared_memory_bytes", ctypes.c_uint32), ("reserved_0", ctypes.c_uint32),
        ("parameter_offset", ctypes.c_uint64), ("parameter_size", ctypes.c_uint64),
        ("function_name", ctypes.c_char * 256), ("reserved", ctypes.c_uint64 * 4),
    ]


class MainDevicePositionKV1(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
        ("active_k", ctypes.c_int32), ("qk_class_index", ctypes.c_int32),
        ("qk_grid_x", ctypes.c_uint32), ("qk_grid_y", ctypes.c_uint32),
        ("qk_grid_z", ctypes.c_uint32), ("pv_class_index", ctypes.c_int32),
        ("pv_grid_x", ctypes.c_uint32), ("pv_grid_y", ctypes.c_uint32),
        ("pv_grid_z", ctypes.c_uint32), ("reserved_0", ctypes.c_uint32),
        ("reserved", ctypes.c_uint64 * 4),
    ]


class MainDevicePositionClassTableV1(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
        ("class_count", ctypes.c_uint32), ("k_count", ctypes.c_uint32),
        ("classes", MainDevicePositionClassV1 * 21),
        ("k_records", MainDevicePositionKV1 * 249),
        ("reserved", ctypes.c_uint64 * 4),
    ]


class Shape(ctypes.Structure):
    _fields_ = [("d_model", I32), ("n_layers", I32), ("n_heads", I32), ("d_ffn", I32)]


class Weights(ctypes.Structure):
    _fields_ = [(n, P) for n in (
        "in_proj_w", "in_proj_b", "pos", "ln_self", "qkv", "o", "ln_ff", "ffn1", "ffn2",
        "head_w", "head_b", "emb", "final_w", "final_b", "emb_proj")]


class SamplingConfig(ctypes.Structure):
    _fields_ = [("top_k", I32), ("temperature", ctypes.c_float), ("cfg_scale", ctypes.c_float),
                ("argmax", I32), ("cfg", I32), ("path", I32)]


PATH_AUTO = 0
PATH_PHASE_KERNELS = 1
PATH_FUSED_CLUSTER = 2
PATH_FUSED_TILE = 3
PATH_FUSED_PAIR = 4
PATH_SPLIT_1 = 5
PATH_SPLIT_2 = 6
PATH_SPLIT_4 = 7
PATH_SPLIT_8 = 8
PATH_SPLIT_2X32 = 9
PATH_QUAD = 10
PATH_OCTO = 11


class StreamBatch(ctypes.Structure):
    _fields_ = [
        ("n_streams", I32), ("reserved_0", I32),
        ("decoder_hidden", P), ("unfinished", P), ("finished", P), ("forbid_eos", P),
        ("active", P), ("rng_seed", P), ("rng_counter", P), ("codec_tokens", P),
        ("invalid_rows", P), ("end_frame_index", P), ("next_embedding", P),
        ("forced_tokens", P), ("logits_out", P),
        ("codec_frames_stride", I32), ("codec_frame_offset", I32), ("finished_latch", P),
        ("codec_frames", P), ("eos_projection", P),
    ]


class AlignmentContract(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "text_length", "ignored_terminal_tokens", "short_text_no_prior_max_tokens", "lookahead",
        "sink_threshold")]


class AlignmentBatch(ctypes.Structure):
    _fields_ = [
        ("n_sessions", I32), ("token_stride", ctypes.c_uint32),
        ("ignored_terminal_tokens", ctypes.c_uint32), ("short_text_no_prior_max_tokens", ctypes.c_uint32),
        ("lookahead", ctypes.c_uint32), ("sink_threshold", ctypes.c_uint32),
        ("text_length", P), ("active", P), ("alignment_scores", P), ("counters", P),
        ("last_attended", P), ("next_prior", P), ("attended_token_index", P), ("unfinished", P),
        ("invalid_state", P), ("decoder_steps", P), ("forbid_eos", P), ("end_frame_index", P),
        ("finished", P),
    ]


class MainDecoderWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in ("pos", "ln_self", "qkv", "o", "ln_xq", "xq", "xo", "ln_ff", "ffn1", "ffn2",
                                 "norm_out")] + [("n_layers", I32), ("pos_rows", I32), ("final_w", P),
                                                 ("final_b", P)]


class MainDecoderBatch(ctypes.Structure):
    _fields_ = [
        ("n_sessions", I32), ("cache_capacity", I32), ("token_stride", I32), ("reserved_0", I32),
        ("embedded", P), ("position", P), ("text_length", P), ("active", P), ("self_k", P), ("self_v", P),
        ("self_mask", P), ("cross_k", P), ("cross_v", P), ("cond_mask", P), ("prior", P), ("hidden", P),
        ("alignment", P), ("status", P), ("eos_projection", P), ("eos_cfg_scale", ctypes.c_float),
        ("reserved_1", I32),
    ]


class SessionEngineConfig(ctypes.Structure):
    _fields_ = [
        ("max_sessions", I32), ("token_stride", I32), ("with_decoder", I32), ("cache_capacity", I32),
        ("ignored_terminal_tokens", ctypes.c_uint32), ("short_text_no_prior_max_tokens", ctypes.c_uint32),
        ("lookahead", ctypes.c_uint32), ("sink_threshold", ctypes.c_uint32),
        ("shape", Shape), ("local_ar", Weights), ("sampling", SamplingConfig), ("decoder", MainDecoderWeights),
        ("decoder_hidden", P), ("alignment_scores", P), ("next_embedding", P),
    ]


class SessionEngineBuffers(ctypes.Structure):
    _fields_ = [(n, P) for n in ("stream", "decoder_hidden", "alignment_scores", "next_embedding", "codec_tokens",
                                 "end_frame_index", "invalid_rows", "rng_counter", "finished", "position",
                                 "decoder_status")]


# name -> (restype, argtypes)
SIGNATURES = {
    "mtt_plugin_get_api_v1": (I32, [ctypes.POINTER(PluginApiV1)]),
    "mtt_plugin_get_main_device_position_class_table_v1": (
        I32, [ctypes.POINTER(MainDevicePositionClassTableV1)]),
    "mtt_b200_launch_local_ar_sampling": (I32, [P] * 11 + [P]),
    "mtt_b200_local_ar_eos_workspace_size": (SZ, []),
    "mtt_b200_launch_local_ar_eos": (I32, [P] * 9 + [P]),
    "mtt_b200_launch_finalize_local_step": (
        I32, [P, P, ctypes.c_uint32, P, P, P, P, P, P, P, P]),
    "mtt_b200_launch_layer_norm": (I32, [P, P, P, I32, P]),
    "mtt_b200_launch_gelu_tanh": (I32, [P, P, SZ, P]),
    "mtt_b200_launch_softmax": (I32, [P, P, I32, I32, P]),
    "mtt_b200_local_ar_frame_workspace_size": (SZ, [ctypes.POINTER(Shape), I32, I32]),
    "mtt_b200_launch_local_ar_frame": (
        I32, [ctypes.POINTER(Shape), ctypes.POINTER(Weights), ctypes.POINTER(SamplingConfig),
              ctypes.POINTER(StreamBatch), P, SZ, P]),
    "mtt_b200_local_ar_frame_launch_count": (
        I32, [ctypes.POINTER(Shape), ctypes.POINTER(SamplingConfig), I32]),
    "mtt_b200_local_ar_frame_path": (I32, [ctypes.POINTER(Shape), ctypes.POINTER(SamplingConfig), I32]),
    "mtt_b200_local_ar_frame_path_clusters": (I32, [I32]),
    "mtt_b200_fold_in_projection_bytes": (SZ, [ctypes.POINTER(Shape)]),
    "mtt_b200_launch_fold_in_projection": (
        I32, [ctypes.POINTER(Shape), ctypes.POINTER(Weights), P, P]),
    "mtt_b200_launch_alignment_controller": (
        I32, [P, ctypes.POINTER(AlignmentContract), P, P, P, P, P, P, P]),
    "mtt_b200_launch_alignment_batch": (I32, [ctypes.POINTER(AlignmentBatch), P]),
    "mtt_b200_main_decoder_workspace_size": (SZ, [I32, I32]),
    "mtt_b200_launch_main_decoder_step": (
        I32, [ctypes.POINTER(MainDecoderWeights), ctypes.POINTER(MainDecoderBatch), P, SZ, P]),
    "mtt_b200_launch_test_clamped_gumbel": (I32, [P, P, SZ, P]),
    "mtt_b200_launch_test_log": (I32, [P, P, SZ, P]),
    "mtt_b200_launch_test_gemm": (I32, [P, P, P, I32, I32, I32, I32, I32, P, P]),
    "mtt_b200_test_umma_cycles": (I32, [I32, I32, I32, I32, P, P]),
    "mtt_b200_test_dsmem_cycles": (I32, [I32, I32, I32, P, P]),
    "mtt_b200_test_frame_trace": (I32, [P]),
    "mtt_b200_session_engine_create": (I32, [ctypes.POINTER(SessionEngineConfig), ctypes.POINTER(P)]),
    "mtt_b200_session_engine_destroy": (None, [P]),
    "mtt_b200_session_engine_buffers": (I32, [P, ctypes.POINTER(SessionEngineBuffers)]),
    "mtt_b200_session_engine_open": (I32, [P, I32, ctypes.c_int64, ctypes.c_uint32, P, P, P, P]),
    "mtt_b200_session_engine_close": (I32, [P, I32]),
    "mtt_b200_session_engine_step": (I32, [P]),
    "mtt_b200_session_engine_collect": (I32, [P, I32, P, P, P]),
}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIBRARY):
        raise ImportError(
            f"{LIBRARY} is missing: build it with `python -m magpie_tts_rt_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIBRARY)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if not exported
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
