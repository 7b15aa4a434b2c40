"""ctypes binding of libsvla.so (include/svla.h).

The library is built in-tree (``python -m smolvla_mujoco_libero_b200.build``) and loaded from the package
directory.  There is no fallback: if the library is missing or fails to load, every call raises.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsvla.so"

KIND_I8, KIND_BF16, KIND_W8A16 = 0, 1, 2
EPI_BF16, EPI_I32, EPI_ROPE, EPI_RESID, EPI_SILU_MUL, EPI_GELU_QUANT, EPI_EULER, EPI_SILU, EPI_F32 = range(9)
ATTN_AUTO, ATTN_MMA_SYNC, ATTN_TCGEN05 = range(3)


class GemmSeg(ctypes.Structure):
    _fields_ = [
        ("a", c_void_p), ("lda", c_int32), ("b", c_void_p), ("ldb", c_int32), ("wscale", c_void_p),
        ("bias", c_void_p), ("bias_f32", c_void_p), ("out", c_void_p), ("ldo", c_int32), ("n", c_int32),
        ("act_scale", c_float), ("rope", c_int32),
    ]


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("kind", c_int32), ("epi", c_int32), ("m", c_int32), ("k", c_int32), ("nseg", c_int32), ("pair", c_int32),
        ("seg", GemmSeg * 3), ("block_n", c_int32), ("rows_per_group", c_int32), ("group_stride", c_int32),
        ("row_offset", c_int32), ("post_scale", c_float), ("resid", c_void_p), ("ldr", c_int32),
        ("resid_rows", c_int32), ("rope_cs", c_void_p), ("pos", c_void_p), ("max_pos", c_int32),
        ("q_smooth", c_void_p), ("q_rsmooth", c_void_p), ("q_act", c_float), ("qout", c_void_p), ("ldq", c_int32), ("dt", c_float),
        ("xt", c_void_p), ("xt_bf16", c_void_p), ("debug_clock", c_void_p), ("weights_resident", c_int32),
        ("split_k", c_int32), ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("cta_pair", c_int32),
    ]


SPLITK_COUNTER_BYTES = 65536  # SVLA_SPLITK_COUNTER_BYTES


class NormDesc(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("ldx", c_int32), ("weight", c_void_p), ("bias", c_void_p), ("eps", c_float),
        ("layernorm", c_int32), ("m", c_int32), ("k", c_int32), ("y", c_void_p), ("ldy", c_int32), ("nq", c_int32),
        ("q", c_void_p * 3), ("ldq", c_int32), ("smooth", c_void_p * 3), ("rsmooth", c_void_p * 3), ("act", c_float * 3),
        ("pixel_shuffle", c_int32), ("ps_grid", c_int32),
    ]


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_bs", c_int64), ("q_rs", c_int32),
        ("k1", c_void_p), ("v1", c_void_p), ("kv1_bs", c_int64), ("kv1_rs", c_int32), ("l1", c_int32),
        ("k2", c_void_p), ("v2", c_void_p), ("kv2_bs", c_int64), ("kv2_rs", c_int32), ("l2", c_int32),
        ("mask", c_void_p), ("mask_bs", c_int64), ("mask_rs", c_int32),
        ("o", c_void_p), ("o_bs", c_int64), ("o_rs", c_int32),
        ("qo", c_void_p), ("qo_bs", c_int64), ("qo_rs", c_int32),
        ("qo_smooth", c_void_p), ("qo_rsmooth", c_void_p), ("qo_act", c_float),
        ("batch", c_int32), ("lq", c_int32), ("hq", c_int32), ("hkv", c_int32), ("scale", c_float),
        ("impl", c_int32), ("debug_clock", c_void_p),
        ("key_mask", c_void_p), ("key_mask_bs", c_int64), ("mask_keys", c_int32),
    ]


FLOW_MAX_LAYERS, FLOW_MAX_ROWS = 32, 64
ERR_MBAR_TIMEOUT, ERR_BAD_SHAPE, ERR_FLOW_BARRIER = 101, 102, 103  # device error word codes


class FlowLayer(ctypes.Structure):
    _fields_ = [
        ("input_norm", c_void_p), ("post_norm", c_void_p), ("wq", c_void_p), ("sq", c_void_p), ("wk", c_void_p),
        ("sk", c_void_p), ("wv", c_void_p), ("sv", c_void_p), ("wo", c_void_p), ("so", c_void_p), ("wg", c_void_p),
        ("sg", c_void_p), ("wu", c_void_p), ("su", c_void_p), ("wd", c_void_p), ("sd", c_void_p),
        ("keys", c_void_p), ("values", c_void_p), ("cross", c_int32),
    ]


class FlowDesc(ctypes.Structure):
    _fields_ = [
        ("batch", c_int32), ("chunk", c_int32), ("prefix_len", c_int32), ("hidden", c_int32), ("action_dim", c_int32),
        ("heads", c_int32), ("kv_heads", c_int32), ("mlp", c_int32), ("n_layers", c_int32), ("num_steps", c_int32),
        ("eps", c_float), ("noise", c_void_p), ("xt", c_void_p), ("xt_bf16", c_void_p),
        ("w_action_in", c_void_p), ("b_action_in", c_void_p), ("w_time_in", c_void_p),
        ("time_in_const", c_void_p), ("w_time_out", c_void_p), ("b_time_out", c_void_p), ("final_norm", c_void_p),
        ("w_action_out", c_void_p), ("b_action_out", c_void_p), ("key_mask", c_void_p), ("key_mask_bs", c_int64),
        ("suffix_pos", c_void_p), ("cross_pos", c_void_p), ("rope_cs", c_void_p), ("max_pos", c_int32),
        ("a_emb", c_void_p), ("a_t", c_void_p), ("eh", c_void_p), ("eq", c_void_p), ("ek", c_void_p), ("ev", c_void_p),
        ("ectx", c_void_p), ("emlp", c_void_p), ("norm_part", c_void_p), ("sync", c_void_p), ("spin_limit", ctypes.c_uint32),
        ("debug_clock", c_void_p),
        ("layer", FlowLayer * FLOW_MAX_LAYERS),
    ]


class EngineInfo(ctypes.Structure):
    _fields_ = [
        ("n_cams", c_int32), ("channels", c_int32), ("image_size", c_int32), ("n_lang", c_int32),
        ("max_state_dim", c_int32), ("max_action_dim", c_int32), ("chunk", c_int32), ("num_steps", c_int32),
        ("action_dim", c_int32), ("prefix_len", c_int32), ("vis_layers", c_int32), ("text_layers", c_int32),
        ("expert_layers", c_int32), ("n_linears", c_int32), ("n_tensors", c_int32), ("launches_per_call", c_int32),
        ("max_batch", c_int32), ("weight_bytes", c_int64), ("buffer_bytes", c_int64),
    ]


ENGINE_NO_GRAPH, ENGINE_NO_SPLIT_K, ENGINE_NO_FLOW = 1, 2, 4  # SVLA_ENGINE_* flags

# SVLA_DT_*: TensorRT's nvinfer1::DataType numbering
DT_FLOAT, DT_HALF, DT_INT32, DT_BF16, DT_INT64 = 0, 1, 3, 7, 8


class RopeParams(ctypes.Structure):
    _fields_ = [("q_heads", c_int32), ("kv_heads", c_int32), ("head_dim", c_int32), ("max_wavelength", c_float)]

# name -> (restype, argtypes) for every symbol in include/svla.h
SIGNATURES = {
    "svla_last_error": (c_char_p, []),
    "svla_version": (c_char_p, []),
    "svla_device_error": (c_int32, [POINTER(c_int32), c_int32]),
    "svla_pack_weight_i8": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "svla_dequant_weight_bf16": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "svla_quantize_smooth": (c_int32, [c_void_p, c_int32, c_void_p, c_float, c_void_p, c_int32, c_int32, c_int32,
                                       c_void_p]),
    "svla_channel_percentile": (c_int32, [c_void_p, c_int64, c_int32, c_int32, c_int32, c_float, c_void_p, c_void_p,
                                          c_void_p]),
    "svla_gemm_i8_i32": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "svla_sq_linear_w8a8_workspace_size": (c_size_t, [c_int32, c_int32]),
    "svla_sq_linear_w8a8": (c_int32, [c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                      c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    "svla_sq_linear_w8a8_static_scratch": (c_int32, [c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                                     c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "svla_w8a16_linear": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
                                    c_void_p]),
    "svla_gemm": (c_int32, [POINTER(GemmDesc), c_void_p]),
    "svla_norm_quant": (c_int32, [POINTER(NormDesc), c_void_p]),
    "svla_attention": (c_int32, [POINTER(AttnDesc), c_void_p]),
    "svla_rope_layout": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                   c_int32, c_float, c_void_p]),
    "svla_fused_rope_layout": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                         POINTER(RopeParams), c_int32, c_int32, c_void_p]),
    "svla_fused_rope_attention": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
                                            c_int32, POINTER(RopeParams), c_int32, c_int32, c_void_p]),
    "svla_fused_rope_attention_f32_mask_implicit_pos": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                                                  c_int32, c_int32, POINTER(RopeParams), c_void_p]),
    "svla_resize_pad_images": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64,
                                         c_int32, c_int32, c_float, c_void_p]),
    "svla_normalize_state": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int32, c_int32,
                                       c_void_p, c_void_p]),
    "svla_unnormalize_actions": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int32, c_void_p,
                                           c_void_p]),
    "svla_rope_table": (c_int32, [c_void_p, c_int32, c_float, c_void_p]),
    "svla_build_masks": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "svla_embed_tokens": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32, c_float, c_void_p,
                                    c_int32, c_int32, c_void_p]),
    "svla_im2col": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "svla_f32_to_bf16": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p]),
    "svla_euler_init": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "svla_reciprocal": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p]),
    "svla_flow_packed_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "svla_flow_pack_weight": (c_int32, [c_void_p, c_int32, c_int64, c_int32, c_int32, c_void_p, c_void_p]),
    "svla_flow": (c_int32, [POINTER(FlowDesc), c_void_p]),
    "svla_engine_inspect": (c_int32, [c_char_p, POINTER(EngineInfo)]),
    "svla_engine_create": (c_int32, [c_char_p, c_int32, c_int32, c_void_p, POINTER(c_void_p)]),
    "svla_engine_get_info": (c_int32, [c_void_p, POINTER(EngineInfo)]),
    "svla_engine_sample_actions": (c_int32, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_void_p,
                                             c_int32, c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p]),
    "svla_engine_destroy": (c_int32, [c_void_p]),
}


class SvlaError(RuntimeError):
    pass


_lib = None


def lib() -> ctypes.CDLL:
    """Load libsvla.so once; raise if it is missing (there is no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise SvlaError(f"{LIB_PATH} is missing: build it with `python -m smolvla_mujoco_libero_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().svla_last_error().decode(errors="replace")
        kind = {1: "bad argument", 2: "CUDA error"}.get(rc, f"status {rc}")
        raise SvlaError(f"{what or 'svla'}: {kind}: {msg}")


def device_error(reset: bool = True) -> int:
    code = c_int32(0)
    check(lib().svla_device_error(ctypes.byref(code), 1 if reset else 0), "svla_device_error")
    return int(code.value)
