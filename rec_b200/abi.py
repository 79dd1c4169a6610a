"""ctypes mirror of include/rec_b200.h (structures and constants)."""
from __future__ import annotations

import ctypes as C

REC_OK = 0
REC_EINVAL = -1
REC_ECUDA = -2
REC_ESTATE = -3
REC_ELIMIT = -4
REC_DEV_BULK_TIMEOUT = 1
REC_DEV_COUNTER_TIMEOUT = 2
REC_DEV_BAD_TOKEN = 3
REC_DEV_BAD_POSITION = 4

REC_SCALE_FP16 = 0
REC_SCALE_BF16 = 1
REC_ROUTER_SOFTMAX = 0
REC_ROUTER_SIGMOID = 1
REC_FLAG_SINKS = 1
REC_FLAG_QK_NORM = 2
# layer kinds (RecLayerWeights.kind bits)
REC_LAYER_DENSE = 1
REC_LAYER_NO_ROPE = 2
REC_LAYER_SLIDING = 4


class RecModelDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32),
        ("n_layers", C.c_int32),
        ("n_q_heads", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("n_experts", C.c_int32),
        ("top_k", C.c_int32),
        ("moe_inter", C.c_int32),
        ("vocab", C.c_int32),
        ("group_size", C.c_int32),
        ("scale_dtype", C.c_int32),
        ("kv_bits", C.c_int32),
        ("router_mode", C.c_int32),
        ("flags", C.c_int32),
        ("rms_eps", C.c_float),
        ("rope_theta", C.c_float),
        ("shared_inter", C.c_int32),
        ("dense_inter", C.c_int32),
        ("sliding_window", C.c_int32),
        ("embed_bits", C.c_int32),
        ("kv_value_bits", C.c_int32),
    ]


class RecQMat(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p)]


class RecLayerWeights(C.Structure):
    _fields_ = [
        ("input_norm", C.c_void_p),
        ("post_norm", C.c_void_p),
        ("q", RecQMat),
        ("k", RecQMat),
        ("v", RecQMat),
        ("o", RecQMat),
        ("router", C.c_void_p),
        ("expert_bias", C.c_void_p),
        ("gate", RecQMat),
        ("up", RecQMat),
        ("down", RecQMat),
        ("sinks", C.c_void_p),
        ("q_norm", C.c_void_p),
        ("k_norm", C.c_void_p),
        ("kind", C.c_int32),
        ("shared_gate", RecQMat),
        ("shared_up", RecQMat),
        ("shared_down", RecQMat),
    ]


class RecGlobalWeights(C.Structure):
    _fields_ = [("embed", RecQMat), ("final_norm", C.c_void_p), ("lm_head", RecQMat)]


class RecKVLayer(C.Structure):
    _fields_ = [
        ("k_codes", C.c_void_p),
        ("k_scales", C.c_void_p),
        ("k_biases", C.c_void_p),
        ("v_codes", C.c_void_p),
        ("v_scales", C.c_void_p),
        ("v_biases", C.c_void_p),
    ]


class RecSampling(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_int32),
        ("top_p", C.c_float),
        ("repetition_penalty", C.c_float),
        ("presence_penalty", C.c_float),
    ]


class RecShard(C.Structure):
    _fields_ = [
        ("world", C.c_int32),
        ("rank", C.c_int32),
        ("expert_lo", C.c_int32),
        ("expert_hi", C.c_int32),
        ("super_lo", C.c_int32),
        ("super_hi", C.c_int32),
        ("capacity_total", C.c_int32),
        ("exchange", C.c_void_p * 8),
        ("schedule", C.c_int32),
    ]
