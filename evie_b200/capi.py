"""ctypes declarations of every entry point in include/evie_cuda.h."""
from __future__ import annotations

import ctypes as C


class Seq(C.Structure):
    """evie_seq"""
    _fields_ = [("slot", C.c_int32), ("pos0", C.c_int32), ("tokens", C.c_void_p), ("n_tokens", C.c_int32)]


class Op(C.Structure):
    """evie_op"""
    _fields_ = [("layer", C.c_int32), ("neuron", C.c_int32), ("mode", C.c_int32), ("value", C.c_float)]


class PlanOp(C.Structure):
    """evie_plan_op"""
    _fields_ = [("layer", C.c_int32), ("neuron", C.c_int32), ("mode", C.c_int32), ("value", C.c_float),
                ("gate", C.c_int32)]


class Detector(C.Structure):
    """evie_detector"""
    _fields_ = [("gate", C.c_int32), ("layer", C.c_int32), ("neuron", C.c_int32), ("weight", C.c_float)]


class SampleParams(C.Structure):
    """evie_sample_params"""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("min_p", C.c_float),
                ("repetition_penalty", C.c_float), ("seed", C.c_uint64)]


class ModelInfo(C.Structure):
    """evie_model_info"""
    _fields_ = [
        ("hidden", C.c_int32), ("intermediate", C.c_int32), ("n_layers", C.c_int32), ("vocab", C.c_int32),
        ("n_linear_layers", C.c_int32), ("n_full_layers", C.c_int32), ("slots", C.c_int32), ("max_ctx", C.c_int32),
        ("max_rows", C.c_int32), ("max_ops", C.c_int32), ("weight_bytes", C.c_int64), ("cache_bytes", C.c_int64),
    ]


P, I, F, SZ = C.c_void_p, C.c_int, C.c_float, C.c_size_t

SIGNATURES = {
    "evie_create": (I, [C.c_char_p, I, I, I, I, C.POINTER(P)]),
    "evie_destroy": (None, [P]),
    "evie_last_error": (C.c_char_p, [P]),
    "evie_last_global_error": (C.c_char_p, []),
    "evie_info": (I, [P, C.POINTER(ModelInfo)]),
    "evie_forward": (I, [P, P, I, I, I, P, P, P, P]),
    "evie_decode_greedy": (I, [P, P, I, I, P, I, P, P]),
    "evie_stream": (P, [P]),
    "evie_profile": (I, [P, I]),
    "evie_profile_read": (I, [P, I, C.POINTER(C.c_char_p), C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "evie_set_ops": (I, [P, I, P, I]),
    "evie_set_plan": (I, [P, I, P, I, P, I, P, I]),
    "evie_gate_state": (I, [P, I, P, P, I]),
    "evie_reset_gates": (I, [P, I]),
    "evie_set_sampler": (I, [P, I, P]),
    "evie_read_top_active": (I, [P, I, P, P]),
    "evie_neuron_sigma": (I, [P, P, SZ, P, P]),
    "evie_set_lens": (I, [P, P, I, I, I]),
    "evie_clear_lens": (I, [P]),
    "evie_lens_logits": (I, [P, I, P, I, P]),
    "evie_neuron_logits": (I, [P, P, P, I, P]),
    "evie_search_scores": (I, [P, P, I, P, P, P, P]),
    "evie_top_active": (I, [P, I, C.c_longlong, I, P, P]),
    "evie_sampler_seed_state": (C.c_uint64, [C.c_uint64]),
    "evie_sample": (I, [P, I, I, P, P, P, P, P, P]),
    "evie_reset_slot": (I, [P, I]),
    "evie_set_scale": (I, [P, P, SZ]),
    "evie_track_max": (I, [P, I]),
    "evie_read_max": (I, [P, P, SZ]),
    "evie_gdn_decode_step": (I, [P, P, P, P, P, P, P, I, I, I, I, P]),
    "evie_gdn_chunk_prefill": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, P]),
    "evie_gdn_prefill_tokenwise": (I, [P, P, P, P, P, P, P, I, I, I, I, I, P]),
    "evie_proj_gemm": (I, [P, P, P, SZ, I, I, I, I, P, P]),
    "evie_poll_device_errors": (I, []),
    "evie_bounded_wait_probe": (I, [C.c_uint64, P]),
    "evie_gqa_decode_paged": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, F, P]),
    "evie_gqa_prefill_paged": (I, [P, P, P, P, I, P, I, P, P, I, P, I, I, I, I, F, P]),
    "evie_gqa_decode_paged_noalloc": (I, [P, P, P, P, P, P, P, I, I, I, I, I, I, F, P]),
}


def declare(L) -> None:
    """Sets restype/argtypes for every exported function that the library has."""
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name, None)
        if f is None:
            continue
        f.restype = res
        f.argtypes = args


def header_functions(header_path: str) -> list:
    """Names of every function the C header declares (used to check that the library exports all of them)."""
    import re

    with open(header_path) as f:
        text = f.read()
    return sorted(set(re.findall(r"EVIE_API\s+[\w\s\*]+?\b(evie_\w+)\s*\(", text)))
