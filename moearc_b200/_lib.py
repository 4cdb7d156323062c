"""ctypes binding to libmoearc_b200.so — every symbol include/moearc.h declares.

The library is the product: there is no Python or CPU fallback. If the shared object is
missing this module raises, so a machine without the CUDA build fails loudly instead of
quietly running something else.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
# MOEARC_LIB selects another build of the same library (e.g. one compiled with timestamps).
LIB_PATH = os.environ.get("MOEARC_LIB") or os.path.join(PKG, "libmoearc_b200.so")

P = C.c_void_p
UL = C.c_ulong
U = C.c_uint
I = C.c_int
F = C.c_float

# name -> (restype, argtypes). Kept in the order of include/moearc.h.
SIGNATURES: dict[str, tuple] = {
    "moearc_ctx_create": (P, []),
    "moearc_ctx_destroy": (None, [P]),
    "moearc_profile_events_enabled": (I, [P]),
    "moearc_profile_events_reset": (I, [P]),
    "moearc_profile_events_report": (I, [P, C.c_char_p, UL]),
    "moearc_sync": (I, [P]),
    "moearc_zero": (I, [P, P, UL]),
    "moearc_device_name": (I, [P, C.c_char_p, UL]),
    "moearc_alloc_device": (P, [P, UL]),
    "moearc_free_device": (None, [P, P]),
    "moearc_copy_h2d": (I, [P, P, P, UL]),
    "moearc_copy_h2d_async": (I, [P, P, P, UL]),
    "moearc_copy_d2h": (I, [P, P, P, UL]),
    "moearc_gather_experts": (I, [P, P, P, P, U, UL]),
    "moearc_dequant": (I, [P, U, P, P, UL]),
    "moearc_matvec_q": (I, [P, U, P, P, P, UL, UL]),
    "moearc_matvec_q_batched": (I, [P, U, P, P, U, P, UL, UL, UL]),
    "moearc_moe_combine": (I, [P, P, P, P, U, UL]),
    "moearc_matvec_f32": (I, [P, P, P, P, UL, UL]),
    "moearc_rmsnorm": (I, [P, P, P, P, UL, UL, F]),
    "moearc_silu": (I, [P, P, P, UL]),
    "moearc_swiglu": (I, [P, P, P, P, UL]),
    "moearc_swiglu_halves": (I, [P, P, P, UL]),
    "moearc_swiglu_oai": (I, [P, P, P, P, UL, F, F]),
    "moearc_swiglu_oai_halves": (I, [P, P, P, UL, F, F]),
    "moearc_add_bias_id": (I, [P, P, P, P, U, UL]),
    "moearc_softmax": (I, [P, P, P, P, UL, UL, F]),
    "moearc_add": (I, [P, P, P, P, UL]),
    "moearc_mul": (I, [P, P, P, P, UL]),
    "moearc_axpy": (I, [P, P, P, F, UL]),
    "moearc_quantize_f16": (I, [P, P, P, UL]),
    "moearc_embed_rows": (I, [P, U, P, P, P, UL, UL]),
    "moearc_kv_append": (I, [P, P, P, P, P, U, U, UL, UL, UL, U]),
    "moearc_attn_decode": (I, [P, P, P, P, P, P, P, UL, UL, UL, UL, UL, UL, F, U]),
    "moearc_rope": (I, [P, P, P, P, UL, UL, UL, UL, F, F, F, F, F, F, I]),
    "moearc_topk_router": (I, [P, P, P, P, UL, UL, U, U]),
    "moearc_x_stream": (P, [P]),
    "moearc_x_timer_start": (I, [P]),
    "moearc_x_timer_stop": (I, [P, C.POINTER(F)]),
    "moearc_x_sm_count": (I, [P]),
    "moearc_x_quantize_bf16": (I, [P, P, P, UL]),
    "moearc_x_synth": (I, [P, P, UL, U, C.c_ulonglong, F, I, I]),
    "moearc_x_host_alloc": (P, [UL]),
    "moearc_x_host_free": (None, [P]),
    "moearc_x_copy_d2h_async": (I, [P, P, P, UL]),
    "moearc_x_moe_create": (P, [P, P]),
    "moearc_x_moe_destroy": (None, [P]),
    "moearc_x_moe_packed_bytes": (UL, [P, I]),
    "moearc_x_moe_pack": (I, [P, P, P, P, U, P, P]),
    "moearc_x_moe_forward": (I, [P, P, U, P, P, P, P, P, P]),
    "moearc_x_moe_buffer": (P, [P, I]),
    "moearc_x_moe_status": (I, [P]),
    "moearc_x_moe_set_wait": (I, [P, C.c_ulonglong, I]),
    "moearc_x_moe_set_bias": (I, [P, P, P]),
    "moearc_x_moe_tc_bytes": (UL, [P, I]),
    "moearc_x_ep_unique_id": (I, [P]),
    "moearc_x_ep_comm_init": (I, [P, P, I, P, I]),
    "moearc_x_ep_comm_destroy": (I, [P]),
    "moearc_x_ep_create": (P, [P, P, P, P, I, I, U]),
    "moearc_x_ep_destroy": (None, [P]),
    "moearc_x_ep_forward": (I, [P, P, U, P, P, P, P]),
    "moearc_x_ep_counts": (I, [P, P]),
    "moearc_x_ep_received": (U, [P]),
    "moearc_x_moe_has_tc": (I, [P]),
    "moearc_x_moe_pack_tc": (I, [P, P, P, P, U, P, P]),
    "moearc_x_moe_forward_tc": (I, [P, P, U, P, P, P, P, P, P]),
    "moearc_x_host_pool_create": (P, [I]),
    "moearc_x_host_pool_destroy": (None, [P]),
    "moearc_x_host_pool_threads": (I, [P]),
    "moearc_x_host_submit": (I, [P, P, P, P, P, P, U, P]),
    "moearc_x_host_sync": (I, [P, P]),
    "moearc_x_host_ffn": (I, [P, P, P, P, P, P, U, P, P]),
    "moearc_x_host_stats": (None, [P, P]),
    "moearc_x_moe_pack_host": (I, [P, P, P, P, U, P, P]),
    "moearc_x_prefill_create": (P, [P, P]),
    "moearc_x_prefill_destroy": (None, [P]),
    "moearc_x_prefill_set_bias": (I, [P, P, P]),
    "moearc_x_prefill_load8": (I, [P, P, P]),
    "moearc_x_prefill_load": (I, [P, P, P]),
    "moearc_x_prefill_forward": (I, [P, P, U, P, P, P, P]),
    "moearc_x_prefill_buffer": (P, [P, I]),
    "moearc_x_prefill_status": (I, [P]),
    "moearc_x_prefill_profile": (I, [P, P, U, P, P, P, P, P, I]),
    "moearc_x_prefill_load_range": (I, [P, P, P, U, U]),
    "moearc_x_prefill_route": (I, [P, P, U, P, P]),
    "moearc_x_prefill_experts": (I, [P, P, U, P, P, U, P, P]),
    "moearc_x_prefill_combine": (I, [P, P, U, P, P]),
    "moearc_x_prefill_load_list": (I, [P, P, P, P, U]),
    "moearc_x_decoder_uses_step_kernel": (I, [P]),
    "moearc_x_decoder_has_step_kernel": (I, [P]),
    "moearc_x_decoder_use_step_kernel": (I, [P, I]),
    "moearc_x_decoder_set_wait": (I, [P, C.c_ulonglong, U]),
    "moearc_x_decoder_trace_words": (C.c_ulong, [P]),
    "moearc_x_decoder_set_trace": (I, [P, P]),
    "moearc_x_batch_decoder_create": (P, [P, P, U]),
    "moearc_x_batch_decoder_create_ep": (P, [P, P, U, P, I, I]),
    "moearc_x_batch_decoder_destroy": (None, [P]),
    "moearc_x_batch_decoder_input": (P, [P]),
    "moearc_x_batch_decoder_output": (P, [P]),
    "moearc_x_batch_decoder_set_pos": (I, [P, U, I, C.c_ulonglong]),
    "moearc_x_batch_decoder_step": (I, [P]),
    "moearc_x_batch_decoder_status": (I, [P]),
    "moearc_x_batch_decoder_routing": (P, [P, U]),
    "moearc_x_prefill_set_order": (I, [P, P]),
    "moearc_x_prefill_load4": (I, [P, P, P]),
    "moearc_x_prefill_load4_list": (I, [P, P, P, P, U]),
    "moearc_x_prefill_route_begin": (I, [P, P, U, P, P]),
    "moearc_x_prefill_route_dispatch": (I, [P, P, P, U, U]),
    "moearc_x_prefill_experts_to": (I, [P, P, U, P, P, U, P, P]),
    "moearc_x_ipc_handle": (I, [P, P]),
    "moearc_x_ipc_open": (I, [P, P]),
    "moearc_x_ipc_close": (I, [P]),
    "moearc_x_decoder_create": (P, [P, P]),
    "moearc_x_decoder_destroy": (None, [P]),
    "moearc_x_decoder_input": (P, [P]),
    "moearc_x_decoder_output": (P, [P]),
    "moearc_x_decoder_logits": (P, [P]),
    "moearc_x_decoder_pos": (I, [P]),
    "moearc_x_decoder_set_pos": (I, [P, U]),
    "moearc_x_decoder_fill_kv": (I, [P, U, C.c_ulonglong]),
    "moearc_x_decoder_step": (I, [P]),
    "moearc_x_decoder_step_host": (I, [P, P, P]),
    "moearc_x_decoder_use_graph": (I, [P, I]),
    "moearc_x_decoder_kernel_spans": (I, [P, I]),
    "moearc_x_decoder_host_experts": (I, [P, I, F, U, I]),
    "moearc_x_decoder_host_stats": (I, [P, P]),
    "moearc_x_decoder_host_wait": (I, [P, C.c_ulonglong, I]),
    "moearc_x_decoder_status": (I, [P]),
    "moearc_x_decoder_fetched": (C.c_ulonglong, [P]),
    "moearc_x_decoder_profile": (I, [P, C.POINTER(F), C.POINTER(I), I]),
    "moearc_x_decoder_tensor": (P, [P, I, U, C.POINTER(UL)]),
    "moearc_x_decoder_seed": (C.c_ulonglong, [P, I, U, C.c_ulonglong]),
    "moearc_x_gguf_open": (P, [C.c_char_p]),
    "moearc_x_gguf_close": (None, [P]),
    "moearc_x_gguf_last_error": (C.c_char_p, []),
    "moearc_x_gguf_version": (U, [P]),
    "moearc_x_gguf_alignment": (C.c_ulonglong, [P]),
    "moearc_x_gguf_n_tensors": (C.c_ulonglong, [P]),
    "moearc_x_gguf_key_u64": (I, [P, C.c_char_p, C.POINTER(C.c_ulonglong)]),
    "moearc_x_gguf_key_f64": (I, [P, C.c_char_p, C.POINTER(C.c_double)]),
    "moearc_x_gguf_key_str": (I, [P, C.c_char_p, C.POINTER(C.c_char_p)]),
    "moearc_x_gguf_find": (I, [P, C.c_char_p, P]),
    "moearc_x_gguf_tensor_at": (I, [P, C.c_ulonglong, P, C.POINTER(C.c_char_p)]),
    "moearc_x_gguf_slice_last": (I, [P, C.c_char_p, C.c_ulonglong, P]),
    "moearc_x_mma_peak": (I, [P, I, I, C.POINTER(C.c_double)]),
    "moearc_x_attn_decode_static": (I, [P, P, P, P, P, P, P, UL, UL, UL, UL, UL, UL, F, U]),
}


class GgufTensor(C.Structure):
    """moearc_x_gguf_tensor (include/moearc.h)."""
    _fields_ = [("n_dims", U), ("dims", C.c_ulonglong * 4), ("type_id", U), ("offset", C.c_ulonglong),
                ("nbytes", C.c_ulonglong), ("data", P)]


class DecoderCfg(C.Structure):
    """moearc_x_decoder_cfg (include/moearc.h)."""
    _fields_ = [("n_layer", U), ("n_embd", U), ("n_head", U), ("n_head_kv", U), ("head_dim", U),
                ("n_expert", U), ("n_expert_used", U), ("n_ff", U), ("expert_type", U), ("gating", U),
                ("act", U), ("alpha", F), ("limit", F), ("n_swa", U), ("swa_pattern", U),
                ("rope_base", F), ("rope_freq_scale", F), ("rope_ext_factor", F), ("rope_attn_factor", F),
                ("rope_corr_lo", F), ("rope_corr_hi", F), ("rms_eps", F), ("has_sinks", U), ("n_ctx", U),
                ("seed", C.c_ulonglong), ("n_offload", U), ("n_cache", U), ("has_qk_norm", U), ("n_vocab", U),
                ("expert_layout", U)]


class MoeDesc(C.Structure):
    """moearc_x_moe_desc (include/moearc.h)."""
    _fields_ = [("n_embd", U), ("n_ff", U), ("n_expert", U), ("k", U), ("gating", U), ("act", U),
                ("alpha", F), ("limit", F), ("wtype", U), ("max_tokens", U)]

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load the shared library once and declare every signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m moearc_b200.build` "
            "(there is no fallback implementation)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declare(name: str, restype, argtypes) -> None:
    """Register one more signature (used by modules that add extension entry points)."""
    SIGNATURES[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
