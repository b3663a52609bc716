"""ctypes prototypes of every symbol declared in include/jimotono_b200.h.

PROTOTYPES is also the list the CPU test suite checks against the header and
the library's dynamic symbol table."""
from __future__ import annotations

import ctypes as C

P = C.c_void_p
I = C.c_int
SZ = C.c_size_t
F = C.c_float
D = C.c_double

# name: (restype, [argtypes])
PROTOTYPES = {
    # ---- reference-compatible W8A8 (w8a8.h) ----
    "jt_w8a8_set_enabled": (I, [I]),
    "jt_w8a8_get_enabled": (I, [P]),
    "jt_w8a8_is_enabled": (I, []),
    "jt_w8a8_quant_per_tensor": (I, [P, SZ, P, P]),
    "jt_w8a8_dequant_per_tensor": (I, [P, F, SZ, P]),
    "jt_w8a8_quant_per_channel": (I, [P, SZ, SZ, P, P]),
    "jt_w8a8_dequant_per_channel": (I, [P, P, SZ, SZ, P]),
    "jt_w8a8_gemm_per_tensor": (I, [P, P, F, F, P, I, I, I]),
    "jt_w8a8_gemm_per_channel": (I, [P, P, F, P, P, I, I, I]),
    "jt_w8a8_fakequant_per_tensor": (I, [P, SZ, P]),
    "jt_w8a8_fakequant_per_channel": (I, [P, SZ, SZ, P]),
    # ---- device entry points ----
    "jt_routing_topk": (I, [P, SZ, SZ, P, P]),
    "jt_moe_batch_sort": (I, [P, I, I, I, F, P, P, P, P, P]),
    "jt_gemm_mat_f32": (I, [P, P, P, I, I, I]),
    "jt_transpose_f32": (I, [P, P, I, I]),
    "jt_lowbit_set_mode": (I, [I]),
    "jt_lowbit_get_mode": (I, []),
    "jt_lowbit_bits_for": (I, [I, P]),
    "jt_lowbit_fakequant": (I, [P, P, SZ, I]),
    "jt_lowbit_col_to_idx": (I, [P, SZ, I, P, P]),
    "jt_lowbit_gemm_lut": (I, [P, P, P, I, I, I, I]),
    "jt_moe_fwd_batch": (I, [P] * 9 + [I] * 6 + [P] * 7 + [F] + [P] * 5),
    "jt_moe_fwd_batch_unchecked": (I, [P] * 9 + [I] * 6 + [P] * 7 + [F] + [P] * 5),
    "jt_moe_fwd": (I, [P] * 9 + [I] * 5 + [P] * 8),
    "jt_moe_fwd_unchecked": (I, [P] * 9 + [I] * 5 + [P] * 8),
    "jt_tmac_qlut_bytes": (I, [SZ, SZ, P]),
    "jt_tmac_param_bytes": (I, [SZ, SZ, P]),
    "jt_tmac_lut_ctor": (I, [P, SZ, SZ, P, P, P]),
    "jt_tmac_lookup_accum": (I, [P, P, P, P, SZ, SZ, I, F, P]),
    "jt_b200_w8a8_gemm": (I, [P, I, P, P, I, P, P, I, I, I, I, P]),
    "jt_b200_w8a8_gemm_i32": (I, [P, I, P, I, P, I, I, I, I, P]),
    "jt_b200_w8a8_linear_noalloc": (I, [P, I, I, P, I, P, P, I, I, P]),
    "jt_b200_lowbit_gemv": (I, [P, F, P, P, I, P, P, I, I, P, P]),
    "jt_b200_lowbit_pack": (I, [P, I, I, I, I, P, P, P]),
    "jt_b200_lowbit_planes_to_packed": (I, [P, P, I, I, I, I, P, P, P]),
    "jt_b200_moe_plan_create": (I, [P, P]),
    "jt_b200_moe_plan_destroy": (I, [P]),
    "jt_b200_moe_plan_bytes": (SZ, [P]),
    "jt_b200_moe_weights_sizes": (I, [P, P]),
    "jt_b200_moe_weights_write_host": (I, [C.c_char_p, P, P]),
    "jt_b200_moe_weights_read_host": (I, [C.c_char_p, P, P]),
    "jt_b200_moe_weights_save": (I, [C.c_char_p, P, P]),
    "jt_b200_moe_weights_load": (I, [C.c_char_p, P, P]),
    "jt_b200_moe_router_logits": (I, [P, P, I, I, I, P, P]),
    "jt_b200_moe_forward": (I, [P, P, P, P, P, I, P, I, P]),
    "jt_b200_moe_debug_copy": (I, [P, I, P, SZ]),
    "jt_b200_moe_profile_begin": (I, [P, I]),
    "jt_b200_moe_profile_end": (I, [P, P, I, P]),
    "jt_b200_ep_unique_id": (I, [P]),
    "jt_b200_ep_comm_create": (I, [P, I, I, P]),
    "jt_b200_ep_comm_destroy": (I, [P]),
    "jt_b200_ep_comm_set_timeout": (I, [P, I]),
    "jt_b200_ep_comm_failed": (I, [P]),
    "jt_b200_watchdog_selftest": (I, [I, I, P]),
    "jt_b200_moe_ep_plan_create": (I, [P, P, P]),
    "jt_b200_moe_ep_plan_destroy": (I, [P]),
    "jt_b200_moe_ep_forward": (I, [P, P, P, P, P, P, I, P]),
    "jt_b200_moe_ep_debug_copy": (I, [P, I, P, SZ]),
    "jt_b200_ep_capacity": (I, [C.c_longlong, I, I, F]),
    "jt_b200_ep_layout": (I, [P, I, I, I, I, P, P, P, P, P, P]),
    "jt_b200_sync": (I, []),
    "jt_b200_sync_code": (I, [P]),
    "jt_b200_selftest_bounded_wait": (I, [C.c_longlong, P]),
    "jt_b200_last_error": (C.c_char_p, []),
    "jt_b200_version": (C.c_char_p, []),
}


def declare(handle: C.CDLL) -> None:
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
