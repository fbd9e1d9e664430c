"""ctypes binding of the C ABI in ``include/beam_b200.h``.

The library is built in-tree (``beam_engine_b200/lib/libbeam_b200.so``).  There
is no fallback: if the library is missing every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libbeam_b200.so")
_lib = None

i32, i64, f32, f64 = C.c_int32, C.c_int64, C.c_float, C.c_double
vp = C.c_void_p
P32 = C.POINTER(C.c_int32)
PP32 = C.POINTER(P32)

(BE_OK, BE_EINVAL, BE_ENOMEM, BE_ECUDA, BE_ENOT_ALLOCATED, BE_ECAPACITY, BE_EDEVICE_RANGE,
 BE_EDEVICE_TIMEOUT, BE_ENOTSUP) = range(9)
BE_F32, BE_F16, BE_BF16 = 0, 1, 2
BE_CAPS_SLOTS = 1


class AttnPlanInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "n_work", "n_work_wide", "n_queries", "n_parts", "n_merge", "off_work", "off_qlist",
        "off_kvlist", "off_merge_q", "off_merge_ptr", "off_merge_parts", "total_ints",
        "page_size", "group_size", "any_slots", "max_item_tokens", "total_tokens", "max_wide_tokens")]


class TilePlanInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "n_tiles", "n_pieces", "n_entries", "n_queries", "off_tiles", "off_pieces", "off_entries",
        "total_ints", "page_size", "group_size", "tile_rows", "n_part_pieces", "total_tokens",
        "max_piece_entries", "cluster", "pad1")]


class AttnCaps(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("max_work", "max_wide", "max_merge", "cluster", "flags")]


_SIGS = {
    "be_last_error": (C.c_char_p, []),
    "be_version": (C.c_int, []),
    "be_device_status": (C.c_int, [P32, vp]),
    "be_device_status_clear": (C.c_int, [vp]),
    "be_append_paged_kv": (C.c_int, [vp, vp, i64, i64, vp, vp, vp, vp, C.c_int, vp, i64, C.c_int,
                                     C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
    "be_fork_tail_copy": (C.c_int, [vp, i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    vp, vp, vp, C.c_int, vp]),
    "be_cascade_plan": (C.c_int, [C.c_int, PP32, PP32, PP32, PP32, P32, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_int, P32, i64,
                                  C.POINTER(AttnPlanInfo)]),
    "be_tree_plan": (C.c_int, [C.c_int, P32, C.c_int, P32, P32, P32, P32, P32, P32, P32, C.c_int,
                               C.c_int, C.c_int, C.c_int, P32, i64, C.POINTER(AttnPlanInfo)]),
    "be_attn_run": (C.c_int, [vp, C.POINTER(AttnPlanInfo), vp, i64, vp, C.c_int, C.c_int, C.c_int,
                              C.c_int, C.c_int, f32, vp, i64, vp, vp, vp, vp, vp]),
    "be_add_rmsnorm": (C.c_int, [vp, vp, vp, vp, C.c_int, C.c_int, f32, C.c_int, vp]),
    "be_rope_qkv_append": (C.c_int, [vp, i64, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp,
                                     C.c_int, C.c_int, vp, vp, C.c_int, C.c_int, vp]),
    "be_silu_mul": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp]),
    "be_gemm_lt": (C.c_int, [vp, i64, vp, i64, vp, i64, C.c_int, C.c_int, C.c_int, C.c_int, vp,
                             i64, vp]),
    "be_gemm_tn": (C.c_int, [vp, i64, vp, i64, vp, i64, C.c_int, C.c_int, C.c_int, C.c_int,
                             C.c_int, vp, i64, vp]),
    "be_logsoftmax_topk": (C.c_int, [vp, i64, C.c_int, C.c_int, f32, C.c_int, i64, C.c_int, vp, vp,
                                     vp, vp, vp]),
    "be_attn_run_noalloc": (C.c_int, [vp, C.POINTER(AttnPlanInfo), vp, i64, vp, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int, f32, vp, i64, vp, vp, vp]),
    "be_attn_run_fixed": (C.c_int, [vp, vp, C.c_int, vp, i64, vp, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, f32, vp, i64, vp, vp, vp, vp, vp]),
    "be_attn_run_fixed_2s": (C.c_int, [vp, vp, C.c_int, vp, i64, vp, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, f32, vp, i64, vp, vp, vp, vp, vp, vp]),
    # host page manager
    "be_trie_create": (vp, [C.c_int, C.c_int]),
    "be_trie_destroy": (None, [vp]),
    "be_alloc_page": (C.c_int, [vp, P32]),
    "be_free_page": (C.c_int, [vp, i32]),
    "be_num_free_pages": (C.c_int, [vp]),
    "be_is_allocated": (C.c_int, [vp, i32]),
    "be_free_list": (C.c_int, [vp, P32, C.c_int]),
    "be_trie_warnings": (i64, [vp]),
    "be_trie_num_nodes": (C.c_int, [vp]),
    "be_node_new": (C.c_int, [vp, i32, i32, P32, C.c_int, P32]),
    "be_node_info": (C.c_int, [vp, i32, P32, P32, P32, P32]),
    "be_node_tokens": (C.c_int, [vp, i32, P32, C.c_int]),
    "be_node_children": (C.c_int, [vp, i32, P32, C.c_int]),
    "be_node_append_token": (C.c_int, [vp, i32, i32]),
    "be_node_sequence": (i64, [vp, i32, P32, i64]),
    "be_beam_add_root": (C.c_int, [vp, P32, C.c_int, P32, P32]),
    "be_beam_update": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "be_beam_step_inputs": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, vp]),
    "be_cascade_build": (C.c_int, [vp, C.c_int, P32, C.c_int, C.c_int, C.c_int, P32, P32, P32, P32,
                                   P32, P32]),
    "be_tree_build": (C.c_int, [vp, C.c_int, P32, C.c_int, C.c_int, C.c_int, P32, P32, P32, P32, P32, P32,
                                i64, P32, P32, i64]),
    "be_fasttree_prepare": (C.c_int, [C.c_int, P32, P32, P32, P32, P32, i64, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int, P32, P32, P32, P32, P32, P32, P32,
                                      P32, P32]),
    "be_vanilla_select_segments": (C.c_int, [C.c_int, vp, C.c_int, vp, vp,
                                             vp, C.c_int, vp, vp,
                                             vp, vp]),
    "be_beam_decode_inputs": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, vp, i64,
                                        C.c_int, C.POINTER(AttnPlanInfo)]),
    "be_tile_plan": (C.c_int, [C.c_int, PP32, PP32, PP32, PP32, P32, C.c_int, C.c_int, C.c_int,
                               C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P32, i64,
                               C.POINTER(TilePlanInfo)]),
    "be_beam_decode_tiles": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_int, vp, i64, C.c_int, C.POINTER(TilePlanInfo)]),
    "be_attn_tiles_run": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, i64, vp,
                                    C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, f32, vp, i64, vp,
                                    vp, vp, C.c_int, C.c_int, vp]),
    "be_fork_tail_copy_list": (C.c_int, [vp, i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_int, vp, C.c_int, C.c_int, vp]),
    "be_comm_create": (C.c_int, [C.c_int, C.c_int, i64, C.c_int, C.c_int, vp, C.POINTER(vp)]),
    "be_comm_open": (C.c_int, [vp, vp]),
    "be_comm_slot": (vp, [vp, C.c_int]),
    "be_comm_topk_layout": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_int64)]),
    "be_comm_topk_merge": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
    "be_comm_flags": (vp, [vp]),
    "be_comm_close_peers": (C.c_int, [vp]),
    "be_comm_destroy": (C.c_int, [vp]),
    "be_comm_allreduce_rmsnorm": (C.c_int, [vp, C.c_int, vp, vp, vp, C.c_int, C.c_int, C.c_float,
                                            C.c_int, vp]),
    "be_tree_plan_pages": (C.c_int, [C.c_int, vp, C.c_int, vp, vp, vp, vp, vp, i64, C.c_int,
                                      C.c_int, C.c_int, C.c_int, C.c_int, vp, i64,
                                      C.POINTER(AttnPlanInfo)]),
    "be_beam_select_update": (C.c_int, [vp, C.c_int, vp, C.c_int, vp, vp, vp, vp, C.c_int, vp, vp,
                                        vp, vp, vp, vp, vp, vp, vp]),
    "be_cascade_pages_twice": (C.c_int, [C.c_int, vp, vp, vp, vp, C.c_int]),
    "be_vanilla_select_device": (C.c_int, [C.c_int, vp, C.c_int, vp, vp, vp, C.c_int, C.c_int,
                                           vp, vp, vp, vp]),
    "be_beam_update_selected": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, vp, C.c_int, vp, vp, vp, vp,
                                          vp, vp, vp, vp, vp]),
    "be_leaf_sequences": (i64, [vp, C.c_int, vp, vp, vp, i64]),
    "be_diverse_select": (C.c_int, [C.c_int, vp, C.c_int, vp, vp,
                                    vp, vp, vp, C.c_int, C.c_int, C.c_double,
                                    C.c_int, C.c_double, vp, vp, vp, vp]),
    "be_diverse_select_device": (C.c_int, [C.c_int, vp, C.c_int, vp, vp, vp, vp, C.c_int,
                                           C.c_int, C.c_double, C.c_int, C.c_double, C.c_int,
                                           vp, vp, vp, vp, vp]),
    "be_vanilla_select": (C.c_int, [C.c_int, C.c_int, vp, vp,
                                    vp, C.c_int, vp, vp,
                                    vp]),
}


def exported_symbols():
    return list(_SIGS)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(
                f"beam_engine_b200 native library not found at {_LIB_PATH}; build it with "
                "`python -m beam_engine_b200.build_lib` (there is no CPU fallback)")
        L = C.CDLL(_LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class BeamEngineError(RuntimeError):
    pass


def check(rc, what=""):
    if rc == BE_OK:
        return
    msg = lib().be_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == BE_EINVAL:
        raise ValueError(text)
    if rc == BE_ENOMEM:
        raise MemoryError(text)
    raise BeamEngineError(f"[status {rc}] {text}")


def addr(arr):
    """Address of a contiguous numpy array, for arguments bound as void* (half
    the cost of ptr32 on the per-step host path).  A plain int: unlike ptr32 it
    does not keep the array alive, so pass a named array, never a temporary."""
    return arr.ctypes.data


def ptr32(arr):
    """ctypes int32* of a contiguous numpy int32 array."""
    return arr.ctypes.data_as(P32)
