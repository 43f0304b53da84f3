"""ctypes binding of libdash_b200.so (the C ABI declared in include/dash_b200.h).

The structures below mirror the header field by field; ``check_abi()`` compares
their sizes with the library's own ``sizeof`` values.  Loading fails loudly:
there is no CPU or eager fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdash_b200.so")

DASH_OK = 0
DASH_ERR_INVALID = 1
DASH_ERR_UNSUPPORTED = 2
DASH_ERR_CUDA = 3
DASH_ERR_WORKSPACE = 4

DASH_DEV_TIMEOUT = 1
DASH_DEV_BAD_BLOCK = 2
DASH_DEV_BAD_PAGE = 3

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

_p = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f32 = C.c_float


class DashDeviceError(C.Structure):
    _fields_ = [("code", _i32), ("where", _i32), ("info", _i64)]


class DashSeqs(C.Structure):
    _fields_ = [("n_seq", _i32), ("q_len_fixed", _i32), ("kv_len_fixed", _i32),
                ("max_q_len", _i32), ("q_start", _p), ("pos0", _p), ("kv_len", _p)]


class DashKV(C.Structure):
    _fields_ = [("k", _p), ("v", _p), ("dtype", _i32), ("n_kv_heads", _i32),
                ("head_dim", _i32), ("pad0", _i32), ("stride_seq", _i64),
                ("stride_tok", _i64), ("stride_head", _i64), ("block_table", _p),
                ("bt_stride", _i64), ("num_pages", _i64)]


class DashRoutes(C.Structure):
    _fields_ = [("idx", _p), ("bias", _p), ("row_stride", _i64), ("ihead_stride", _i64),
                ("K", _i32), ("n_index_heads", _i32)]


class DashQO(C.Structure):
    _fields_ = [("q", _p), ("out", _p), ("q_stride_seq", _i64), ("q_stride_tok", _i64),
                ("q_stride_head", _i64), ("o_stride_seq", _i64), ("o_stride_tok", _i64),
                ("o_stride_head", _i64), ("n_heads", _i32), ("pad0", _i32), ("lse", _p),
                ("lse_stride_seq", _i64), ("lse_stride_tok", _i64), ("lse_stride_head", _i64)]


class DashKbarArgs(C.Structure):
    _fields_ = [("keys", _p), ("dtype", _i32), ("d", _i32), ("block_size", _i32),
                ("n_seq", _i32), ("seq_len", _i32), ("n_plan", _i32), ("tok_stride", _i64),
                ("seq_stride", _i64), ("page_stride", _i64), ("kbar_seq_rows", _i64),
                ("head_cls", _p), ("pages", _p), ("ntok", _p), ("kbar", _p),
                ("kbar_row_stride", _i64)]


class DashRouteArgs(C.Structure):
    _fields_ = [("seqs", DashSeqs), ("idx_q", _p), ("q_row_stride", _i64), ("kbar", _p),
                ("kbar_row_stride", _i64), ("block_table", _p), ("bt_stride", _i64),
                ("kbar_seq_rows", _i64), ("num_kbar_rows", _i64), ("width", _i32),
                ("d", _i32), ("scores_in", _p), ("scores_in_stride", _i64),
                ("scores_out", _p), ("scores_out_stride", _i64), ("cand", _p),
                ("cand_row_stride", _i64), ("cand_per_seq", _i32), ("block_size", _i32),
                ("local_blocks", _i32), ("topm", _i32), ("K", _i32), ("out_width", _i32),
                ("idx_scale", _f32), ("prior_floor", _f32), ("inv_sigma", _f32),
                ("pad0", _i32), ("out_idx", _p), ("out_bias", _p), ("out_stride", _i64),
                ("out_count", _p), ("device_error", _p), ("page_q", _p), ("page_lo", _p),
                ("page_hi", _p), ("page_bits", _p), ("page_seq_rows", _i64),
                ("num_page_desc", _i64), ("page_bits_words", _i32), ("pad1", _i32)]


class DashBlockMaxArgs(C.Structure):
    _fields_ = [("q", _p), ("q_stride_b", _i64), ("q_stride_c", _i64), ("k", _p),
                ("k_stride_b", _i64), ("k_stride_j", _i64), ("pos", _p),
                ("pos_stride_b", _i64), ("pos_stride_c", _i64), ("seg", _p),
                ("seg_stride_b", _i64), ("seg_stride_c", _i64), ("B", _i32), ("C", _i32),
                ("Sk", _i32), ("d", _i32), ("block_size", _i32), ("nblk", _i32),
                ("local_window", _i32), ("clamp", _i32), ("empty", _f32), ("pad0", _i32),
                ("out", _p), ("out_stride_b", _i64), ("out_stride_c", _i64)]


class DashPrefillArgs(C.Structure):
    _fields_ = [("seqs", DashSeqs), ("kv", DashKV), ("routes", DashRoutes), ("qo", DashQO),
                ("seg_start", _p), ("scale", _f32), ("block_size", _i32),
                ("local_window", _i32), ("mode", _i32), ("workspace", _p),
                ("workspace_bytes", C.c_size_t), ("device_error", _p), ("out_peers", _p),
                ("n_peers", _i32), ("part_budget_mib", _i32)]


class DashPeerHandle(C.Structure):
    # unsigned bytes: a c_char array field would read back as NUL-truncated bytes
    _fields_ = [("handle", C.c_ubyte * 64), ("offset", _i64), ("alloc_bytes", _i64)]


class DashDecodeArgs(C.Structure):
    _fields_ = [("seqs", DashSeqs), ("kv", DashKV), ("routes", DashRoutes), ("qo", DashQO),
                ("scale", _f32), ("block_size", _i32), ("local_window", _i32),
                ("num_splits", _i32), ("workspace", _p), ("workspace_bytes", C.c_size_t),
                ("device_error", _p)]


class DashPageIdsArgs(C.Structure):
    _fields_ = [("token_ids", _p), ("ids_stride", _i64), ("n_seq", _i32), ("ids_len", _i32),
                ("key_length", _i32), ("per_page", _i32), ("image_token_id", _i64),
                ("page_token_id", _i64), ("mm_pad_shift", _i64), ("has_page_token", _i32),
                ("rule", _i32), ("page_scope_prefill", _i32), ("block_size", _i32),
                ("n_blocks", _i32), ("page_elem_bytes", _i32), ("image_mask", _p),
                ("image_mask_stride", _i64), ("image_page", _p), ("image_page_stride", _i64),
                ("query_page", _p), ("query_page_stride", _i64), ("blk_lo", _p),
                ("blk_hi", _p), ("blk_bits", _p), ("blk_has_image", _p),
                ("prompt_pages", _p), ("marker_count", _p), ("n_image", _p),
                ("n_query", _p), ("device_error", _p)]


class DashPageStateArgs(C.Structure):
    _fields_ = [("input_ids", _p), ("q_start", _p), ("start_pos", _p), ("seq_lens", _p),
                ("gen_start", _p), ("block_table", _p), ("bt_stride", _i64),
                ("slot_mapping", _p), ("num_slots", _i64), ("image_token_id", _i64),
                ("page_token_id", _i64), ("mm_pad_shift", _i64), ("num_tokens", _i32),
                ("num_reqs", _i32), ("num_decode_tokens", _i32), ("bt_width", _i32),
                ("block_size", _i32), ("per_page", _i32), ("has_page_token", _i32),
                ("pad0", _i32), ("slot_img_page", _p), ("slot_marker_cum", _p),
                ("slot_img_run", _p), ("slot_prompt_pages", _p), ("q_page", _p),
                ("blk_lo", _p), ("blk_hi", _p), ("device_error", _p)]


class DashPageAllowArgs(C.Structure):
    _fields_ = [("rows", _i32), ("width", _i32), ("out", _p), ("out_stride", _i64),
                ("q_page", _p), ("q_elem_bytes", _i32), ("q_len", _i32), ("q_pos", _p),
                ("q_stride", _i64), ("row_seq", _p), ("rows_per_seq", _i32), ("desc_width", _i32),
                ("page_lo", _p), ("page_hi", _p), ("page_bits", _p), ("page_bits_words", _i32),
                ("block_size", _i32), ("num_desc", _i64), ("block_table", _p),
                ("bt_stride", _i64), ("desc_seq_rows", _i64), ("seq_lens", _p),
                ("fallback", _i32), ("pad0", _i32)]


class DashPageDecodeArgs(C.Structure):
    _fields_ = [("last_ids", _p), ("ids_stride", _i64), ("n_seq", _i32),
                ("has_page_token", _i32), ("page_token_id", _i64), ("marker_count", _p),
                ("prompt_pages", _p), ("q_page", _p)]


class DashBlockAnyArgs(C.Structure):
    _fields_ = [("mask", _p), ("mask_stride", _i64), ("rows", _i32), ("len", _i32),
                ("block_size", _i32), ("n_blocks", _i32), ("out", _p), ("out_stride", _i64)]


class DashPageBlocksArgs(C.Structure):
    _fields_ = [("pages", _p), ("stride", _i64), ("elem_bytes", _i32), ("rows", _i32),
                ("len", _i32), ("block_size", _i32), ("n_blocks", _i32), ("pad0", _i32),
                ("lo", _p), ("hi", _p), ("bits", _p)]


class DashIndexProjArgs(C.Structure):
    _fields_ = [("hidden", _p), ("hidden_stride", _i64), ("w_q", _p), ("w_k", _p),
                ("w_stride", _i64), ("norm_q", _p), ("norm_k", _p), ("cos", _p), ("sin", _p),
                ("cs_stride", _i64), ("eps", _f32), ("norm_clamp", _i32), ("T", _i32),
                ("hidden_dim", _i32), ("d", _i32), ("k_dtype", _i32), ("idx_q", _p),
                ("q_stride", _i64), ("idx_k", _p), ("k_stride", _i64), ("slot_mapping", _p),
                ("k_rows", _i64), ("device_error", _p),
                ("kbar_page", _p), ("kbar_ntok", _p), ("kbar_head_cls", _p), ("kbar", _p),
                ("kbar_row_stride", _i64), ("kbar_block_size", _i32), ("pad1", _i32)]


class DashRopeKVArgs(C.Structure):
    _fields_ = [("q", _p), ("q_stride", _i64), ("q_out", _p), ("q_out_stride", _i64),
                ("k", _p), ("k_stride", _i64), ("v", _p), ("v_stride", _i64), ("cos", _p),
                ("sin", _p), ("cs_stride", _i64), ("k_cache", _p), ("v_cache", _p),
                ("cache_row_stride", _i64), ("slot_mapping", _p), ("num_slots", _i64),
                ("T", _i32), ("n_q_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
                ("device_error", _p)]


class DashAttnBwdArgs(C.Structure):
    _fields_ = [("q", _p), ("k", _p), ("v", _p), ("o", _p), ("dout", _p), ("dq", _p),
                ("dk", _p), ("dv", _p), ("lse", _p), ("idx", _p), ("bias", _p), ("d_bias", _p),
                ("delta", _p), ("flags", _p), ("dq_acc", _p), ("n_seq", _i32), ("seq_len", _i32),
                ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32), ("dtype", _i32),
                ("block_size", _i32), ("local_window", _i32), ("K", _i32), ("pad0", _i32),
                ("scale", _f32), ("pad1", _f32), ("device_error", _p), ("seg_start", _p),
                ("n_index_heads", _i32), ("pad2", _i32)]


class DashEntmaxArgs(C.Structure):
    _fields_ = [("x", _p), ("y", _p), ("dy", _p), ("dx", _p), ("rows", _i64), ("stride", _i64),
                ("n", _i32), ("pad0", _i32)]


class DashServingPlanArgs(C.Structure):
    _fields_ = [("block_table", _p), ("bt_stride", _i64), ("seq_lens", _p), ("context_lens", _p),
                ("cu_seqlens_q", _p), ("n_req", _i32), ("block_size", _i32), ("width", _i32),
                ("mode", _i32), ("bt_width", _i32), ("pad0", _i32), ("pages", _p), ("ntok", _p),
                ("row2req", _p)]


class DashPageCoordArgs(C.Structure):
    _fields_ = [("input_ids", _p), ("q_start", _p), ("start_pos", _p), ("gen_start", _p),
                ("row_key", _p), ("image_token_id", _i64), ("page_token_id", _i64),
                ("mm_pad_shift", _i64), ("num_tokens", _i32), ("num_reqs", _i32),
                ("num_decode_tokens", _i32), ("has_page_token", _i32), ("max_rows", _i32),
                ("max_pages", _i32), ("state_key", _p), ("state_stamp", _p), ("step", _p),
                ("c_marker", _p), ("c_pp", _p), ("cnt", _p), ("rows", _p), ("tok_pos", _p),
                ("page_pos", _p)]


class DashCosSin2DArgs(C.Structure):
    _fields_ = [("tok_pos", _p), ("page_pos", _p), ("inv_tok", _p), ("inv_page", _p),
                ("cos", _p), ("sin", _p), ("stride", _i64), ("page_mod", _i64),
                ("num_tokens", _i32), ("dim", _i32), ("n_tok", _i32), ("out_bf16", _i32)]


ABI_ORDER = [DashSeqs, DashKV, DashRoutes, DashQO, DashKbarArgs, DashRouteArgs,
             DashBlockMaxArgs, DashPrefillArgs, DashDecodeArgs, DashDeviceError,
             DashPageIdsArgs, DashPageStateArgs, DashPageAllowArgs, DashPageDecodeArgs,
             DashBlockAnyArgs, DashPageBlocksArgs, DashIndexProjArgs, DashRopeKVArgs,
             DashAttnBwdArgs, DashEntmaxArgs, DashServingPlanArgs, DashPeerHandle,
             DashPageCoordArgs, DashCosSin2DArgs]

# every function the header declares
EXPORTS = [
    "dash_kbar_pool", "dash_route", "dash_block_max", "dash_prefill_workspace_size",
    "dash_prefill_attn", "dash_decode_workspace_size", "dash_decode_attn", "dash_last_error",
    "dash_library_version", "dash_count_launches", "dash_abi_sizes",
    "dash_decode_attn_noalloc", "dash_noalloc_scratch_bytes", "dash_selftest_bounded_wait",
    "dash_page_ids", "dash_page_state_step", "dash_page_allow", "dash_page_decode_query",
    "dash_block_any", "dash_page_blocks", "dash_index_proj", "dash_rope_kv_write",
    "dash_attn_bwd", "dash_attn_bwd_flag_words", "dash_entmax15_fwd", "dash_entmax15_bwd",
    "dash_serving_plan", "dash_peer_export", "dash_peer_import", "dash_peer_close",
    "dash_page_coords", "dash_cos_sin_2d", "dash_route_refresh",
]


class DashError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"dash status {code}: {msg}")
        self.code = code


_lib = None


def load(path: str = LIB_PATH):
    """Load the library (once).  Raises if it is missing: no fallback exists."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing; build it with `python -m ananta_ocr_b200.build` "
            "(the DASH kernels have no CPU or eager fallback)")
    L = C.CDLL(path)
    for name, args in [
        ("dash_kbar_pool", [C.POINTER(DashKbarArgs), _p]),
        ("dash_route", [C.POINTER(DashRouteArgs), _p]),
        ("dash_block_max", [C.POINTER(DashBlockMaxArgs), _p]),
        ("dash_prefill_attn", [C.POINTER(DashPrefillArgs), _p]),
        ("dash_decode_attn", [C.POINTER(DashDecodeArgs), _p]),
        ("dash_page_ids", [C.POINTER(DashPageIdsArgs), _p]),
        ("dash_page_state_step", [C.POINTER(DashPageStateArgs), _p]),
        ("dash_page_allow", [C.POINTER(DashPageAllowArgs), _p]),
        ("dash_page_decode_query", [C.POINTER(DashPageDecodeArgs), _p]),
        ("dash_block_any", [C.POINTER(DashBlockAnyArgs), _p]),
        ("dash_page_blocks", [C.POINTER(DashPageBlocksArgs), _p]),
        ("dash_index_proj", [C.POINTER(DashIndexProjArgs), _p]),
        ("dash_rope_kv_write", [C.POINTER(DashRopeKVArgs), _p]),
        ("dash_attn_bwd", [C.POINTER(DashAttnBwdArgs), _p]),
        ("dash_entmax15_fwd", [C.POINTER(DashEntmaxArgs), _p]),
        ("dash_entmax15_bwd", [C.POINTER(DashEntmaxArgs), _p]),
        ("dash_serving_plan", [C.POINTER(DashServingPlanArgs), _p]),
        ("dash_page_coords", [C.POINTER(DashPageCoordArgs), _p]),
        ("dash_cos_sin_2d", [C.POINTER(DashCosSin2DArgs), _p]),
    ]:
        f = getattr(L, name)
        f.argtypes = args
        f.restype = C.c_int
    L.dash_route_refresh.argtypes = [C.POINTER(DashRouteArgs), C.POINTER(DashKbarArgs), _p]
    L.dash_route_refresh.restype = C.c_int
    L.dash_prefill_workspace_size.argtypes = [C.POINTER(DashPrefillArgs)]
    L.dash_prefill_workspace_size.restype = C.c_size_t
    L.dash_decode_workspace_size.argtypes = [C.POINTER(DashDecodeArgs)]
    L.dash_decode_workspace_size.restype = C.c_size_t
    L.dash_decode_attn_noalloc.argtypes = [C.POINTER(DashDecodeArgs), _p]
    L.dash_decode_attn_noalloc.restype = C.c_int
    L.dash_noalloc_scratch_bytes.argtypes = []
    L.dash_noalloc_scratch_bytes.restype = C.c_size_t
    L.dash_last_error.argtypes = [C.c_char_p, C.c_int]
    L.dash_last_error.restype = C.c_int
    L.dash_library_version.restype = C.c_int
    L.dash_count_launches.argtypes = [C.c_int]
    L.dash_count_launches.restype = C.c_int
    L.dash_abi_sizes.argtypes = [C.POINTER(_i64), C.c_int]
    L.dash_abi_sizes.restype = C.c_int
    L.dash_attn_bwd_flag_words.argtypes = [C.POINTER(DashAttnBwdArgs)]
    L.dash_attn_bwd_flag_words.restype = C.c_int64
    L.dash_peer_export.argtypes = [_p, C.POINTER(DashPeerHandle)]
    L.dash_peer_export.restype = C.c_int
    L.dash_peer_import.argtypes = [C.POINTER(DashPeerHandle), C.POINTER(_p)]
    L.dash_peer_import.restype = C.c_int
    L.dash_peer_close.argtypes = [_p]
    L.dash_peer_close.restype = C.c_int
    L.dash_selftest_bounded_wait.argtypes = [C.c_uint64, _p, _p]
    L.dash_selftest_bounded_wait.restype = C.c_int
    _lib = L
    check_abi()
    return L


def check_abi():
    L = _lib
    out = (_i64 * len(ABI_ORDER))()
    n = L.dash_abi_sizes(out, len(ABI_ORDER))
    if n != len(ABI_ORDER):
        raise RuntimeError(f"ABI mismatch: library reports {n} structs, python {len(ABI_ORDER)}")
    for i, cls in enumerate(ABI_ORDER[:n]):
        if C.sizeof(cls) != out[i]:
            raise RuntimeError(f"ABI mismatch for {cls.__name__}: python {C.sizeof(cls)} "
                               f"vs library {out[i]}")


def last_error() -> str:
    buf = C.create_string_buffer(512)
    load().dash_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def call(fn_name: str, args) -> None:
    L = load()
    rc = getattr(L, fn_name)(C.byref(args), current_stream())
    if rc != DASH_OK:
        raise DashError(rc, last_error())


def current_stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def launches(reset: bool = False) -> int:
    return load().dash_count_launches(1 if reset else 0)
