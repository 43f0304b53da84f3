"""C-ABI checks that need no GPU: the library loads, exports every function the
header declares, its struct layouts match the Python binding, and malformed
calls are rejected on the host with a status and a message."""
import ctypes as C
import os
import re

import pytest

from ananta_ocr_b200 import _lib as L

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "dash_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t)\s+(dash_\w+)\s*\(", text, re.M)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(L.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_struct_sizes():
    L.load()
    L.check_abi()


def _call_status(fn, args):
    lib = L.load()
    return getattr(lib, fn)(C.byref(args), None)


def test_route_rejects_bad_arguments():
    a = L.DashRouteArgs()
    assert _call_status("dash_route", a) == L.DASH_ERR_INVALID     # null outputs
    assert "null" in L.last_error()
    a.out_idx = a.out_bias = 16
    a.width = 10
    a.K, a.out_width = 4, 2
    assert _call_status("dash_route", a) == L.DASH_ERR_INVALID     # K > out_width
    a.out_width = 4
    a.topm = 0
    a.width = 1000
    assert _call_status("dash_route", a) == L.DASH_ERR_UNSUPPORTED  # entmax window too wide


def _prefill_args(head_dim=128, block_size=64, heads=10, kv_heads=10, K=4):
    a = L.DashPrefillArgs()
    a.seqs.n_seq, a.seqs.q_len_fixed, a.seqs.kv_len_fixed, a.seqs.max_q_len = 1, 256, 256, 256
    a.kv.k = a.kv.v = 1 << 20
    a.kv.dtype = L.DTYPE_BF16
    a.kv.n_kv_heads, a.kv.head_dim = kv_heads, head_dim
    a.kv.stride_seq, a.kv.stride_tok, a.kv.stride_head = 256 * kv_heads * 128, kv_heads * 128, 128
    a.routes.idx = 1 << 21
    a.routes.K = K
    a.routes.row_stride = K
    a.qo.q = a.qo.out = 1 << 22
    a.qo.n_heads = heads
    a.qo.q_stride_tok = a.qo.o_stride_tok = heads * 128
    a.qo.q_stride_head = a.qo.o_stride_head = 128
    a.block_size, a.local_window, a.scale = block_size, 256, 0.088
    return a


def test_prefill_mode_checks_and_workspace():
    """Mode 2 (routed part gathered by key block) is refused outside its
    shapes; its workspace adds the per-block row flags and a partial scratch
    that the budget bounds (one chunk's partials)."""
    a = _prefill_args(heads=8, kv_heads=1)
    a.mode = 2
    assert _call_status("dash_prefill_attn", a) == L.DASH_ERR_UNSUPPORTED   # 8 heads per kv head
    a = _prefill_args(block_size=192)
    a.mode = 2
    assert _call_status("dash_prefill_attn", a) == L.DASH_ERR_UNSUPPORTED
    a = _prefill_args()
    a.mode = 3
    assert _call_status("dash_prefill_attn", a) == L.DASH_ERR_INVALID
    lib = L.load()

    def size(mode, budget=0, T=9248, K=16):
        a = _prefill_args(K=K)
        a.seqs.n_seq, a.seqs.q_len_fixed, a.seqs.kv_len_fixed, a.seqs.max_q_len = 4, T, T, T
        a.mode, a.part_budget_mib = mode, budget
        return lib.dash_prefill_workspace_size(C.byref(a))

    union, full = size(1), size(2)
    # every (row, head, slot) partial: 128 bf16 + one fp32
    assert full - union >= 4 * 9248 * 10 * 16 * 260
    assert size(0) == union                     # automatic: tile-major for 64-token blocks, K = 16

    def size128(mode, K):
        a = _prefill_args(K=K, block_size=128)
        a.seqs.n_seq, a.seqs.q_len_fixed, a.seqs.kv_len_fixed, a.seqs.max_q_len = 1, 16384, 16384, 16384
        a.mode = mode
        return lib.dash_prefill_workspace_size(C.byref(a))
    # automatic: gathered for 128-token blocks with K >= 32 (the long-document shape)
    assert size128(0, 64) == size128(2, 64) > size128(1, 64)
    assert size128(0, 16) == size128(1, 16)
    small = size(2, budget=8)
    assert union < small <= union + 8 * 2**20 + 4 * 145 * 292 * 4 + 3 * 256


def test_prefill_rejects_unsupported_shapes():
    assert _call_status("dash_prefill_attn", _prefill_args(head_dim=64)) == L.DASH_ERR_UNSUPPORTED
    assert "head_dim" in L.last_error()
    assert _call_status("dash_prefill_attn", _prefill_args(block_size=16)) == L.DASH_ERR_UNSUPPORTED
    assert _call_status("dash_prefill_attn", _prefill_args(block_size=96)) == L.DASH_ERR_UNSUPPORTED
    assert "32" in L.last_error()
    assert _call_status("dash_prefill_attn", _prefill_args(heads=12, kv_heads=8)) == L.DASH_ERR_INVALID
    assert _call_status("dash_prefill_attn", _prefill_args(heads=24, kv_heads=8)) == L.DASH_ERR_UNSUPPORTED
    assert _call_status("dash_prefill_attn", _prefill_args(K=300)) == L.DASH_ERR_UNSUPPORTED


def test_prefill_requires_workspace():
    a = _prefill_args()
    lib = L.load()
    need = lib.dash_prefill_workspace_size(C.byref(a))
    assert need > 0
    assert _call_status("dash_prefill_attn", a) == L.DASH_ERR_WORKSPACE
    assert "workspace" in L.last_error()


def test_decode_workspace_and_validation():
    a = L.DashDecodeArgs()
    a.seqs.n_seq, a.seqs.q_len_fixed, a.seqs.kv_len_fixed, a.seqs.max_q_len = 64, 1, 27556, 1
    a.kv.k = a.kv.v = 1 << 20
    a.kv.dtype = L.DTYPE_BF16
    a.kv.n_kv_heads, a.kv.head_dim = 10, 128
    a.kv.stride_seq, a.kv.stride_tok, a.kv.stride_head = 64 * 1280, 1280, 128
    a.kv.block_table, a.kv.bt_stride, a.kv.num_pages = 1 << 23, 431, 27584
    a.routes.idx, a.routes.K, a.routes.row_stride = 1 << 21, 32, 32
    a.qo.q = a.qo.out = 1 << 22
    a.qo.n_heads = 10
    a.qo.q_stride_seq = a.qo.o_stride_seq = 1280
    a.qo.q_stride_tok = a.qo.o_stride_tok = 1280
    a.qo.q_stride_head = a.qo.o_stride_head = 128
    a.block_size, a.local_window, a.scale = 64, 256, 0.088
    lib = L.load()
    a.num_splits = 4
    assert lib.dash_decode_workspace_size(C.byref(a)) >= 64 * 10 * 4 * 130 * 4
    assert _call_status("dash_decode_attn", a) == L.DASH_ERR_WORKSPACE
    a.num_splits = 1
    assert lib.dash_decode_workspace_size(C.byref(a)) == 0
    a.kv.dtype = L.DTYPE_F32
    assert _call_status("dash_decode_attn", a) == L.DASH_ERR_UNSUPPORTED
    a.kv.dtype = L.DTYPE_BF16
    # malformed calls are rejected before anything is sized, by the workspace
    # query (0), the workspace entry point and the allocation-free one alike
    for field, bad in (("block_size", 0), ("num_splits", -1), ("n_seq", -1)):
        saved = getattr(a.seqs if field == "n_seq" else a, field)
        setattr(a.seqs if field == "n_seq" else a, field, bad)
        a.num_splits = -1 if field == "num_splits" else 0
        assert lib.dash_decode_workspace_size(C.byref(a)) == 0, field
        for fn in ("dash_decode_attn", "dash_decode_attn_noalloc"):
            assert _call_status(fn, a) == L.DASH_ERR_INVALID, (fn, field, L.last_error())
        setattr(a.seqs if field == "n_seq" else a, field, saved)
    a.num_splits = 65
    for fn in ("dash_decode_attn", "dash_decode_attn_noalloc"):
        assert _call_status(fn, a) == L.DASH_ERR_UNSUPPORTED


def test_kbar_validation():
    a = L.DashKbarArgs()
    assert _call_status("dash_kbar_pool", a) == L.DASH_ERR_INVALID
    a.keys = a.kbar = 1 << 20
    a.dtype, a.d, a.block_size = L.DTYPE_F16, 128, 64
    assert _call_status("dash_kbar_pool", a) == L.DASH_ERR_UNSUPPORTED


def test_package_fails_loudly_without_library(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU or eager fallback"):
        saved = L._lib
        try:
            L._lib = None
            L.load(str(tmp_path / "missing.so"))
        finally:
            L._lib = saved


def test_attn_bwd_rejects_bad_arguments():
    a = L.DashAttnBwdArgs()
    a.n_seq, a.seq_len, a.n_heads, a.n_kv_heads, a.head_dim = 1, 128, 4, 2, 128
    a.dtype, a.block_size, a.local_window, a.K, a.scale = L.DTYPE_BF16, 64, 64, 4, 0.1
    assert L.load().dash_attn_bwd_flag_words(C.byref(a)) == 2 * 4
    for field, bad in (("head_dim", 64), ("block_size", 48), ("K", 300), ("n_heads", 3),
                       ("n_heads", 32), ("dtype", 9)):
        old = getattr(a, field)
        setattr(a, field, bad)
        assert _call_status("dash_attn_bwd", a) != 0, field
        assert L.load().dash_attn_bwd_flag_words(C.byref(a)) == -1
        setattr(a, field, old)
    assert _call_status("dash_attn_bwd", a) == L.DASH_ERR_INVALID     # null pointers
    assert "null" in L.last_error()


def test_entmax_rejects_bad_arguments():
    a = L.DashEntmaxArgs()
    a.rows, a.n, a.stride = 4, 10, 5
    assert _call_status("dash_entmax15_fwd", a) == L.DASH_ERR_INVALID
    a.stride = 10
    assert _call_status("dash_entmax15_bwd", a) == L.DASH_ERR_INVALID
    a.rows = 0
    assert _call_status("dash_entmax15_fwd", a) == 0
