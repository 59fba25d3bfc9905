"""ctypes binding of the C ABI (include/cascade_b200.h).

This is the binding a non-torch host (or a test) uses: plain pointers and
sizes. ``load()`` opens ``libcascade_b200.so`` without importing the torch
extension. Tensor helpers accept torch tensors only to read ``data_ptr()``.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libcascade_b200.so")

BF16, FP16, FP32 = 0, 1, 2
OK, ERR_INVALID, ERR_CUDA, ERR_WORKSPACE, ERR_UNSUPPORTED = 0, 1, 2, 3, 4

EXPORTED = [
    "cascade_fa_fp32_stage1_workspace_size",
    "cascade_fa_fp32_stage1",
    "cascade_suffix_decode_workspace_size",
    "cascade_suffix_decode",
    "cascade_suffix_decode_noalloc",
    "cascade_decode_step_workspace_size",
    "cascade_decode_step",
    "cascade_lse_merge",
    "cascade_f3_gateup_epilogue",
    "cascade_add_rms_norm_stats",
    "cascade_last_error",
    "cascade_device_error",
    "cascade_version",
    "cascade_plan_paged_attn",
    "cascade_check_block_table",
    "cascade_probe_hbm_read",
]


class PagedAttn(ctypes.Structure):
    _fields_ = [
        ("query", ctypes.c_void_p),
        ("key", ctypes.c_void_p),
        ("value", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("actual_q_seqlens", ctypes.c_void_p),
        ("actual_kv_seqlens", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int64),
        ("num_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("batch", ctypes.c_int64),
        ("block_cols", ctypes.c_int64),
        ("q_seqlen_value", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class AttnPlan(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("rows_per_group", ctypes.c_int32),
        ("split_tokens", ctypes.c_int64),
        ("num_splits", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_size_t),
    ]


_lib = None


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} not built; run vllm-hust-cascade-kernel_b200/build.py")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER(PagedAttn)
    vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t
    lib.cascade_fa_fp32_stage1_workspace_size.argtypes = [P]
    lib.cascade_fa_fp32_stage1_workspace_size.restype = sz
    lib.cascade_suffix_decode_workspace_size.argtypes = [P]
    lib.cascade_suffix_decode_workspace_size.restype = sz
    lib.cascade_fa_fp32_stage1.argtypes = [P, vp, vp, vp, sz, vp]
    lib.cascade_fa_fp32_stage1.restype = ctypes.c_int
    lib.cascade_suffix_decode.argtypes = [P, vp, vp, vp, sz, vp]
    lib.cascade_suffix_decode.restype = ctypes.c_int
    lib.cascade_suffix_decode_noalloc.argtypes = [P, vp, vp, vp]
    lib.cascade_suffix_decode_noalloc.restype = ctypes.c_int
    lib.cascade_decode_step_workspace_size.argtypes = [P, P]
    lib.cascade_decode_step_workspace_size.restype = sz
    lib.cascade_decode_step.argtypes = [P, P, vp, i32, vp, vp, sz, vp]
    lib.cascade_decode_step.restype = ctypes.c_int
    lib.cascade_lse_merge.argtypes = [vp, i32, vp, i32, vp, i64, vp, i64, vp, i32, i64, i64, vp]
    lib.cascade_lse_merge.restype = ctypes.c_int
    lib.cascade_f3_gateup_epilogue.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, vp]
    lib.cascade_f3_gateup_epilogue.restype = ctypes.c_int
    lib.cascade_add_rms_norm_stats.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, ctypes.c_float, vp]
    lib.cascade_add_rms_norm_stats.restype = ctypes.c_int
    lib.cascade_last_error.argtypes = []
    lib.cascade_last_error.restype = ctypes.c_char_p
    lib.cascade_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    lib.cascade_device_error.restype = ctypes.c_int
    lib.cascade_version.argtypes = []
    lib.cascade_version.restype = ctypes.c_int
    lib.cascade_plan_paged_attn.argtypes = [P, i64, i32, ctypes.POINTER(AttnPlan)]
    lib.cascade_plan_paged_attn.restype = ctypes.c_int
    lib.cascade_check_block_table.argtypes = [vp, i64, i64, vp, i64, i64, ctypes.POINTER(i64), ctypes.POINTER(i64)]
    lib.cascade_check_block_table.restype = ctypes.c_int
    lib.cascade_probe_hbm_read.argtypes = [vp, sz, i32, i64, vp, sz, vp]
    lib.cascade_probe_hbm_read.restype = ctypes.c_int
    _lib = lib
    return lib


class CascadeError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def check(rc):
    if rc != OK:
        raise CascadeError(rc, load().cascade_last_error().decode())
    return rc


def last_error():
    return load().cascade_last_error().decode()


def device_error():
    w = ctypes.c_uint32(0)
    check(load().cascade_device_error(ctypes.byref(w)))
    return w.value


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def dtype_code(torch_dtype):
    import torch
    return {torch.bfloat16: BF16, torch.float16: FP16, torch.float32: FP32}[torch_dtype]


FLAG_PARTIALS_ONLY = 1
FLAG_DEBUG_STALL = 2      # test hook: the kernel's bounded waits run out (1 ms) and the call aborts
FLAG_CHECK_BLOCK_IDS = 4  # debug mode: read the block table back and check it before launching


def paged_desc(query, key, value, block_table, q_seqlens, kv_seqlens, q_seqlen_value=0, *,
               shape=None, dtype=None, flags=0):
    """Build the C descriptor from device tensors (or from explicit shapes when
    ``shape`` = dict of sizes is given and the tensors are None)."""
    d = PagedAttn()
    if shape is None:
        d.query, d.key, d.value = query.data_ptr(), key.data_ptr(), value.data_ptr()
        d.block_table = block_table.data_ptr()
        d.actual_q_seqlens, d.actual_kv_seqlens = q_seqlens.data_ptr(), kv_seqlens.data_ptr()
        d.num_tokens, d.num_heads, d.head_dim = query.shape
        d.num_blocks, d.block_size, d.kv_heads = key.shape[0], key.shape[1], key.shape[2]
        d.batch = q_seqlens.numel()
        d.block_cols = block_table.shape[1]
        d.dtype = dtype_code(query.dtype)
    else:
        for k, v in shape.items():
            setattr(d, k, v)
        d.dtype = BF16 if dtype is None else dtype
    d.q_seqlen_value = q_seqlen_value
    d.flags = flags
    return d


def plan(desc, max_q, suffix=False):
    p = AttnPlan()
    check(load().cascade_plan_paged_attn(ctypes.byref(desc), max_q, int(suffix), ctypes.byref(p)))
    return p


def check_block_table(bt, kv_lens, block_size, num_blocks):
    """Host-side paging-contract check (cascade_check_block_table) of numpy
    arrays: bt int32 [rows, cols], kv_lens int64 [rows]. Returns None, or
    raises CascadeError whose ``bad`` attribute is the first offending
    (row, column)."""
    import numpy as np
    bt = np.ascontiguousarray(bt, dtype=np.int32)
    kv = np.ascontiguousarray(kv_lens, dtype=np.int64)
    rows, cols = bt.shape
    r, c = ctypes.c_int64(-1), ctypes.c_int64(-1)
    rc = load().cascade_check_block_table(bt.ctypes.data, rows, cols, kv.ctypes.data, int(block_size),
                                          int(num_blocks), ctypes.byref(r), ctypes.byref(c))
    if rc != OK:
        err = CascadeError(rc, load().cascade_last_error().decode())
        err.bad = (r.value, c.value)
        raise err


def probe_hbm_read(src, mode, row_bytes=0, sink=None, stream=None):
    """cascade_probe_hbm_read over the bytes of device tensor ``src``."""
    import torch
    if sink is None:
        sink = torch.zeros(2048, dtype=torch.int32, device=src.device)
    return check(load().cascade_probe_hbm_read(
        _ptr(src), src.numel() * src.element_size(), int(mode), int(row_bytes), _ptr(sink), sink.numel(),
        stream_ptr(stream)))


def stream_ptr(stream=None):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)


def fa_fp32_stage1(desc, out, lse, workspace=None, stream=None):
    """Call cascade_fa_fp32_stage1 through the C ABI (out/lse/workspace are
    preallocated device tensors)."""
    lib = load()
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    return check(lib.cascade_fa_fp32_stage1(ctypes.byref(desc), _ptr(out), _ptr(lse), _ptr(workspace),
                                            ws_bytes, stream_ptr(stream)))


def suffix_decode(desc, out, lse, workspace=None, stream=None):
    lib = load()
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    return check(lib.cascade_suffix_decode(ctypes.byref(desc), _ptr(out), _ptr(lse), _ptr(workspace),
                                           ws_bytes, stream_ptr(stream)))


def suffix_decode_noalloc(desc, out, lse, stream=None):
    """The allocation-free suffix decode (fixed 16 MiB scratch inside the library)."""
    return check(load().cascade_suffix_decode_noalloc(ctypes.byref(desc), _ptr(out), _ptr(lse),
                                                      stream_ptr(stream)))


def decode_step(prefix, suffix, out, lse_out=None, workspace=None, stream=None):
    """cascade_decode_step through the C ABI (out in its own dtype)."""
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    return check(load().cascade_decode_step(ctypes.byref(prefix), ctypes.byref(suffix), _ptr(out),
                                            dtype_code(out.dtype), _ptr(lse_out), _ptr(workspace), ws_bytes,
                                            stream_ptr(stream)))


def decode_step_workspace_size(prefix, suffix):
    return load().cascade_decode_step_workspace_size(ctypes.byref(prefix), ctypes.byref(suffix))


def stage1_workspace_size(desc):
    return load().cascade_fa_fp32_stage1_workspace_size(ctypes.byref(desc))


def suffix_workspace_size(desc):
    return load().cascade_suffix_decode_workspace_size(ctypes.byref(desc))


def lse_merge(o1, o2, lse1, stride1, lse2, stride2, out, rows, dim, stream=None):
    return check(load().cascade_lse_merge(
        _ptr(o1), dtype_code(o1.dtype), _ptr(o2), dtype_code(o2.dtype), _ptr(lse1), stride1,
        _ptr(lse2), stride2, _ptr(out), dtype_code(out.dtype), rows, dim, stream_ptr(stream)))


def gateup(a, b, ws, d, d_stride, M, K, I, mode, stream=None):
    return check(load().cascade_f3_gateup_epilogue(
        _ptr(a), _ptr(b), _ptr(ws), _ptr(d), d_stride, M, K, I, mode, stream_ptr(stream)))


def add_rms_norm_stats(x1, x2, gamma, beta, x_out, rstd, y, M, K, mode, eps, stream=None):
    """cascade_add_rms_norm_stats through the C ABI (dtype taken from x1)."""
    return check(load().cascade_add_rms_norm_stats(
        _ptr(x1), _ptr(x2), _ptr(gamma), _ptr(beta), _ptr(x_out), _ptr(rstd), _ptr(y), M, K,
        dtype_code(x1.dtype), mode, eps, stream_ptr(stream)))
