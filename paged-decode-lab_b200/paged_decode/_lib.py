"""ctypes binding of the C ABI in ``include/pdl_b200.h`` (``libpdl_b200.so``).

The shared library is built in-tree by ``csrc/build.py``.  There is no
fallback: if it is missing or stale, every op raises instead of computing
anything another way.
"""
import ctypes
from pathlib import Path

LIBRARY = Path(__file__).with_name("libpdl_b200.so")
ABI_VERSION = 5

PDL_OK = 0
STATUS_NAMES = {
    0: "PDL_OK", 1: "PDL_ERR_NULL", 2: "PDL_ERR_GEOMETRY", 3: "PDL_ERR_SHAPE",
    4: "PDL_ERR_WORKSPACE", 5: "PDL_ERR_SCALE", 6: "PDL_ERR_ALIGNMENT", 7: "PDL_ERR_SPLITS",
    8: "PDL_ERR_CUDA", 9: "PDL_ERR_DEVICE", 10: "PDL_ERR_KERNEL", 11: "PDL_ERR_TIMEOUT",
}
PROTOCOL_LSE, PROTOCOL_MLA = 0, 1
KERNEL_AUTO, KERNEL_SIMT, KERNEL_MMA = 0, 1, 2
FLAG_SKIP_EMPTY, FLAG_DIRECT_SINGLE, FLAG_DYNAMIC, FLAG_BALANCED = 1, 2, 8, 16

# Every extern "C" symbol declared in include/pdl_b200.h.
SYMBOLS = ("pdl_partition", "pdl_merge", "pdl_lse_merge", "pdl_paged_decode", "pdl_append_kv",
           "pdl_paged_decode_static_scratch", "pdl_splitkv_plan", "pdl_b200_plan",
           "pdl_spec_geometry", "pdl_exchange_plan", "pdl_peer_buffer_create",
           "pdl_peer_buffer_open", "pdl_peer_buffer_close", "pdl_peer_buffer_free",
           "pdl_exchange_merge",
           "pdl_status_string", "pdl_last_error", "pdl_abi_version", "pdl_read_fault")
STATIC_SCRATCH_BYTES = 4 << 20
MAX_PEERS = 8
FAULT_EXCHANGE_WAIT = 1 << 4

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class PdlSpec(ctypes.Structure):
    _fields_ = [("max_batch", _i32), ("num_heads", _i32), ("num_kv_heads", _i32),
                ("head_dim", _i32), ("max_context_len", _i32), ("page_size", _i32)]


class PdlPlan(ctypes.Structure):
    _fields_ = [("splits", _i32), ("tile_tokens", _i32), ("tokens_per_split", _i32),
                ("table_capacity_tokens", _i32), ("lse_lanes", _i32), ("sm_count", _i32),
                ("explicit_splits", _i32), ("balanced", _i32)]


class PdlDecodeArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("q_stride_batch", _i64), ("q_stride_head", _i64),
                ("k_cache", _vp), ("v_cache", _vp), ("num_pages", _i64),
                ("block_table", _vp), ("table_stride", _i64), ("table_width", _i32),
                ("lengths", _vp), ("batch", _i32), ("num_heads", _i32),
                ("num_kv_heads", _i32), ("head_dim", _i32), ("scale", _f32),
                ("tokens_per_split", _i32), ("splits", _i32), ("protocol", _i32),
                ("kernel", _i32), ("flags", _i32), ("out", _vp), ("partial", _vp),
                ("lse", _vp), ("maxima", _vp), ("denoms", _vp), ("accums", _vp),
                ("counters", _vp)]


class PdlAppendArgs(ctypes.Structure):
    _fields_ = [("key", _vp), ("value", _vp), ("key_stride_token", _i64),
                ("key_stride_head", _i64), ("value_stride_token", _i64),
                ("value_stride_head", _i64), ("k_cache", _vp), ("v_cache", _vp),
                ("num_pages", _i64), ("n_tokens", _i32), ("num_kv_heads", _i32),
                ("head_dim", _i32), ("slot_mapping", _vp), ("block_table", _vp),
                ("table_stride", _i64), ("table_width", _i32), ("lengths", _vp),
                ("increment_lengths", _i32)]


class PdlMergeArgs(ctypes.Structure):
    _fields_ = [("partial", _vp), ("lse", _vp), ("row_stride", _i64), ("part_stride", _i64),
                ("lse_row_stride", _i64), ("lse_part_stride", _i64), ("rows", _i32),
                ("parts", _i32), ("head_dim", _i32), ("out", _vp), ("out_partial", _vp),
                ("out_lse", _vp)]


class PdlIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class PdlExchangePlan(ctypes.Structure):
    _fields_ = [("ctas", _i32), ("reserved", _i32), ("block_words", _i64),
                ("data_offset", _i64), ("buffer_bytes", _i64)]


class PdlExchangeArgs(ctypes.Structure):
    _fields_ = [("partial", _vp), ("lse", _vp), ("lengths", _vp), ("num_heads", _i32),
                ("tokens_per_split", _i32), ("rows", _i32), ("parts", _i32),
                ("head_dim", _i32), ("rank", _i32), ("world", _i32), ("emulate_ranks", _i32),
                ("timeout_us", ctypes.c_uint32), ("buffers", _vp * 8), ("out", _vp)]


_LIB = None


def load():
    """Load the library once; raise with a build hint when it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY.exists():
        raise RuntimeError(
            f"paged-decode CUDA library not found at {LIBRARY}; build it with "
            "`python paged-decode-lab_b200/csrc/build.py` (no CPU fallback exists)")
    lib = ctypes.CDLL(str(LIBRARY))
    args_p = ctypes.POINTER(PdlDecodeArgs)
    for name in ("pdl_partition", "pdl_merge", "pdl_paged_decode",
                 "pdl_paged_decode_static_scratch"):
        fn = getattr(lib, name)
        fn.argtypes = [args_p, ctypes.c_size_t]  # stream handle as an integer
        fn.restype = ctypes.c_int
    lib.pdl_append_kv.argtypes = [ctypes.POINTER(PdlAppendArgs), ctypes.c_size_t]
    lib.pdl_append_kv.restype = ctypes.c_int
    lib.pdl_lse_merge.argtypes = [ctypes.POINTER(PdlMergeArgs), ctypes.c_size_t]
    lib.pdl_lse_merge.restype = ctypes.c_int
    lib.pdl_splitkv_plan.argtypes = [ctypes.POINTER(PdlSpec), _i32, _i32, ctypes.POINTER(PdlPlan)]
    lib.pdl_splitkv_plan.restype = ctypes.c_int
    lib.pdl_b200_plan.argtypes = [ctypes.POINTER(PdlSpec), _i32, ctypes.POINTER(PdlPlan)]
    lib.pdl_b200_plan.restype = ctypes.c_int
    lib.pdl_spec_geometry.argtypes = [ctypes.POINTER(PdlSpec), ctypes.POINTER(_i32),
                                      ctypes.POINTER(_i32), ctypes.POINTER(_i64)]
    lib.pdl_spec_geometry.restype = ctypes.c_int
    lib.pdl_exchange_plan.argtypes = [_i32, _i32, _i32, _i32, _i32,
                                      ctypes.POINTER(PdlExchangePlan)]
    lib.pdl_exchange_plan.restype = ctypes.c_int
    lib.pdl_peer_buffer_create.argtypes = [_i64, ctypes.POINTER(_vp), ctypes.POINTER(PdlIpcHandle)]
    lib.pdl_peer_buffer_create.restype = ctypes.c_int
    lib.pdl_peer_buffer_open.argtypes = [ctypes.POINTER(PdlIpcHandle), ctypes.POINTER(_vp)]
    lib.pdl_peer_buffer_open.restype = ctypes.c_int
    for name in ("pdl_peer_buffer_close", "pdl_peer_buffer_free"):
        getattr(lib, name).argtypes = [_vp]
        getattr(lib, name).restype = ctypes.c_int
    lib.pdl_exchange_merge.argtypes = [ctypes.POINTER(PdlExchangeArgs), ctypes.c_size_t]
    lib.pdl_exchange_merge.restype = ctypes.c_int
    lib.pdl_status_string.argtypes = [ctypes.c_int]
    lib.pdl_status_string.restype = ctypes.c_char_p
    lib.pdl_last_error.argtypes = []
    lib.pdl_last_error.restype = ctypes.c_char_p
    lib.pdl_abi_version.argtypes = []
    lib.pdl_abi_version.restype = ctypes.c_int
    lib.pdl_read_fault.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
    lib.pdl_read_fault.restype = ctypes.c_int
    version = lib.pdl_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"{LIBRARY} has ABI {version}, expected {ABI_VERSION}; rebuild it")
    _LIB = lib
    return lib


def status_text(status):
    lib = load()
    text = f"{STATUS_NAMES.get(status, status)}: {lib.pdl_status_string(status).decode()}"
    detail = lib.pdl_last_error().decode()
    return f"{text} ({detail})" if detail else text


def make_spec(spec):
    return PdlSpec(spec.max_batch, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                   spec.max_context_len, spec.page_size)


def read_fault(clear=False):
    """Sticky device-side fault word of the current device (synchronises)."""
    word = ctypes.c_uint32(0)
    status = load().pdl_read_fault(ctypes.byref(word), int(clear))
    if status != PDL_OK:
        raise RuntimeError(f"pdl_read_fault failed: {status_text(status)}")
    return word.value
