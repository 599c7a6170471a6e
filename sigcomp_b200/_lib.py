"""ctypes binding of libsigcomp_b200.so (the C ABI in include/sigcomp_b200.h).

The shared library is built in-tree (``sigcomp_b200/libsigcomp_b200.so``) by
``sigcomp_b200.build_ext``.  There is no fallback: if the library is missing
or fails to load, every codec entry point raises.
"""

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsigcomp_b200.so"

SC_OK = 0
SC_ERR_INVALID_ARGUMENT = 1
SC_ERR_CAPACITY = 2
SC_ERR_CORRUPT_STREAM = 3
SC_ERR_CUDA = 4
SC_ERR_UNSUPPORTED = 5
SC_ERR_OUT_OF_MEMORY = 6

EXPORTS = (
    "sc_version", "sc_last_error", "sc_kernel_launches", "sc_model_create", "sc_model_destroy",
    "sc_model_set_mlp_path", "sc_compress_chunks", "sc_compress_chunks_device", "sc_decompress_chunks",
    "sc_decompress_chunks_device", "sc_mlp_logits_device", "sc_profile_enable", "sc_profile_read",
    "sc_trace_enable", "sc_trace_read", "sc_mlp_logits_device_noalloc", "sc_split_signal_device",
    "sc_reassemble_signal_device", "sc_selftest_wait_timeout", "sc_encode_logits_device",
    "sc_decode_logits_device", "sc_frame_reads", "sc_unframe_reads", "sc_linear_layer_device",
)

KERNEL_KINDS = ("windows", "layer0", "hidden", "last_layer", "cdf_select", "encode", "compact", "decode_step",
                "fused_compress", "fused_decode", "small_decode", "split", "reassemble")

_lib = None


class CodecError(RuntimeError):
    pass


def load():
    """Load the library (once) and declare the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m sigcomp_b200.build_ext`")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    L.sc_version.restype = ctypes.c_char_p
    L.sc_last_error.restype = ctypes.c_char_p
    L.sc_kernel_launches.restype = i64
    L.sc_model_create.argtypes = [ctypes.c_int, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32,
                                  ctypes.POINTER(vp)]
    L.sc_model_destroy.argtypes = [vp]
    L.sc_model_set_mlp_path.argtypes = [vp, i32]
    L.sc_compress_chunks.argtypes = [vp, vp, vp, i64, vp, i64, vp, vp, vp]
    L.sc_compress_chunks_device.argtypes = [vp, vp, vp, i64, vp, i64, vp, vp, vp]
    L.sc_decompress_chunks.argtypes = [vp, vp, vp, vp, i64, vp, vp, vp]
    L.sc_decompress_chunks_device.argtypes = [vp, vp, vp, vp, vp, i64, vp, vp, vp]
    L.sc_mlp_logits_device.argtypes = [vp, vp, i64, vp, vp]
    L.sc_encode_logits_device.argtypes = [vp, vp, vp, vp, i64, vp, i64, vp, vp, vp]
    L.sc_decode_logits_device.argtypes = [vp, vp, vp, vp, vp, i64, vp, vp, vp]
    L.sc_frame_reads.argtypes = [vp, vp, vp, i64, vp, i64, vp]
    L.sc_linear_layer_device.argtypes = [vp, i32, vp, i64, vp, vp]
    L.sc_unframe_reads.argtypes = [vp, vp, vp, i64, i32, vp, i64, vp, vp, i64, vp, vp]
    L.sc_profile_enable.argtypes = [vp, i32]
    L.sc_profile_read.argtypes = [vp, i32, vp, vp, vp]
    L.sc_trace_enable.argtypes = [vp, i32]
    L.sc_trace_enable.restype = ctypes.c_int
    L.sc_trace_read.argtypes = [vp, i32, vp, i64]
    L.sc_trace_read.restype = i64
    for name in EXPORTS:
        getattr(L, name)
    for name in ("sc_model_create", "sc_model_destroy", "sc_model_set_mlp_path", "sc_compress_chunks",
                 "sc_compress_chunks_device", "sc_decompress_chunks", "sc_decompress_chunks_device",
                 "sc_mlp_logits_device", "sc_mlp_logits_device_noalloc", "sc_profile_enable",
                 "sc_profile_read", "sc_split_signal_device", "sc_reassemble_signal_device",
                 "sc_selftest_wait_timeout", "sc_encode_logits_device", "sc_decode_logits_device",
                 "sc_frame_reads", "sc_unframe_reads", "sc_linear_layer_device"):
        getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


def profile_enable(handle, on=True):
    check(load().sc_profile_enable(handle, 1 if on else 0), "sc_profile_enable")


def profile_read(handle):
    """{kind: (total_ms, launches, work)} for every kernel class."""
    out = {}
    for k, name in enumerate(KERNEL_KINDS):
        ms, n, w = ctypes.c_double(), ctypes.c_int64(), ctypes.c_int64()
        check(load().sc_profile_read(handle, k, ctypes.byref(ms), ctypes.byref(n), ctypes.byref(w)))
        out[name] = (ms.value, n.value, w.value)
    return out


def last_error():
    return load().sc_last_error().decode(errors="replace")


def kernel_launches():
    return int(load().sc_kernel_launches())


def check(rc, what="sigcomp_b200"):
    """Map a status code to the exception the reference codec raises."""
    if rc == SC_OK:
        return
    msg = last_error() or what
    if rc == SC_ERR_INVALID_ARGUMENT or rc == SC_ERR_CORRUPT_STREAM:
        raise ValueError(msg)
    if rc == SC_ERR_CAPACITY:
        raise OverflowError(msg)
    if rc == SC_ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    raise CodecError(f"{what}: {msg} (status {rc})")
