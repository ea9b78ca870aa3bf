"""ctypes binding of the C ABI in include/megaqwen_b200.h.

The shared library is built in-tree (``megaqwen-a10_b200/lib/libmqb200.so``).
There is no fallback: if the library is missing or fails to load, every entry
point raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libmqb200.so")

MQ_ERRORS = {
    -1: "invalid argument (null, misaligned or bad size)",
    -2: "token id outside [0, vocab)",
    -3: "position outside [0, max_seq_len) or cache_len != position + 1",
    -4: "device unsupported",
    -5: "size larger than the entry point supports",
    -6: "the kernel reported a device-side error",
}
ROW_PAD = 16  # padding bytes after every weight row in the layout the decoder classes use
MQ_DEV_ERRORS = {1: "exchange wait timed out", 2: "weight-ring wait timed out", 3: "invalid token",
                 4: "invalid position", 5: "activation outside the fp16 operand range"}

EXPORTED = (
    "launch_a10_int8_decode", "launch_a10_decode", "mq_decode_multi", "mq_quantize_per_channel",
    "mq_matvec", "mq_device_status", "mq_set_wait_budget_ns", "mq_inject_skip_publish", "mq_kernel_info",
    "mq_set_trace", "launch_a10_int8_decode_static", "mq_batch_workspace_bytes", "mq_batch_decode",
    "mq_batch_status", "mq_pack_weight_tiles", "mq_pack_weight_slabs", "mq_batch_matmul_workspace_bytes", "mq_batch_matmul",
    "mq_library_info", "mq_decode_step_host",
)


class LayerWeights(ctypes.Structure):
    """Field order of config.cuh:45-57."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_layernorm_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight", "q_norm_weight",
        "k_norm_weight", "o_proj_weight", "post_attn_layernorm_weight", "gate_proj_weight",
        "up_proj_weight", "down_proj_weight")]


class ScalePointers(ctypes.Structure):
    """Field order of config.cuh:59-67."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "q_scale", "k_scale", "v_scale", "o_scale", "gate_scale", "up_scale", "down_scale")]


class MQStepPlan(ctypes.Structure):
    """Field order of MQStepPlan (include/megaqwen_b200.h)."""
    _fields_ = [("weight_kind", ctypes.c_int), ("num_layers", ctypes.c_int), ("max_seq_len", ctypes.c_int),
                ("row_pad_bytes", ctypes.c_int), ("attn_scale", ctypes.c_float)] + \
               [(n, ctypes.c_void_p) for n in (
                   "embed_weight", "layer_weights", "final_norm_weight", "lm_head_weight", "lm_head_scale", "scales",
                   "cos_table", "sin_table", "k_cache", "v_cache", "g_normalized", "host_token")]


class MQError(RuntimeError):
    pass


_lib = None
_vp, _i, _f, _i64, _u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64, ctypes.c_uint64


def load():
    """Load the library (once) and declare the prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise MQError(f"CUDA library not built: {LIB_PATH} (run megaqwen-a10_b200/build.py)")
    lib = ctypes.CDLL(LIB_PATH)
    ref_args = [_i, _vp, _vp, _vp, _vp, _vp]  # token, out, embed, layers, final_norm, lm_head
    lib.launch_a10_int8_decode.argtypes = ref_args + [_vp, _vp, _vp] + [_vp] * 3 + [_vp] * 10 + [_i, _i, _i, _i, _f, _vp, _vp]
    lib.launch_a10_decode.argtypes = ref_args + [_vp, _vp] + [_vp] * 3 + [_vp] * 10 + [_i, _i, _i, _i, _f, _vp]
    lib.mq_decode_multi.argtypes = [_i, _i, _vp, _vp, _i] + [_vp] * 13 + [_i, _i, _i, _f, _i, _vp]
    lib.mq_quantize_per_channel.argtypes = [_vp, _i64, _i64, _vp, _vp, _vp]
    lib.mq_matvec.argtypes = [_i, _vp, _vp, _vp, _vp, _i, _i, _vp]
    lib.mq_device_status.argtypes = [ctypes.POINTER(_i), ctypes.POINTER(_i), _i]
    lib.mq_set_wait_budget_ns.argtypes = [_u64]
    lib.mq_inject_skip_publish.argtypes = [_i, _i]
    lib.mq_set_trace.argtypes = [_vp, _i]
    lib.mq_batch_workspace_bytes.argtypes = [_i, ctypes.POINTER(ctypes.c_size_t)]
    lib.mq_batch_decode.argtypes = [_vp, _i, _vp]
    lib.mq_batch_status.argtypes = [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i)]
    lib.mq_pack_weight_tiles.argtypes = [_vp, _i64, _i, _i64, _vp, _vp]
    lib.mq_pack_weight_slabs.argtypes = [_vp, _i64, _i, _i64, _i, _vp, _vp]
    lib.mq_batch_matmul_workspace_bytes.argtypes = [_i, ctypes.POINTER(ctypes.c_size_t)]
    lib.mq_batch_matmul.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, ctypes.c_size_t, _vp]
    lib.launch_a10_int8_decode_static.argtypes = [_i] + [_vp] * 11 + [_i, _i, _i, _i, _f, _vp, _vp]
    lib.mq_kernel_info.argtypes = [ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]
    lib.mq_library_info.argtypes = [ctypes.POINTER(_i), ctypes.POINTER(_i)]
    lib.mq_decode_step_host.argtypes = [ctypes.POINTER(MQStepPlan), _i, _i, _vp, ctypes.POINTER(_i)]
    for name in EXPORTED:
        getattr(lib, name).restype = _i
    _lib = lib
    return lib


def check(rc, what):
    if rc == 0:
        return
    if rc < 0:
        raise MQError(f"{what}: {MQ_ERRORS.get(rc, rc)}")
    raise MQError(f"{what}: CUDA error {rc}")


def device_status(clear=False):
    """(code, info) of the device-side error word (MQ_DEV_*); synchronises."""
    code, info = _i(0), _i(0)
    check(load().mq_device_status(ctypes.byref(code), ctypes.byref(info), 1 if clear else 0), "mq_device_status")
    return code.value, info.value


def raise_device_error(what):
    code, info = device_status(clear=True)
    if code:
        raise MQError(f"{what}: device error {code} ({MQ_DEV_ERRORS.get(code, '?')}, at {info})")


def set_wait_budget_ns(ns):
    check(load().mq_set_wait_budget_ns(int(ns)), "mq_set_wait_budget_ns")


def inject_skip_publish(enable, cta=0):
    check(load().mq_inject_skip_publish(1 if enable else 0, int(cta)), "mq_inject_skip_publish")


def library_info():
    """{"binary_version": decode kernel binaryVersion, "workspace_allocated": bool} on the current device."""
    a, b = _i(0), _i(0)
    check(load().mq_library_info(ctypes.byref(a), ctypes.byref(b)), "mq_library_info")
    return {"binary_version": a.value, "workspace_allocated": bool(b.value)}


def kernel_info():
    a, b, c = _i(0), _i(0), _i(0)
    load().mq_kernel_info(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    return {"num_ctas": a.value, "smem_bytes": b.value, "threads": c.value}


def set_trace(buf=None, slots_per_cta=0):
    """buf: device int64 tensor [num_ctas, slots_per_cta], or None to disable."""
    ptr = ctypes.c_void_p(buf.data_ptr() if buf is not None else 0)
    check(load().mq_set_trace(ptr, int(slots_per_cta) if buf is not None else 0), "mq_set_trace")
