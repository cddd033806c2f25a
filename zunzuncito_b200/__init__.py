"""zunzuncito_b200 -- B200 (sm_100a) backend for zunzuncito's quantized matrix hot path.

The product is the C-ABI shared library ``libzz_cuda.so`` built from ``csrc/`` (its
interface is ``include/zz_gpu.h``). This package only loads it and gives Python callers
(tests, the benchmark, host-side plumbing such as the expert-parallel exchange) typed
access to it. There is no CPU fallback: the first use of ``lib`` or of any device entry
point loads the library and raises if it is missing. Importing the package alone (for
example for ``zunzuncito_b200.synth``, the seeded input generators) loads nothing, so a
CPU-only process such as the benchmark's reference arm never maps the product library.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libzz_cuda.so")

GPU_FMT_Q40, GPU_FMT_Q80, GPU_FMT_TQ2, GPU_FMT_Q4A = 1, 2, 3, 4
ZZ_ACT_GEGLU_TANH, ZZ_ACT_SWIGLU, ZZ_ACT_SWIGLU_CLAMP = 0, 1, 2

c_void_p, c_int, c_size_t, c_float, c_int64 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t,
                                               ctypes.c_float, ctypes.c_int64)


class QTensor(ctypes.Structure):
    """zz_qtensor: one weight tensor as structure-of-arrays planes in HBM."""
    _fields_ = [("fmt", c_int), ("O", c_int), ("I", c_int), ("codes", c_void_p), ("scale", c_void_p)]


class ExpertBank(ctypes.Structure):
    """zz_expert_bank: one MoE layer's routed experts, packed for the batch-union FFN."""
    _fields_ = [("fmt", c_int), ("n_experts", c_int), ("hidden", c_int), ("inter", c_int),
                ("gu_codes", c_void_p), ("gu_scale", c_void_p), ("dn_codes", c_void_p),
                ("dn_scale", c_void_p)]


# (name, restype, argtypes): every entry point of include/zz_gpu.h
_PROTOS = [
    ("gpu_init", c_int, []),
    ("gpu_shutdown", None, []),
    ("gpu_ready", c_int, []),
    ("gpu_name", ctypes.c_char_p, []),
    ("gpu_map", c_int, [c_void_p, c_size_t]),
    ("gpu_unmap", c_int, [c_void_p]),
    ("gpu_q40_matmul", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    ("gpu_matmul", c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    ("gpu_last_error", ctypes.c_char_p, []),
    ("zz_gpu_set_act_quant", c_int, [c_int]),
    ("gpu_q40_matvec", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    ("gpu_q80_matvec", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    ("gpu_tq2_matvec", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int, c_int]),
    ("gpu_q4a_matvec", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    ("zz_matvec_f32_dev", c_int, [ctypes.POINTER(QTensor), c_void_p, c_void_p, c_int, c_void_p]),
    ("zz_qtensor_bytes", c_size_t, [c_int, c_int, c_int]),
    ("zz_repack_dev", c_int, [c_int, c_void_p, c_int, c_int, c_void_p, ctypes.POINTER(QTensor), c_void_p]),
    ("zz_unpack_dev", c_int, [ctypes.POINTER(QTensor), c_void_p, c_void_p]),
    ("zz_quant_rows_dev", c_int, [c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    ("zz_quant_act_dev", c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("zz_matvec_dev", c_int, [ctypes.POINTER(QTensor), c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    ("zz_lm_head_dev", c_int, [ctypes.POINTER(QTensor), c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p]),
    ("zz_blocksums_dev", c_int, [ctypes.POINTER(QTensor), c_void_p, c_void_p, c_void_p]),
    ("zz_route_gemma4_dev", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_float,
                                    c_void_p, c_void_p, c_void_p]),
    ("zz_route_ling_dev", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    ("zz_container_open", c_int, [ctypes.c_char_p, ctypes.POINTER(c_void_p)]),
    ("zz_container_close", None, [c_void_p]),
    ("zz_container_cfg", c_int, [c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    ("zz_container_dense_info", c_int, [c_void_p, ctypes.c_char_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                        ctypes.POINTER(c_int), ctypes.POINTER(c_int64), ctypes.POINTER(c_int64)]),
    ("zz_container_expert_offset", c_int64, [c_void_p, c_int, c_int]),
    ("zz_container_bank_bytes", c_size_t, [c_void_p]),
    ("zz_container_load_bank_dev", c_int, [c_void_p, c_int, c_void_p, ctypes.POINTER(ExpertBank), c_void_p]),
    ("zz_container_load_dense_dev", c_int, [c_void_p, ctypes.c_char_p, c_void_p, ctypes.POINTER(QTensor), c_void_p]),
    ("zz_expert_bank_bytes", c_size_t, [c_int, c_int, c_int, c_int]),
    ("zz_expert_bank_pack_dev", c_int, [c_int, c_int, c_int, c_int, c_void_p, c_int64, c_void_p,
                                        ctypes.POINTER(ExpertBank), c_void_p]),
    ("zz_moe_workspace_bytes", c_size_t, [ctypes.POINTER(ExpertBank), c_int, c_int]),
    ("zz_moe_workspace_offset", c_size_t, [ctypes.POINTER(ExpertBank), c_int, c_int, c_int]),
    ("zz_moe_ffn_q8_dev", c_int, [ctypes.POINTER(ExpertBank), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_int, c_int, c_int, c_float, c_void_p, c_size_t, c_int, c_void_p]),
    ("zz_ep_row_bytes", c_size_t, [c_int, c_int]),
    ("zz_ep_pack_dev", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                               c_void_p]),
    ("zz_ep_unpack_dev", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("zz_moe_ffn_noalloc_dev", c_int, [ctypes.POINTER(ExpertBank), c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                       c_int, c_int, c_float, c_void_p]),
    ("zz_prof_enable", c_int, [c_int]),
    ("zz_prof_collect", c_int, [ctypes.POINTER(c_float), ctypes.POINTER(c_int)]),
    ("zz_moe_ffn_dev", c_int, [ctypes.POINTER(ExpertBank), c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                               c_int, c_float, c_void_p, c_size_t, c_int, c_void_p]),
]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python zunzuncito_b200/build.py` "
                          "(this package has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in _PROTOS:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def get_lib():
    """libzz_cuda.so with every prototype set (loaded on first use)."""
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


class ZZError(RuntimeError):
    pass


def check(ok, what=""):
    """Raise with gpu_last_error() when an entry point declined (returned 0)."""
    if not ok:
        msg = get_lib().gpu_last_error().decode()
        raise ZZError(f"{what}: {msg}" if what else msg)
    return ok


_API = None
# the public names of api.py (kept equal to its __all__; a CPU test checks that)
_API_NAMES = frozenset(["ref_row_bytes", "ref_tensor_bytes", "expert_blob_bytes", "quant_act", "quant_rows",
                        "QTensorDev", "matvec", "blocksums", "ExpertBankDev", "moe_ffn", "moe_ffn_q8",
                        "alloc_aligned", "ep_pack", "ep_unpack", "route_gemma4", "route_ling"])


def __getattr__(name):
    # PEP 562: `zz.lib` and the typed wrappers of api.py resolve on first use
    global _API
    if name == "lib":
        return get_lib()
    if name not in _API_NAMES:   # submodules (synth, ep, ...) are imported by the import system
        raise AttributeError(f"module 'zunzuncito_b200' has no attribute {name!r}")
    if _API is None:
        import importlib
        _API = importlib.import_module(__name__ + ".api")
    if name in _API.__all__:
        return getattr(_API, name)
    raise AttributeError(f"module 'zunzuncito_b200' has no attribute {name!r}")
