"""ctypes bindings of libp0mm.so (the C ABI declared in include/p0mm.h).

The library is the product; this module only loads it and declares the structs. It fails loudly when the
library is missing: there is no CPU or library fallback behind these entry points.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libp0mm.so")

# status codes (p0_status)
P0_OK, P0_EINVAL, P0_EALIGN, P0_ENOMEM, P0_EDEVICE, P0_ETIMEOUT, P0_ECOMM = range(7)
STATUS = {0: "P0_OK", 1: "P0_EINVAL", 2: "P0_EALIGN", 3: "P0_ENOMEM", 4: "P0_EDEVICE", 5: "P0_ETIMEOUT", 6: "P0_ECOMM"}
ENC = {"q4g32a.t64": 1, "q8g64s.t64": 2, "f16": 3}
PRO = {"raw": 0, "rms": 1, "sum": 2, "pleg": 3}
EPI = {"store": 0, "geglu": 1, "softcap": 2}
GEPI = {"f16": 0, "f32": 1, "bias": 2, "resadd": 3, "swiglu": 4, "heads": 5, "onormgate": 6}
ACT = {"silu": 0, "gelu": 1}
XPRO = {"f16": 0, "lnmod": 1, "rms": 2}
P0_ROPE_INTER, P0_ROPE_HALF = 0, 1

# every symbol include/p0mm.h declares
EXPORTS = ["p0_init", "p0_destroy", "p0_set_stream", "p0_set_overlap", "p0_last_error", "p0_stats", "p0_buffer", "p0_wrap", "p0_upload", "p0_read",
           "p0_free", "p0_done", "p0_device_ptr", "p0_gemv", "p0_gemvM", "p0_gemvM_noalloc", "p0_gemm", "p0_pack_q4", "p0_pack_q8",
           "p0_dequant_f16", "p0_version", "p0_argmaxM", "p0_embed", "p0_normadd", "p0_dhead",
           "p0_upload_file", "p0_qkrope", "p0_attn_dec", "p0_wait_selftest",
           "p0_chain_begin", "p0_chain_end", "p0_chain_run", "p0_chain_info", "p0_chain_free", "p0_copy"]
P0_NOALLOC_SCRATCH_BYTES = 16 << 20   # include/p0mm.h
P0_OVERLAP_WEIGHTS = 1
P0_NOALLOC_COUNTER_BYTES = 64 << 10


class p0_buf(ctypes.Structure):
    _fields_ = [("id", ctypes.c_uint64)]


class p0_wview(ctypes.Structure):
    _fields_ = [("buf", p0_buf), ("off", ctypes.c_uint64), ("bytes", ctypes.c_uint64), ("enc", ctypes.c_uint32),
                ("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32), ("ld", ctypes.c_uint32)]


_u32 = ctypes.c_uint32


class p0_gemv_args(ctypes.Structure):
    _fields_ = [("w", p0_wview), ("x", p0_buf), ("x_rowB", _u32), ("N", _u32), ("K", _u32), ("kPer", _u32), ("pro", _u32),
                ("epi", _u32), ("y", p0_buf), ("ldy", _u32), ("stat", p0_buf), ("stat_off", _u32), ("norm", p0_buf),
                ("norm_off", _u32), ("ev", p0_buf), ("ev_off", _u32), ("src_n", _u32), ("src_ld", _u32), ("mx", p0_buf),
                ("cap", ctypes.c_float)]


class p0_gemvM_args(ctypes.Structure):
    _fields_ = [("w", p0_wview), ("x", p0_buf), ("x_rowB", _u32), ("x_ldx", _u32), ("M", _u32), ("N", _u32), ("K", _u32),
                ("kPer", _u32), ("pro", _u32), ("epi", _u32), ("y", p0_buf), ("ldy", _u32), ("ldm", _u32), ("stat", p0_buf),
                ("stat_off", _u32), ("stat_ld", _u32), ("norm", p0_buf), ("norm_off", _u32), ("ev", p0_buf), ("ev_off", _u32),
                ("ev_ld", _u32), ("src_n", _u32), ("src_ld", _u32), ("mx", p0_buf), ("cap", ctypes.c_float)]


class p0_gemm_args(ctypes.Structure):
    _fields_ = [("w", p0_wview), ("x", p0_buf), ("x_off", ctypes.c_uint64), ("x_ld", _u32), ("x_k0", _u32), ("M", _u32),
                ("N", _u32), ("K", _u32), ("wr0", _u32), ("wr1", _u32), ("wk0", _u32), ("epi", _u32), ("act", _u32), ("acc", _u32),
                ("y", p0_buf), ("y_off", ctypes.c_uint64), ("y_ld", _u32), ("y_n0", _u32), ("ev", p0_buf), ("ev_off", _u32),
                ("bv", p0_buf), ("bv_off", _u32), ("bv_up", _u32), ("res", _u32), ("store", _u32), ("post_gelu", _u32),
                ("x_mode", _u32), ("stats", p0_buf), ("stats_off", _u32), ("pv", p0_buf), ("pv_off", _u32), ("pv_stride", _u32),
                ("h_Ltot", _u32), ("h_Hq", _u32), ("h_Hkv", _u32), ("h_rowOff", _u32), ("h_eps", ctypes.c_float),
                ("h_rope_mode", _u32), ("rope", p0_buf), ("gt", p0_buf)]



class p0_embed_args(ctypes.Structure):
    _fields_ = [("w", p0_wview), ("ids", p0_buf), ("x", p0_buf), ("st", p0_buf), ("st_off", _u32), ("K", _u32), ("n", _u32),
                ("rowOut", _u32), ("scale", ctypes.c_float), ("eps", ctypes.c_float)]


class p0_normadd_args(ctypes.Structure):
    _fields_ = [("t", p0_buf), ("t_n", _u32), ("t_ld", _u32), ("w", p0_buf), ("w_off", _u32), ("x", p0_buf), ("st", p0_buf),
                ("st_off", _u32), ("D", _u32), ("M", _u32), ("mode", _u32), ("eps", ctypes.c_float), ("scale", ctypes.c_float)]


class p0_dhead_args(ctypes.Structure):
    _fields_ = [("w", p0_wview), ("x", p0_buf), ("stat", p0_buf), ("stat_off", _u32), ("norm", p0_buf), ("norm_off", _u32),
                ("sel", p0_buf), ("mx", p0_buf), ("K", _u32), ("tPer", _u32), ("nsel", _u32)]



class p0_qkrope_args(ctypes.Structure):
    _fields_ = [("s", p0_buf), ("s_n", _u32), ("s_ld", _u32), ("norm", p0_buf), ("qw", _u32), ("kw", _u32), ("rope", p0_buf),
                ("rope_off", _u32), ("npairs", _u32), ("pos", _u32), ("q", p0_buf), ("kc", p0_buf), ("vc", p0_buf), ("D", _u32),
                ("nq", _u32), ("nkv", _u32), ("hasKV", _u32), ("kvRow", _u32), ("kvLen", _u32), ("eps", ctypes.c_float)]


class p0_attn_dec_args(ctypes.Structure):
    _fields_ = [("q", p0_buf), ("kc", p0_buf), ("vc", p0_buf), ("part", p0_buf), ("out", p0_buf), ("D", _u32), ("nh", _u32),
                ("nkv", _u32), ("kvLen", _u32), ("kStart", _u32), ("kEnd", _u32), ("ring", _u32)]


_lib = None


def load():
    """Load libp0mm.so (built in-tree by p0pc0rn_b200.build). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libp0mm.so is not built (run python -m p0pc0rn_b200.build): no fallback exists")
    L = ctypes.CDLL(LIB_PATH)
    vp, st = ctypes.c_void_p, ctypes.c_int
    L.p0_init.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
    L.p0_destroy.argtypes = [vp]
    L.p0_set_stream.argtypes = [vp, vp]
    L.p0_set_overlap.argtypes = [vp, ctypes.c_uint32]
    L.p0_last_error.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
    L.p0_stats.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
    L.p0_buffer.argtypes = [vp, ctypes.c_size_t, ctypes.c_char_p, ctypes.POINTER(p0_buf)]
    L.p0_wrap.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_char_p, ctypes.POINTER(p0_buf)]
    L.p0_upload.argtypes = [vp, p0_buf, ctypes.c_size_t, vp, ctypes.c_size_t]
    L.p0_read.argtypes = [vp, p0_buf, ctypes.c_size_t, ctypes.c_size_t, vp]
    L.p0_free.argtypes = [vp, p0_buf]
    L.p0_done.argtypes = [vp, ctypes.c_uint32]
    L.p0_device_ptr.argtypes = [vp, p0_buf, ctypes.POINTER(ctypes.c_uint64)]
    L.p0_gemv.argtypes = [vp, ctypes.POINTER(p0_gemv_args), ctypes.POINTER(ctypes.c_uint32)]
    L.p0_gemvM.argtypes = [vp, ctypes.POINTER(p0_gemvM_args), ctypes.POINTER(ctypes.c_uint32)]
    L.p0_gemvM_noalloc.argtypes = [vp, ctypes.POINTER(p0_gemvM_args), ctypes.POINTER(ctypes.c_uint32)]
    L.p0_gemm.argtypes = [vp, ctypes.POINTER(p0_gemm_args), ctypes.POINTER(ctypes.c_double)]
    L.p0_pack_q4.argtypes = [vp, p0_buf, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, p0_buf, ctypes.c_uint64]
    L.p0_pack_q8.argtypes = [vp, p0_buf, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, p0_buf, ctypes.c_uint64]
    L.p0_dequant_f16.argtypes = [vp, ctypes.POINTER(p0_wview), p0_buf]
    L.p0_upload_file.argtypes = [vp, p0_buf, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64]
    L.p0_qkrope.argtypes = [vp, ctypes.POINTER(p0_qkrope_args)]
    L.p0_attn_dec.argtypes = [vp, ctypes.POINTER(p0_attn_dec_args)]
    L.p0_argmaxM.argtypes = [vp, p0_buf, ctypes.c_uint32, ctypes.c_uint32, p0_buf]
    L.p0_embed.argtypes = [vp, ctypes.POINTER(p0_embed_args)]
    L.p0_normadd.argtypes = [vp, ctypes.POINTER(p0_normadd_args)]
    L.p0_dhead.argtypes = [vp, ctypes.POINTER(p0_dhead_args)]
    L.p0_wait_selftest.argtypes = [vp, ctypes.c_uint32]
    L.p0_copy.argtypes = [vp, p0_buf, ctypes.c_size_t, p0_buf, ctypes.c_size_t, ctypes.c_size_t]
    L.p0_chain_begin.argtypes = [vp]
    L.p0_chain_end.argtypes = [vp, ctypes.POINTER(vp)]
    L.p0_chain_run.argtypes = [vp, vp]
    L.p0_chain_info.argtypes = [vp, vp] + [ctypes.POINTER(ctypes.c_uint32)] * 4
    L.p0_chain_free.argtypes = [vp, vp]
    L.p0_version.restype = ctypes.c_char_p
    for name in EXPORTS:
        if name != "p0_version":
            getattr(L, name).restype = st
    _lib = L
    return L
