"""TEST INFRASTRUCTURE ONLY -- the CPU checkers for the CUDA hot path.

Two libraries with one calling convention (numpy in, numpy out):
  ORC  _build/liboracle.so  the scalar restatement in zz_oracle.c
  REF  _ref/libzzref.so     the reference's own gemma4.c / maple.c TUs (and q40.h /
                            tq2.h through them), compiled from the reference sources
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libzzref.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


def build():
    """make -C oracle: the restatement always, the reference build where REF exists."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


class _Lib:
    def __init__(self, path, prefix):
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix

    def fn(self, name, res, args):
        f = getattr(self.lib, self.prefix + name)
        f.restype = res
        f.argtypes = args
        return f

    # ---- quantizers ----
    def q40_quant_rows(self, w):
        w = np.ascontiguousarray(w, np.float32)
        O, I = w.shape
        out = np.zeros((O, I // 32 * 18), np.uint8)
        f = self.fn("q40_quant_row", None, [_P, _P, _I])
        for o in range(O):
            f(_ptr(w[o]), _ptr(out[o]), I)
        return out

    def q80_quant_rows(self, w):
        w = np.ascontiguousarray(w, np.float32)
        O, I = w.shape
        out = np.zeros((O, I // 32 * 34), np.uint8)
        f = self.fn("q80_quant_row", None, [_P, _P, _I])
        for o in range(O):
            f(_ptr(w[o]), _ptr(out[o]), I)
        return out

    def quant_act(self, x):
        """q40_quant_act over rows of x [S, I] -> (xq [S, I] int8, sx [S, I/32] f32)"""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        S, I = x.shape
        xq = np.zeros((S, I), np.int8)
        sx = np.zeros((S, I // 32), np.float32)
        f = self.fn("quant_act", None, [_P, _P, _P, _I])
        for s in range(S):
            f(_ptr(x[s]), _ptr(xq[s]), _ptr(sx[s]), I)
        return xq, sx

    def tq2_quant_act(self, x):
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        S, I = x.shape
        xq = np.zeros((S, I), np.int8)
        sx = np.zeros((S, I // 32), np.float32)
        tot = np.zeros((S,), np.float32)
        f = self.fn("tq2_quant_act", _F, [_P, _P, _P, _I])
        for s in range(S):
            tot[s] = f(_ptr(x[s]), _ptr(xq[s]), _ptr(sx[s]), I)
        return xq, sx, tot

    # ---- dots ----
    def q40_dot(self, w_row, xq, sx):
        f = self.fn("q40_dot", _F, [_P, _P, _P, _I])
        return f(_ptr(np.ascontiguousarray(w_row)), _ptr(np.ascontiguousarray(xq)),
                 _ptr(np.ascontiguousarray(sx, np.float32)), xq.shape[-1])

    def q80_dot(self, w_row, xq, sx):
        f = self.fn("q80_dot", _F, [_P, _P, _P, _I])
        return f(_ptr(np.ascontiguousarray(w_row)), _ptr(np.ascontiguousarray(xq)),
                 _ptr(np.ascontiguousarray(sx, np.float32)), xq.shape[-1])

    def tq2_dot(self, codes_row, alpha, xq, sx, sxtot):
        f = self.fn("tq2_dot", _F, [_P, _F, _P, _P, _F, _I])
        return f(_ptr(np.ascontiguousarray(codes_row)), float(alpha), _ptr(np.ascontiguousarray(xq)),
                 _ptr(np.ascontiguousarray(sx, np.float32)), float(sxtot), xq.shape[-1])

    # ---- routed-expert FFN ----
    def route_topk(self, logits, K):
        logits = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
        S, E = logits.shape
        idx = np.zeros((S, K), np.int32)
        wts = np.zeros((S, K), np.float32)
        f = self.fn("route_topk", None, [_P, _I, _I, _P, _P])
        for s in range(S):
            f(_ptr(logits[s]), E, K, _ptr(idx[s]), _ptr(wts[s]))
        return idx, wts


    def gemma4_route(self, res, proj, scale, pes, K, eps=1e-6):
        """gemma4 route_row over rows res [S, D] -> idx, wts [S, K]"""
        res = np.ascontiguousarray(np.atleast_2d(res), np.float32)
        S, D = res.shape
        E = proj.shape[0]
        idx = np.zeros((S, K), np.int32)
        wts = np.zeros((S, K), np.float32)
        if self.prefix == "ref_":
            self.fn("gemma4_route", None, [_P, _I, _I, _I, _I, _P, _P, _P, _F, _P, _P])(
                _ptr(res), S, D, E, K, _ptr(np.ascontiguousarray(proj, np.float32)),
                _ptr(np.ascontiguousarray(scale, np.float32)), _ptr(np.ascontiguousarray(pes, np.float32)),
                float(eps), _ptr(idx), _ptr(wts))
        else:
            f = self.fn("gemma4_route", None, [_P, _I, _I, _I, _P, _P, _P, _F, _P, _P])
            for s in range(S):
                f(_ptr(res[s]), D, E, K, _ptr(np.ascontiguousarray(proj, np.float32)),
                  _ptr(np.ascontiguousarray(scale, np.float32)), _ptr(np.ascontiguousarray(pes, np.float32)),
                  float(eps), _ptr(idx[s]), _ptr(wts[s]))
        return idx, wts

    def ling_route(self, xn, router, bias, K, n_group, topk_group, norm_topk=1, routed_scale=1.0):
        """ling grouped route_row over normalized rows xn [S, D] -> idx, wts [S, K]"""
        xn = np.ascontiguousarray(np.atleast_2d(xn), np.float32)
        S, D = xn.shape
        E = router.shape[0]
        idx = np.zeros((S, K), np.int32)
        wts = np.zeros((S, K), np.float32)
        rt = np.ascontiguousarray(router, np.float32)
        bi = np.ascontiguousarray(bias, np.float32)
        if self.prefix == "ref_":
            self.fn("ling_route", None, [_P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P])(
                _ptr(xn), S, D, E, K, n_group, topk_group, norm_topk, float(routed_scale), _ptr(rt), _ptr(bi),
                _ptr(idx), _ptr(wts))
        else:
            f = self.fn("ling_route", None, [_P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P])
            for s in range(S):
                f(_ptr(xn[s]), D, E, K, n_group, topk_group, norm_topk, float(routed_scale), _ptr(rt), _ptr(bi),
                  _ptr(idx[s]), _ptr(wts[s]))
        return idx, wts


class Oracle(_Lib):
    """The restatement (zz_oracle.c)."""

    def __init__(self):
        if not os.path.exists(ORC_PATH):
            build()
        super().__init__(ORC_PATH, "orc_")

    def q40_matvec(self, W, xq, sx):
        O = W.shape[0]
        y = np.zeros(O, np.float32)
        self.fn("q40_matvec", None, [_P, _P, _P, _P, _I, _I])(_ptr(y), _ptr(W), _ptr(xq), _ptr(sx), O, xq.shape[-1])
        return y

    def q80_matvec(self, W, xq, sx):
        O = W.shape[0]
        y = np.zeros(O, np.float32)
        self.fn("q80_matvec", None, [_P, _P, _P, _P, _I, _I])(_ptr(y), _ptr(W), _ptr(xq), _ptr(sx), O, xq.shape[-1])
        return y

    def tq2_matvec(self, T, O, xq, sx, sxtot):
        y = np.zeros(O, np.float32)
        self.fn("tq2_matvec", None, [_P, _P, _P, _P, _F, _I, _I])(_ptr(y), _ptr(T), _ptr(xq), _ptr(sx),
                                                                  float(sxtot), O, xq.shape[-1])
        return y

    def blocksums(self, fmt, W, xq):
        """per-block ints [O, I/32] of W rows against one activation row"""
        O, I = W.shape[0], xq.shape[-1]
        out = np.zeros((O, I // 32), np.int32)
        name = {1: "q40_blocksums", 2: "q80_blocksums", 3: "tq2_blocksums"}[fmt]
        f = self.fn(name, None, [_P, _P, _I, _P])
        for o in range(O):
            f(_ptr(np.ascontiguousarray(W[o])), _ptr(xq), I, _ptr(out[o]))
        return out

    def f32_to_fp16(self, v):
        return self.fn("f32_to_fp16", ctypes.c_uint16, [_F])(float(v))

    def fp16_to_f32(self, h):
        return self.fn("fp16_to_f32", _F, [ctypes.c_uint16])(int(h))

    def act_vec(self, act, g, u, clamp=7.0):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        h = np.zeros_like(g)
        self.fn("act_vec", None, [_I, _P, _P, _P, _I, _F])(act, _ptr(g), _ptr(u), _ptr(h), g.size, float(clamp))
        return h

    def moe_layer(self, kind, blobs, X, eidx, ewt, D, MI, clamp=7.0):
        """kind 0 q4_0 GeGLU, 1 q4_0 SwiGLU, 2 q8_0 SwiGLU, 3 tq2 clamped SwiGLU"""
        X = np.ascontiguousarray(X, np.float32)
        S, K = eidx.shape
        E = blobs.shape[0]
        out = np.zeros((S, D), np.float32)
        ptrs = (_P * E)(*[blobs[e].ctypes.data for e in range(E)])
        f = self.fn("moe_layer", None, [_I, _P, _I, _P, _P, _I, _I, _P, _P, _I, _I, _F])
        f(kind, ptrs, E, _ptr(X), _ptr(out), S, K, _ptr(np.ascontiguousarray(eidx, np.int32)),
          _ptr(np.ascontiguousarray(ewt, np.float32)), D, MI, float(clamp))
        return out


    def moe_layer_q8(self, kind, blobs, XQ, XS, eidx, ewt, D, MI, clamp=7.0):
        """the layer on pre-quantized rows; eidx entries outside [0, E) are skipped"""
        S, K = eidx.shape
        E = blobs.shape[0]
        out = np.zeros((S, D), np.float32)
        if S == 0:
            return out
        ptrs = (_P * max(E, 1))(*[blobs[e].ctypes.data for e in range(E)])
        f = self.fn("moe_layer_q8", None, [_I, _P, _I, _P, _P, _P, _I, _I, _P, _P, _I, _I, _F])
        f(kind, ptrs, E, _ptr(np.ascontiguousarray(XQ, np.int8)), _ptr(np.ascontiguousarray(XS, np.float32)),
          _ptr(out), S, K, _ptr(np.ascontiguousarray(eidx, np.int32)), _ptr(np.ascontiguousarray(ewt, np.float32)),
          D, MI, float(clamp))
        return out


    def matvec_f32(self, fmt, T, O, I, x):
        """exact-activation matvec (q40_dot_f32 / q80_dot_f32 / tq2_dot_f32 / q4a_dot_f32)"""
        y = np.zeros(O, np.float32)
        self.fn("matvec_f32", None, [_I, _P, _P, _P, _I, _I])(fmt, _ptr(y), _ptr(np.ascontiguousarray(T)),
                                                              _ptr(np.ascontiguousarray(x, np.float32)), O, I)
        return y

    def q4a_matvec(self, T, O, xq, sx):
        I = xq.shape[-1]
        y = np.zeros(O, np.float32)
        self.fn("q4a_matvec", None, [_P, _P, _P, _P, _I, _I])(_ptr(y), _ptr(np.ascontiguousarray(T)),
                                                              _ptr(np.ascontiguousarray(xq)),
                                                              _ptr(np.ascontiguousarray(sx, np.float32)), O, I)
        return y

    def moe_pairs_hidden(self, kind, blobs, X, eidx, D, MI, clamp=7.0):
        """stage 1 for every routed pair: hq [S*K, MI] int8, hs [S*K, MI/32] f32"""
        X = np.ascontiguousarray(X, np.float32)
        S, K = eidx.shape
        E = blobs.shape[0]
        hq = np.zeros((S * K, MI), np.int8)
        hs = np.zeros((S * K, MI // 32), np.float32)
        ptrs = (_P * E)(*[blobs[e].ctypes.data for e in range(E)])
        f = self.fn("moe_pairs_hidden", None, [_I, _P, _I, _P, _I, _I, _P, _I, _I, _F, _P, _P])
        f(kind, ptrs, E, _ptr(X), S, K, _ptr(np.ascontiguousarray(eidx, np.int32)), D, MI, float(clamp),
          _ptr(hq), _ptr(hs))
        return hq, hs

    def moe_pairs_combine(self, kind, blobs, hq, hs, eidx, ewt, D, MI):
        """stage 2 from given per-pair hidden rows (pair p = s*K + k): OUT [S, D]"""
        S, K = eidx.shape
        E = blobs.shape[0]
        out = np.zeros((S, D), np.float32)
        ptrs = (_P * E)(*[blobs[e].ctypes.data for e in range(E)])
        f = self.fn("moe_pairs_combine", None, [_I, _P, _I, _P, _P, _I, _I, _P, _P, _I, _I, _P])
        f(kind, ptrs, E, _ptr(np.ascontiguousarray(hq, np.int8)), _ptr(np.ascontiguousarray(hs, np.float32)), S, K,
          _ptr(np.ascontiguousarray(eidx, np.int32)), _ptr(np.ascontiguousarray(ewt, np.float32)), D, MI, _ptr(out))
        return out


class Reference(_Lib):
    """The reference's own kernels and engine routines (oracle/_ref/libzzref.so)."""

    def __init__(self):
        if not os.path.exists(REF_PATH):
            raise FileNotFoundError(REF_PATH)
        super().__init__(REF_PATH, "ref_")

    def set_threads(self, n):
        self.fn("set_threads", None, [_I])(int(n))

    def max_threads(self):
        return self.fn("max_threads", _I, [])()

    def q40_matvec(self, W, xq, sx):
        O = W.shape[0]
        y = np.zeros(O, np.float32)
        self.fn("q40_matvec_omp", None, [_P, _P, _P, _P, _I, _I])(_ptr(y), _ptr(W), _ptr(xq), _ptr(sx), O,
                                                                  xq.shape[-1])
        return y

    def q80_matvec(self, W, xq, sx):
        O = W.shape[0]
        y = np.zeros(O, np.float32)
        self.fn("q80_matvec_omp", None, [_P, _P, _P, _P, _I, _I])(_ptr(y), _ptr(W), _ptr(xq), _ptr(sx), O,
                                                                  xq.shape[-1])
        return y

    def tq2_matvec(self, T, O, xq, sx, sxtot):
        y = np.zeros(O, np.float32)
        self.fn("tq2_matvec_omp", None, [_P, _P, _P, _P, _F, _I, _I])(_ptr(y), _ptr(T), _ptr(xq), _ptr(sx),
                                                                      float(sxtot), O, xq.shape[-1])
        return y

    def f32_to_fp16(self, v):
        return self.fn("f32_to_fp16", ctypes.c_uint16, [_F])(float(v))

    def fp16_to_f32(self, h):
        return self.fn("fp16_to_f32", _F, [ctypes.c_uint16])(int(h))

    def moe_layer(self, kind, blobs, X, eidx, ewt, D, MI, clamp=7.0):
        """gemma4 engine (kind 0: q4_0 GeGLU) or maple engine (kind 3: tq2)"""
        X = np.ascontiguousarray(X, np.float32)
        S, K = eidx.shape
        E = blobs.shape[0]
        out = np.zeros((S, D), np.float32)
        ptrs = (_P * E)(*[blobs[e].ctypes.data for e in range(E)])
        ei = _ptr(np.ascontiguousarray(eidx, np.int32))
        ew = _ptr(np.ascontiguousarray(ewt, np.float32))
        if kind == 0:
            f = self.fn("gemma4_moe_layer", None, [_P, _P, _P, _I, _I, _P, _P, _I, _I, _I])
            f(ptrs, _ptr(X), _ptr(out), S, K, ei, ew, D, MI, E)
        elif kind == 3:
            f = self.fn("maple_moe_layer", None, [_P, _P, _P, _I, _I, _P, _P, _I, _I, _I, _F])
            f(ptrs, _ptr(X), _ptr(out), S, K, ei, ew, D, MI, E, float(clamp))
        else:
            raise ValueError("the reference engines built here cover kinds 0 (gemma4) and 3 (maple)")
        return out

    def expert_apply(self, kind, blob, X, OUT, rows, w, D, MI, clamp=7.0):
        rows = np.ascontiguousarray(rows, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        if kind == 0:
            f = self.fn("gemma4_expert_apply", None, [_P, _P, _P, _P, _I, _P, _I, _I])
            f(_ptr(blob), _ptr(X), _ptr(OUT), _ptr(rows), len(rows), _ptr(w), D, MI)
        else:
            f = self.fn("maple_expert_apply", None, [_P, _P, _P, _P, _I, _P, _I, _I, _F])
            f(_ptr(blob), _ptr(X), _ptr(OUT), _ptr(rows), len(rows), _ptr(w), D, MI, float(clamp))


def reference_available():
    return os.path.exists(REF_PATH)
