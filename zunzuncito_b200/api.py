"""Typed access to libzz_cuda.so for callers holding torch CUDA tensors.

torch supplies device memory and the current stream only; every kernel that touches
the data is in libzz_cuda.so.
"""
import ctypes

import torch

from . import (GPU_FMT_Q40, GPU_FMT_Q4A, GPU_FMT_Q80, GPU_FMT_TQ2, ExpertBank, QTensor, check, lib)

__all__ = ["ref_row_bytes", "ref_tensor_bytes", "expert_blob_bytes", "quant_act", "quant_rows",
           "QTensorDev", "matvec", "blocksums", "ExpertBankDev", "moe_ffn", "moe_ffn_q8", "alloc_aligned",
           "ep_pack", "ep_unpack", "route_gemma4", "route_ling"]


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def ref_row_bytes(fmt, I):
    """Bytes of one row in the reference layout (q40.h:313, 460; tq2.h:81, 286)."""
    return {GPU_FMT_Q40: I // 32 * 18, GPU_FMT_Q80: I // 32 * 34, GPU_FMT_TQ2: I // 4, GPU_FMT_Q4A: I // 64 * 36}[fmt]


def ref_tensor_bytes(fmt, O, I):
    """Bytes of one [O, I] tensor in the reference layout; tq2 adds the O f32 alphas."""
    return O * ref_row_bytes(fmt, I) + (4 * O if fmt == GPU_FMT_TQ2 else 0)


def expert_blob_bytes(fmt, D, MI):
    """One expert blob [gate MI x D | up MI x D | down D x MI] (gemma4.c:660, maple.c:616-619)."""
    return 2 * ref_tensor_bytes(fmt, MI, D) + ref_tensor_bytes(fmt, D, MI)


def alloc_aligned(nbytes, device="cuda"):
    """uint8 device buffer whose data_ptr is 256-byte aligned."""
    raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % 256
    return raw[off:off + nbytes]


def quant_act(x, want_sxtot=False):
    """q40_quant_act / tq2_quant_act on device for each row of x [S, I] f32."""
    x = x.contiguous()
    S, I = x.shape
    xq = torch.empty((S, I), dtype=torch.int8, device=x.device)
    sx = torch.empty((S, I // 32), dtype=torch.float32, device=x.device)
    tot = torch.empty((S,), dtype=torch.float32, device=x.device) if want_sxtot else None
    check(lib.zz_quant_act_dev(_p(x), S, I, _p(xq), _p(sx), _p(tot), _stream()), "zz_quant_act_dev")
    return xq, sx, tot


def quant_rows(fmt, w):
    """q40_quant_row / q80_quant_row on device: w [O, I] f32 -> reference-layout bytes."""
    w = w.contiguous()
    O, I = w.shape
    dst = torch.empty(O * ref_row_bytes(fmt, I), dtype=torch.uint8, device=w.device)
    check(lib.zz_quant_rows_dev(fmt, _p(w), O, I, _p(dst), _stream()), "zz_quant_rows_dev")
    return dst


class QTensorDev:
    """A weight tensor repacked into structure-of-arrays planes (keeps its memory alive)."""

    def __init__(self, fmt, src, O, I):
        nbytes = lib.zz_qtensor_bytes(fmt, O, I)
        if nbytes == 0:
            raise ValueError(f"unsupported fmt {fmt} / shape {O}x{I}")
        self.mem = alloc_aligned(nbytes, src.device)
        self.t = QTensor()
        check(lib.zz_repack_dev(fmt, _p(src), O, I, _p(self.mem), ctypes.byref(self.t), _stream()),
              "zz_repack_dev")
        self.fmt, self.O, self.I = fmt, O, I

    def unpack(self):
        dst = torch.empty(ref_tensor_bytes(self.fmt, self.O, self.I), dtype=torch.uint8, device=self.mem.device)
        check(lib.zz_unpack_dev(ctypes.byref(self.t), _p(dst), _stream()), "zz_unpack_dev")
        return dst


def matvec(W, xq, sx, sxtot=None, y=None):
    """y[S, O] = W . q8_0 rows (zz_matvec_dev)."""
    S = xq.shape[0]
    if y is None:
        y = torch.empty((S, W.O), dtype=torch.float32, device=xq.device)
    check(lib.zz_matvec_dev(ctypes.byref(W.t), _p(xq), _p(sx), _p(sxtot), _p(y), S, _stream()), "zz_matvec_dev")
    return y


def blocksums(W, xq_row):
    """Per-block integer sums [O, I/32] for one activation row (zz_blocksums_dev)."""
    out = torch.empty((W.O, W.I // 32), dtype=torch.int32, device=xq_row.device)
    check(lib.zz_blocksums_dev(ctypes.byref(W.t), _p(xq_row), _p(out), _stream()), "zz_blocksums_dev")
    return out


class ExpertBankDev:
    """One MoE layer's experts packed from reference blobs (zz_expert_bank_pack_dev).

    blobs: uint8 CUDA tensor [E, blob_stride] holding each expert's [gate|up|down]."""

    def __init__(self, fmt, blobs, D, MI):
        E, stride = blobs.shape
        nbytes = lib.zz_expert_bank_bytes(fmt, E, D, MI)
        if nbytes == 0:
            raise ValueError(f"unsupported bank fmt {fmt} E={E} D={D} MI={MI}")
        self.mem = alloc_aligned(nbytes, blobs.device)
        self.b = ExpertBank()
        check(lib.zz_expert_bank_pack_dev(fmt, E, D, MI, _p(blobs), stride, _p(self.mem), ctypes.byref(self.b),
                                          _stream()), "zz_expert_bank_pack_dev")
        self.fmt, self.E, self.D, self.MI = fmt, E, D, MI
        self._ws = None

    def workspace(self, S, K):
        n = lib.zz_moe_workspace_bytes(ctypes.byref(self.b), S, K)
        if self._ws is None or self._ws.numel() < n:
            self._ws = alloc_aligned(n, self.mem.device)
        return self._ws


def moe_ffn(bank, X, eidx, ewt, act, clamp=0.0, out=None, validate=False):
    """Batch-union routed-expert FFN of one layer (zz_moe_ffn_dev)."""
    S, D = X.shape
    K = eidx.shape[1]
    if out is None:
        out = torch.empty((S, D), dtype=torch.float32, device=X.device)
    ws = bank.workspace(S, K)
    check(lib.zz_moe_ffn_dev(ctypes.byref(bank.b), _p(X), _p(eidx), _p(ewt), _p(out), S, K, act, float(clamp),
                             _p(ws), ws.numel(), int(validate), _stream()), "zz_moe_ffn_dev")
    return out


def moe_ffn_q8(bank, xq, xs, eidx, ewt, act, clamp=0.0, out=None, validate=False):
    """The same layer for q8_0 rows (zz_moe_ffn_q8_dev); eidx entries of -1 are skipped."""
    S, D = xq.shape
    K = eidx.shape[1]
    if out is None:
        out = torch.empty((S, D), dtype=torch.float32, device=xq.device)
    if S == 0:
        return out
    ws = bank.workspace(S, K)
    check(lib.zz_moe_ffn_q8_dev(ctypes.byref(bank.b), _p(xq), _p(xs), _p(eidx), _p(ewt), _p(out), S, K, act,
                                float(clamp), _p(ws), ws.numel(), int(validate), _stream()), "zz_moe_ffn_q8_dev")
    return out


def ep_pack(xq, xs, eidx, ewt, world, per_rank):
    """Expert-parallel dispatch rows [world, S, row] (zz_ep_pack_dev)."""
    S, D = xq.shape
    K = eidx.shape[1]
    out = torch.empty((world, S, lib.zz_ep_row_bytes(D, K)), dtype=torch.uint8, device=xq.device)
    check(lib.zz_ep_pack_dev(_p(xq), _p(xs), _p(eidx), _p(ewt), S, D, K, world, per_rank, _p(out), _stream()),
          "zz_ep_pack_dev")
    return out


def ep_unpack(rows, D, K):
    """Received exchange rows [R, row] -> xq, xs, eidx, ewt (zz_ep_unpack_dev)."""
    R = rows.numel() // lib.zz_ep_row_bytes(D, K)
    dev = rows.device
    xq = torch.empty((R, D), dtype=torch.int8, device=dev)
    xs = torch.empty((R, D // 32), dtype=torch.float32, device=dev)
    eidx = torch.empty((R, K), dtype=torch.int32, device=dev)
    ewt = torch.empty((R, K), dtype=torch.float32, device=dev)
    check(lib.zz_ep_unpack_dev(_p(rows), R, D, K, _p(xq), _p(xs), _p(eidx), _p(ewt), _stream()), "zz_ep_unpack_dev")
    return xq, xs, eidx, ewt


def route_gemma4(res, proj, scale, pes, K, eps=1e-6):
    """gemma4 router on device (zz_route_gemma4_dev): res [S, D] -> eidx, ewt [S, K]"""
    res = res.contiguous()
    S, D = res.shape
    E = proj.shape[0]
    idx = torch.empty((S, K), dtype=torch.int32, device=res.device)
    wts = torch.empty((S, K), dtype=torch.float32, device=res.device)
    check(lib.zz_route_gemma4_dev(_p(res), S, D, E, K, _p(proj.contiguous()), _p(scale.contiguous()),
                                  _p(pes.contiguous()), float(eps), _p(idx), _p(wts), _stream()), "zz_route_gemma4_dev")
    return idx, wts


def route_ling(xn, router, bias, K, n_group, topk_group, norm_topk_prob=1, routed_scale=1.0):
    """ling grouped router on device (zz_route_ling_dev): xn [S, D] -> eidx, ewt [S, K]"""
    xn = xn.contiguous()
    S, D = xn.shape
    E = router.shape[0]
    idx = torch.empty((S, K), dtype=torch.int32, device=xn.device)
    wts = torch.empty((S, K), dtype=torch.float32, device=xn.device)
    check(lib.zz_route_ling_dev(_p(xn), S, D, E, K, n_group, topk_group, int(norm_topk_prob), float(routed_scale),
                                _p(router.contiguous()), _p(bias.contiguous()), _p(idx), _p(wts), _stream()),
          "zz_route_ling_dev")
    return idx, wts
