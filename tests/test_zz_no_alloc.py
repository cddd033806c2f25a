"""The allocation-free MoE entry point (zz_moe_ffn_noalloc_dev), called through the C
ABI. It exists for callers that may not allocate device memory once running -- an
engine with a fixed GPU budget, or a host that forbids cudaMalloc after start-up -- so
its scratch is a fixed array inside the library. Two calls in a row, with different
inputs, must each match the workspace entry point (zz_moe_ffn_dev) within the MoE
tolerance, which also shows that the previous call's leftovers in the shared array do
not leak into the next result. Kept in its own file so pytest collects it last."""
import ctypes

import numpy as np
import pytest
import torch

import zunzuncito_b200 as zz
from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max |a - b| / max |b|, the end-to-end MoE tolerance used elsewhere


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(bank, X, eidx, ewt, out):
    S, K = eidx.shape
    return zz.lib.zz_moe_ffn_noalloc_dev(ctypes.byref(bank.b), _p(X), _p(eidx), _p(ewt), _p(out), S, K,
                                         zz.ZZ_ACT_GEGLU_TANH, 0.0,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_workspace_entry_twice(orc):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    E, D, MI, K = 16, 512, 128, 4
    blobs = np.stack([np.concatenate([orc.q40_quant_rows(synth.gaussian(900 + 3 * e + i, shp, 0.02)).ravel()
                                      for i, shp in enumerate([(MI, D), (MI, D), (D, MI)])]) for e in range(E)])
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, torch.from_numpy(blobs).cuda(), D, MI)
    for call, S in enumerate((37, 200)):
        X = torch.from_numpy(synth.gaussian(950 + call, (S, D))).cuda()
        ei, ew, _ = synth.zipf_routing(960 + call, S, E, K)
        eidx, ewt = torch.from_numpy(ei).cuda(), torch.from_numpy(ew).cuda()
        want = zz.moe_ffn(bank, X, eidx, ewt, zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
        out = torch.full((S, D), float("nan"), device="cuda")
        assert _noalloc(bank, X, eidx, ewt, out) == 1, zz.lib.gpu_last_error()
        got = out.cpu().numpy()
        assert np.max(np.abs(got - want)) <= TOL * np.max(np.abs(want)), call


def test_noalloc_rejects_oversize():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    D, MI, E = 2816, 704, 8
    blobs = torch.zeros((E, zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)), dtype=torch.uint8, device="cuda")
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
    S, K = 4096, 8
    X = torch.zeros((S, D), device="cuda")
    eidx = torch.zeros((S, K), dtype=torch.int32, device="cuda")
    ewt = torch.zeros((S, K), device="cuda")
    out = torch.zeros((S, D), device="cuda")
    assert _noalloc(bank, X, eidx, ewt, out) == 0
    assert b"scratch" in zz.lib.gpu_last_error()


def test_noalloc_gemma_shape_at_capacity():
    """Gemma-4 layer shape (128 q4_0 experts, hidden 2816, inter 704, top-8) at the largest
    batch the fixed scratch holds, S = 862: matches the workspace entry point; S = 863
    declines with a reason instead of running."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    D, MI, E, K = synth.GEMMA_D, synth.GEMMA_MI, synth.GEMMA_E, synth.GEMMA_K
    stride = zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)
    g = torch.Generator(device="cuda").manual_seed(990)
    gb = zz.ref_tensor_bytes(zz.GPU_FMT_Q40, MI, D)
    blobs = torch.empty((E, stride), dtype=torch.uint8, device="cuda")
    for i, (O, I) in enumerate([(MI, D), (MI, D), (D, MI)]):
        w = torch.randn((E * O, I), generator=g, device="cuda") * 0.02
        blobs[:, i * gb:i * gb + O * I // 32 * 18] = zz.quant_rows(zz.GPU_FMT_Q40, w).view(E, -1)
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
    S = 862
    X = torch.from_numpy(synth.gaussian(991, (S + 1, D))).cuda()
    ei, ew, _ = synth.zipf_routing(992, S + 1, E, K)
    eidx, ewt = torch.from_numpy(ei).cuda(), torch.from_numpy(ew).cuda()
    want = zz.moe_ffn(bank, X[:S], eidx[:S], ewt[:S], zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    out = torch.full((S + 1, D), float("nan"), device="cuda")
    assert _noalloc(bank, X[:S], eidx[:S], ewt[:S], out[:S]) == 1, zz.lib.gpu_last_error()
    got = out[:S].cpu().numpy()
    assert np.max(np.abs(got - want)) <= TOL * np.max(np.abs(want))
    assert _noalloc(bank, X, eidx, ewt, out) == 0
    assert b"scratch" in zz.lib.gpu_last_error()
