"""Batch-union routed-expert FFN on the GPU (zz_moe_ffn_dev) against the oracle.

Parity is checked stage by stage, as the survey of the path defines it:
  1. gate/up stage: the requantized hidden hq/hs of every (token, expert) pair equals
     the oracle's; only elements whose q8 rounding sits at a tie within fp32 noise may
     differ, by one step (the GPU's fp32 dot order and tanhf differ from glibc's);
  2. down stage: fed the GPU's own hq/hs, the combine equals the oracle within 1e-5;
  3. end to end: rows with no requant flip within 1e-4 of max|out|.
At the full Gemma-4 layer shape the same checks run on a sample of pairs, plus the
size-independent properties (linearity in the router weights, token permutation)."""
import ctypes

import numpy as np
import pytest
import torch

import zunzuncito_b200 as zz
from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu

ENGINES = ("mma", "tc")
KINDS = {0: (zz.GPU_FMT_Q40, zz.ZZ_ACT_GEGLU_TANH), 1: (zz.GPU_FMT_Q40, zz.ZZ_ACT_SWIGLU),
         2: (zz.GPU_FMT_Q80, zz.ZZ_ACT_SWIGLU), 3: (zz.GPU_FMT_TQ2, zz.ZZ_ACT_SWIGLU_CLAMP)}
CLAMP = 7.0


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_blobs(orc, kind, seed, E, D, MI):
    fmt = KINDS[kind][0]
    if fmt == zz.GPU_FMT_TQ2:
        return np.stack([np.concatenate([synth.tq2_tensor(seed + 3 * e, MI, D), synth.tq2_tensor(seed + 3 * e + 1, MI, D),
                                         synth.tq2_tensor(seed + 3 * e + 2, D, MI)]) for e in range(E)])
    q = orc.q40_quant_rows if fmt == zz.GPU_FMT_Q40 else orc.q80_quant_rows
    return np.stack([np.concatenate([q(synth.gaussian(seed + 3 * e, (MI, D), 0.02)).ravel(),
                                     q(synth.gaussian(seed + 3 * e + 1, (MI, D), 0.02)).ravel(),
                                     q(synth.gaussian(seed + 3 * e + 2, (D, MI), 0.02)).ravel()]) for e in range(E)])


def split_blob(fmt, blob, D, MI):
    gb = zz.ref_tensor_bytes(fmt, MI, D)
    return blob[:gb], blob[gb:2 * gb], blob[2 * gb:]


def ws_views(bank, S, K):
    """pair rows of the last call (padding rows, src < 0, dropped), their hq / hs"""
    ws = bank._ws
    MI = bank.MI
    off = lambda w: zz.lib.zz_moe_workspace_offset(ctypes.byref(bank.b), S, K, w)
    P = off(6)  # pair-row capacity incl. per-expert alignment padding
    src = ws[off(0):off(0) + 4 * P].view(torch.int32).cpu().numpy()
    hq = ws[off(2):off(2) + P * MI].view(torch.int8).cpu().numpy().reshape(P, MI)
    hs = ws[off(3):off(3) + P * (MI // 32) * 4].view(torch.float32).cpu().numpy().reshape(P, MI // 32)
    err = int(ws[off(5):off(5) + 4].view(torch.int32).cpu().numpy()[0])
    assert err == 0, f"tensor-core pipeline wait {err} ran out"
    keep = src >= 0
    assert keep.sum() == S * K
    return src[keep], hq[keep], hs[keep]


def matvec(orc, fmt, T, O, xq, sx, tot):
    if fmt == zz.GPU_FMT_Q40:
        return orc.q40_matvec(T.reshape(O, -1), xq, sx)
    if fmt == zz.GPU_FMT_Q80:
        return orc.q80_matvec(T.reshape(O, -1), xq, sx)
    return orc.tq2_matvec(T, O, xq, sx, tot)


def tq2_total(hq, hs):
    s = hq.reshape(-1, 32).astype(np.int64).sum(1)
    return np.float32(np.sum(hs.astype(np.float64) * s.astype(np.float64)))


def check_pairs(orc, kind, blobs, X, eidx, ewt, out_gpu, bank, pairs=None):
    """stage 1 + 2 on the listed pair rows (all by default); returns flipped tokens"""
    fmt, act = KINDS[kind]
    S, K = eidx.shape
    D, MI = bank.D, bank.MI
    src, hq, hs = ws_views(bank, S, K)
    rows = range(S * K) if pairs is None else pairs
    flipped_tok = set()
    n_flip = 0
    for r in rows:
        p = int(src[r])
        s, k = divmod(p, K)
        e = int(eidx[s, k])
        G, U, Dn = split_blob(fmt, blobs[e], D, MI)
        xq, sx, tot = orc.tq2_quant_act(X[s:s + 1])
        g = matvec(orc, fmt, G, MI, xq[0], sx[0], tot[0])
        u = matvec(orc, fmt, U, MI, xq[0], sx[0], tot[0])
        h = orc.act_vec(act, g, u, CLAMP)
        eq, es = orc.quant_act(h[None])
        diff = hq[r].astype(np.int32) - eq[0]
        if np.any(diff):
            assert np.max(np.abs(diff)) <= 1, (r, np.max(np.abs(diff)))
            n_flip += int(np.count_nonzero(diff))
            flipped_tok.add(s)
        # scales: amax/127 of h; h itself carries fp32 accumulation-order noise
        assert np.allclose(hs[r], es[0], rtol=1e-5, atol=0), r
    total = len(rows) * MI
    assert n_flip <= max(3, total // 500), (n_flip, total)
    if pairs is None:
        # stage 2: combine from the GPU's own hidden rows, all pairs
        want = np.zeros((S, D), np.float32)
        for r in range(S * K):
            s, k = divmod(int(src[r]), K)
            e = int(eidx[s, k])
            Dn = split_blob(fmt, blobs[e], D, MI)[2]
            y = matvec(orc, fmt, Dn, D, hq[r], hs[r], tq2_total(hq[r], hs[r]))
            want[s] += ewt[s, k] * y
        scale = np.max(np.abs(want))
        assert np.max(np.abs(out_gpu - want)) <= 1e-5 * scale
    return flipped_tok


@pytest.fixture(params=["auto", "mma", "mma8", "tc", "tcw", "dec"])
def engine(request, monkeypatch):
    """every expert engine: auto (GEMV for small S*K, else mma.sync), mma.sync, tcgen05 (32- and 128-token tiles),
    and the small-batch GEMV kernels forced (ZZ_MOE_KERNEL; calls of more than 64 pairs
    take the int8 mma.sync engine there)"""
    monkeypatch.setenv("ZZ_MOE_KERNEL", request.param)
    return request.param


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
@pytest.mark.parametrize("S", [1, 7, 100])
def test_moe_small(orc, kind, S, engine):
    fmt, act = KINDS[kind]
    E, D, MI, K = 8, 256, 128, 2 if S > 1 else 4
    blobs = make_blobs(orc, kind, 300 + kind, E, D, MI)
    X = synth.gaussian(400 + S, (S, D))
    eidx, ewt, _ = synth.zipf_routing(500 + S, S, E, K)
    bank = zz.ExpertBankDev(fmt, dev(blobs), D, MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), act, CLAMP, validate=True).cpu().numpy()
    flipped = check_pairs(orc, kind, blobs, X, eidx, ewt, out, bank)
    want = orc.moe_layer(kind, blobs, X, eidx, ewt, D, MI, CLAMP)
    scale = np.max(np.abs(want))
    for s in range(S):
        if s not in flipped:
            assert np.max(np.abs(out[s] - want[s])) <= 1e-4 * scale, s
        else:
            assert np.max(np.abs(out[s] - want[s])) <= 1e-2 * scale, s


@pytest.mark.parametrize("key,kind", [("g4", 0), ("mp", 3)])
def test_moe_golden(orc, key, kind, engine):
    import os
    G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    E, D, MI, K, S = (int(v) for v in G["dims"])
    fmt, act = KINDS[kind]
    bank = zz.ExpertBankDev(fmt, dev(G[key + "_blobs"]), D, MI)
    out = zz.moe_ffn(bank, dev(G[key + "_X"]), dev(G[key + "_eidx"]), dev(G[key + "_ewt"]), act, CLAMP).cpu().numpy()
    flipped = check_pairs(orc, kind, G[key + "_blobs"], G[key + "_X"], G[key + "_eidx"], G[key + "_ewt"], out, bank)
    ref = G[key + "_out"]
    for s in range(S):
        lim = 1e-2 if s in flipped else 1e-4
        assert np.max(np.abs(out[s] - ref[s])) <= lim * np.max(np.abs(ref))


def test_moe_declines():
    E, D, MI, K, S = 4, 128, 64, 2, 3
    blobs = torch.zeros((E, zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)), dtype=torch.uint8, device="cuda")
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
    X = torch.zeros((S, D), device="cuda")
    bad = torch.tensor([[0, 1], [2, 9], [3, 0]], dtype=torch.int32, device="cuda")
    w = torch.ones((S, K), device="cuda")
    with pytest.raises(zz.ZZError, match="outside"):
        zz.moe_ffn(bank, X, bad, w, zz.ZZ_ACT_GEGLU_TANH, validate=True)
    with pytest.raises(zz.ZZError):
        zz.moe_ffn(bank, X, bad, w, 7)


def _full_layer(seed, S):
    """Gemma-4 layer shape: 128 q4_0 experts, D 2816, MI 704, top-8,
    weights N(0, 0.02) quantized on device by the parity-tested device quantizer."""
    D, MI, E, K = synth.GEMMA_D, synth.GEMMA_MI, synth.GEMMA_E, synth.GEMMA_K
    stride = zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)
    blobs = torch.empty((E, stride), dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed)
    gb = zz.ref_tensor_bytes(zz.GPU_FMT_Q40, MI, D)
    for e in range(E):
        for i, (O, I) in enumerate([(MI, D), (MI, D), (D, MI)]):
            w = torch.randn((O, I), generator=g, device="cuda") * 0.02
            blobs[e, i * gb:i * gb + O * I // 32 * 18] = zz.quant_rows(zz.GPU_FMT_Q40, w)
    X = synth.gaussian(seed + 1, (S, D))
    eidx, ewt, _ = synth.zipf_routing(seed + 2, S, E, K)
    return blobs, X, eidx, ewt


def test_moe_full_layer_config3(orc, engine):
    S = 512
    blobs, X, eidx, ewt = _full_layer(600, S)
    D, MI = synth.GEMMA_D, synth.GEMMA_MI
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), zz.ZZ_ACT_GEGLU_TANH)
    out_np = out.cpu().numpy()
    # stage 1 on a sample of pair rows
    pairs = list(synth.rng(7).choice(S * 8, size=24, replace=False))
    blobs_np = blobs.cpu().numpy()
    check_pairs(orc, 0, blobs_np, X, eidx, ewt, out_np, bank, pairs=pairs)
    # stage 2 on a few whole tokens from the GPU's own hidden rows
    src, hq, hs = ws_views(bank, S, 8)
    slot = {int(p): r for r, p in enumerate(src)}
    for s in (0, 17, 511):
        want = np.zeros(D, np.float32)
        for k in range(8):
            r = slot[s * 8 + k]
            Dn = split_blob(zz.GPU_FMT_Q40, blobs_np[eidx[s, k]], D, MI)[2]
            want += ewt[s, k] * orc.q40_matvec(Dn.reshape(D, -1), hq[r], hs[r])
        assert np.max(np.abs(out_np[s] - want)) <= 1e-5 * np.max(np.abs(want))
    # linearity in the router weights (an exact power-of-two scaling)
    out2 = zz.moe_ffn(bank, dev(X), dev(eidx), dev(2 * ewt), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out2 - 2 * out_np)) <= 1e-6 * np.max(np.abs(out_np))
    # token permutation: outputs permute with the tokens
    perm = synth.rng(8).permutation(S)
    out3 = zz.moe_ffn(bank, dev(X[perm]), dev(eidx[perm]), dev(ewt[perm]), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out3 - out_np[perm])) <= 1e-6 * np.max(np.abs(out_np))
