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
import os

import numpy as np
import pytest
import torch

import zunzuncito_b200 as zz
from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu

KINDS = {0: (zz.GPU_FMT_Q40, zz.ZZ_ACT_GEGLU_TANH), 1: (zz.GPU_FMT_Q40, zz.ZZ_ACT_SWIGLU),
         2: (zz.GPU_FMT_Q80, zz.ZZ_ACT_SWIGLU), 3: (zz.GPU_FMT_TQ2, zz.ZZ_ACT_SWIGLU_CLAMP)}
CLAMP = 7.0


def hs_rtol():
    """relative tolerance of the requantized hidden scales (amax / 127 of h). The int8
    engines carry each 32-block sum exactly, so h differs from the oracle's only by fp32
    summation order (1e-5). The folded-scale fp16 engine (h3) also has the tensor core's
    truncating f32 adds inside each chunk of 16 K steps (measured up to 8e-6 at the
    Gemma-4 shape), so its scales are held to 2e-5; the layer output stays within the
    1e-4 of the spec either way."""
    return 2e-5 if os.environ.get("ZZ_MOE_KERNEL") == "h3" else 1e-5


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
        assert np.allclose(hs[r], es[0], rtol=hs_rtol(), atol=0), r
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


@pytest.fixture(params=["auto", "i8", "mma8", "mma8w", "h3", "hyb"])
def engine(request, monkeypatch):
    """every expert engine: auto (the decode GEMV kernels for calls of <= 64 pairs, else the
    int8 mma.sync GEMM with 32- or 64-row items by the rows per expert), and the int8
    tcgen05 engine and the narrow / wide mma.sync items forced for every call size
    (ZZ_MOE_KERNEL)"""
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
    for s in range(S):   # a flipped token's combine is checked from the GPU's own hidden rows above
        if s not in flipped:
            assert np.max(np.abs(out[s] - want[s])) <= 1e-4 * scale, s


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
        if s not in flipped:
            assert np.max(np.abs(out[s] - ref[s])) <= 1e-4 * np.max(np.abs(ref))


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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_moe_two_devices_one_thread(orc):
    # the library's per-device state (side stream, fork/join events): one host thread runs
    # the layer on device 0, then device 1, then device 0 again, with the same result
    E, D, MI, K, S = 8, 256, 128, 4, 80
    blobs = make_blobs(orc, 0, 1300, E, D, MI)
    X = synth.gaussian(1310, (S, D))
    eidx, ewt, _ = synth.zipf_routing(1320, S, E, K)
    outs = []
    for d in (0, 1, 0):
        with torch.cuda.device(d):
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{d}")
            bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, t(blobs), D, MI)
            outs.append(zz.moe_ffn(bank, t(X), t(eidx), t(ewt), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy())
    scale = np.max(np.abs(outs[0]))
    for o in outs[1:]:
        assert np.max(np.abs(o - outs[0])) <= 1e-6 * scale


def _gemma_blobs(seed, E=synth.GEMMA_E):
    """Gemma-4 expert blobs (3): 128 q4_0 experts, D 2816, MI 704,
    weights N(0, 0.02) quantized on device by the parity-tested device quantizer."""
    D, MI = synth.GEMMA_D, synth.GEMMA_MI
    stride = zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)
    blobs = torch.empty((E, stride), dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed)
    gb = zz.ref_tensor_bytes(zz.GPU_FMT_Q40, MI, D)
    for i, (O, I) in enumerate([(MI, D), (MI, D), (D, MI)]):
        w = torch.randn((E * O, I), generator=g, device="cuda") * 0.02
        blobs[:, i * gb:i * gb + O * I // 32 * 18] = zz.quant_rows(zz.GPU_FMT_Q40, w).view(E, -1)
    return blobs


def _maple_blobs(seed, E=synth.MAPLE_E):
    """Maple tq2 expert blobs: codes uniform in {0,1,2}, alpha
    |N(0,0.02)| + 1e-3 per row, packed as tq2.h:46-51, generated on the device"""
    D, MI = synth.MAPLE_D, synth.MAPLE_MI
    gen = torch.Generator(device="cuda").manual_seed(seed)

    def tensor(O, I):
        c = torch.randint(0, 3, (E, O, I // 64, 4, 16), generator=gen, device="cuda", dtype=torch.uint8)
        b = c[:, :, :, 0] | (c[:, :, :, 1] << 2) | (c[:, :, :, 2] << 4) | (c[:, :, :, 3] << 6)
        al = torch.randn((E, O), generator=gen, device="cuda").abs() * 0.02 + 1e-3
        return torch.cat([al.view(torch.uint8).view(E, -1), b.reshape(E, -1)], dim=1)
    return torch.cat([tensor(MI, D), tensor(MI, D), tensor(D, MI)], dim=1).contiguous()


def _full_check(orc, kind, blobs_np, bank, X, eidx, ewt, out, max_flip_frac=0.002):
    """Every pair and every token: stage 1 (hq equal but for rounding-tie flips of one
    step, hs within 1e-5), stage 2 (the combine of the GPU's own hidden rows within 1e-5
    of max|out|), end to end (tokens without a flip within 1e-4). Returns the flip count."""
    S, K = eidx.shape
    D, MI = bank.D, bank.MI
    src, hq, hs = ws_views(bank, S, K)
    order = np.argsort(src)                       # pair rows -> pair index p = s*K + k
    hq_g, hs_g = hq[order], hs[order]
    hq_r, hs_r = orc.moe_pairs_hidden(kind, blobs_np, X, eidx, D, MI, CLAMP)
    diff = hq_g.astype(np.int32) - hq_r
    assert np.max(np.abs(diff)) <= 1
    flips = int(np.count_nonzero(diff))
    assert flips <= max(3, max_flip_frac * diff.size), (flips, diff.size)
    print(f"hs max rel dev {float(np.max(np.abs(hs_g / hs_r - 1))):.2e}, mean {float(np.mean(hs_g / hs_r - 1)):.2e}")
    assert np.allclose(hs_g, hs_r, rtol=hs_rtol(), atol=0)
    want2 = orc.moe_pairs_combine(kind, blobs_np, hq_g, hs_g, eidx, ewt, D, MI)
    assert np.max(np.abs(out - want2)) <= 1e-5 * np.max(np.abs(want2))
    want = orc.moe_pairs_combine(kind, blobs_np, hq_r, hs_r, eidx, ewt, D, MI)
    flipped_tok = np.any(diff.reshape(S, K * MI) != 0, axis=1)
    scale = np.max(np.abs(want))
    err = np.max(np.abs(out - want), axis=1)
    assert np.all(err[~flipped_tok] <= 1e-4 * scale), float(np.max(err[~flipped_tok]) / scale)
    print(f"pairs {S * K}: {flips} requant flips of {diff.size} hidden codes in {int(flipped_tok.sum())} tokens; "
          f"max err unflipped {float(np.max(err[~flipped_tok]) / scale):.2e}")
    return flips


def test_moe_full_layer_config3(orc, engine):
    """S = 512, 128 q4_0 experts, Zipf-routed top-8, full output"""
    S = 512
    blobs = _gemma_blobs(600)
    X = synth.gaussian(601, (S, synth.GEMMA_D))
    eidx, ewt, _ = synth.zipf_routing(602, S, synth.GEMMA_E, synth.GEMMA_K)
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, synth.GEMMA_D, synth.GEMMA_MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), zz.ZZ_ACT_GEGLU_TANH)
    out_np = out.cpu().numpy()
    _full_check(orc, 0, blobs.cpu().numpy(), bank, X, eidx, ewt, out_np)
    # linearity in the router weights (an exact power-of-two scaling)
    out2 = zz.moe_ffn(bank, dev(X), dev(eidx), dev(2 * ewt), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out2 - 2 * out_np)) <= 1e-6 * np.max(np.abs(out_np))
    # token permutation: outputs permute with the tokens
    perm = synth.rng(8).permutation(S)
    out3 = zz.moe_ffn(bank, dev(X[perm]), dev(eidx[perm]), dev(ewt[perm]), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out3 - out_np[perm])) <= 1e-6 * np.max(np.abs(out_np))


@pytest.mark.parametrize("S", [1, 8])
def test_moe_decode_config2(orc, S):
    """Gemma-4 experts at decode (S = 1: 8 of 128 experts; S = 8: 64
    pairs, the largest call the decode kernels take) on the default engine, which routes
    these calls to the decode kernels; every pair and token checked"""
    blobs = _gemma_blobs(700)
    X = synth.gaussian(701 + S, (S, synth.GEMMA_D))
    eidx, ewt, _ = synth.zipf_routing(702 + S, S, synth.GEMMA_E, synth.GEMMA_K)
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, synth.GEMMA_D, synth.GEMMA_MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    _full_check(orc, 0, blobs.cpu().numpy(), bank, X, eidx, ewt, out)


@pytest.mark.parametrize("S", [1, 512])
def test_moe_maple_config4(orc, S, engine):
    """Maple ternary layer, 256 tq2 experts, D 2048, MI 512, top-8,
    clamped SwiGLU, decode and S = 512"""
    blobs = _maple_blobs(800)
    X = synth.gaussian(801 + S, (S, synth.MAPLE_D))
    eidx, ewt, _ = synth.zipf_routing(802 + S, S, synth.MAPLE_E, synth.MAPLE_K)
    bank = zz.ExpertBankDev(zz.GPU_FMT_TQ2, blobs, synth.MAPLE_D, synth.MAPLE_MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), zz.ZZ_ACT_SWIGLU_CLAMP, CLAMP).cpu().numpy()
    _full_check(orc, 3, blobs.cpu().numpy(), bank, X, eidx, ewt, out)


def test_moe_prefill_4096(orc, engine):
    """S = 4096 (BASELINE config 5's largest batch): many full 128-row items per expert
    on the tcgen05 engine, the capped-grid item striding on the mma.sync engine; sampled
    pairs (stage 1), sampled tokens (stage 2) and the size-independent properties"""
    S, K, D, MI = 4096, synth.GEMMA_K, synth.GEMMA_D, synth.GEMMA_MI
    blobs = _gemma_blobs(900)
    X = synth.gaussian(901, (S, D))
    eidx, ewt, _ = synth.zipf_routing(902, S, synth.GEMMA_E, K)
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
    out = zz.moe_ffn(bank, dev(X), dev(eidx), dev(ewt), zz.ZZ_ACT_GEGLU_TANH)
    out_np = out.cpu().numpy()
    blobs_np = blobs.cpu().numpy()
    src, hq, hs = ws_views(bank, S, K)
    slot = {int(p): r for r, p in enumerate(src)}
    toks = [0, 1, 777, 2048, 4095] + list(synth.rng(9).choice(S, size=11, replace=False))
    sub_e, sub_w = eidx[toks], ewt[toks]
    hq_r, hs_r = orc.moe_pairs_hidden(0, blobs_np, X[toks], sub_e, D, MI)
    rows = [slot[s * K + k] for s in toks for k in range(K)]
    diff = hq[rows].astype(np.int32) - hq_r
    assert np.max(np.abs(diff)) <= 1 and np.count_nonzero(diff) <= max(3, diff.size // 500)
    want2 = orc.moe_pairs_combine(0, blobs_np, hq[rows], hs[rows], sub_e, sub_w, D, MI)
    assert np.max(np.abs(out_np[toks] - want2)) <= 1e-5 * np.max(np.abs(want2))
    out2 = zz.moe_ffn(bank, dev(X), dev(eidx), dev(0.5 * ewt), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(2 * out2 - out_np)) <= 1e-6 * np.max(np.abs(out_np))
    perm = synth.rng(10).permutation(S)
    out3 = zz.moe_ffn(bank, dev(X[perm]), dev(eidx[perm]), dev(ewt[perm]), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out3 - out_np[perm])) <= 1e-6 * np.max(np.abs(out_np))
