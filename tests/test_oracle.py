"""The CPU restatement (oracle/zz_oracle.c) against the reference's own kernels and
engine routines compiled from its sources (oracle/_ref/libzzref.so). Integer and byte
results must be identical; fp32 results agree to accumulation-order rounding."""
import numpy as np
import pytest

from zunzuncito_b200 import synth


def test_fp16_all_halves(orc, ref):
    for h in range(0, 65536, 1):
        a, b = orc.fp16_to_f32(h), ref.fp16_to_f32(h)
        assert (np.isnan(a) and np.isnan(b)) or a == b, h


def test_fp16_from_f32(orc, ref):
    r = synth.rng(1)
    vals = np.concatenate([
        r.standard_normal(20000).astype(np.float32) * np.float32(0.01),
        (r.standard_normal(5000) * 1e-6).astype(np.float32),          # subnormal halves
        (r.standard_normal(2000) * 3e4).astype(np.float32),           # near overflow
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, 2.0 ** -14, np.inf, -np.inf], np.float32)])
    for v in vals:
        assert orc.f32_to_fp16(v) == ref.f32_to_fp16(v), v


@pytest.mark.parametrize("scale", [0.02, 1.0, 1e-6])
def test_weight_quantizers_bit_exact(orc, ref, scale):
    w = synth.gaussian(2, (64, 512), scale)
    w[3, :32] = 0.0                       # all-zero block
    w[4, :32] = 0.25; w[4, 5] = -0.25     # ties in |x|
    assert np.array_equal(orc.q40_quant_rows(w), ref.q40_quant_rows(w))
    assert np.array_equal(orc.q80_quant_rows(w), ref.q80_quant_rows(w))


def test_act_quantizers_bit_exact(orc, ref):
    x = synth.gaussian(3, (16, 2816))
    x[1, :64] = 0.0
    x[2, :32] = np.float32(127.0) * np.arange(32, dtype=np.float32) / 32
    a, b = orc.quant_act(x), ref.quant_act(x)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    a, b = orc.tq2_quant_act(x), ref.tq2_quant_act(x)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)


def _summand_scale(fmt, wrow_deq, xq, sx):
    return float(np.sum(np.abs(wrow_deq * xq.astype(np.float64) * np.repeat(sx, 32)))) + 1e-6


def _deq_q40(row):
    blk = row.reshape(-1, 18)
    d = blk[:, :2].copy().view(np.float16).astype(np.float64)
    q = np.concatenate([blk[:, 2:] & 15, blk[:, 2:] >> 4], axis=1).astype(np.float64) - 8
    return (q * d).reshape(-1)


def test_q40_dot_matches_reference(orc, ref):
    I = 2816
    W = orc.q40_quant_rows(synth.gaussian(4, (40, I), 0.02))
    x = synth.gaussian(5, (1, I))
    xq, sx = orc.quant_act(x)
    for o in range(W.shape[0]):
        a, b = orc.q40_dot(W[o], xq[0], sx[0]), ref.q40_dot(W[o], xq[0], sx[0])
        assert abs(a - b) / _summand_scale(1, _deq_q40(W[o]), xq[0], sx[0]) < 1e-5


def test_q40_blocksums_exact(orc):
    I = 704
    W = orc.q40_quant_rows(synth.gaussian(6, (8, I), 0.02))
    xq, sx = orc.quant_act(synth.gaussian(7, (1, I)))
    got = orc.blocksums(1, W, xq[0])
    blk = W.reshape(8, -1, 18)
    q = np.concatenate([blk[:, :, 2:] & 15, blk[:, :, 2:] >> 4], axis=2).astype(np.int64) - 8
    want = np.einsum("obj,bj->ob", q, xq[0].reshape(-1, 32).astype(np.int64))
    assert np.array_equal(got, want)


def test_q80_dot_and_matvec(orc, ref):
    I = 2048
    W = orc.q80_quant_rows(synth.gaussian(8, (96, I), 0.02))
    xq, sx = orc.quant_act(synth.gaussian(9, (1, I)))
    ya, yb = orc.q80_matvec(W, xq[0], sx[0]), ref.q80_matvec(W, xq[0], sx[0])
    assert np.max(np.abs(ya - yb)) <= 1e-5 * np.max(np.abs(yb))
    bs = orc.blocksums(2, W, xq[0])
    q = W.reshape(96, -1, 34)[:, :, 2:].view(np.int8).astype(np.int64)
    assert np.array_equal(bs, np.einsum("obj,bj->ob", q, xq[0].reshape(-1, 32).astype(np.int64)))


def test_tq2_dot_and_matvec(orc, ref):
    O, I = 96, 2048
    T = synth.tq2_tensor(10, O, I)
    xq, sx, tot = orc.tq2_quant_act(synth.gaussian(11, (1, I)))
    ya = orc.tq2_matvec(T, O, xq[0], sx[0], tot[0])
    yb = ref.tq2_matvec(T, O, xq[0], sx[0], tot[0])
    assert np.max(np.abs(ya - yb)) <= 1e-5 * np.max(np.abs(yb))


def test_q40_matvec_config1(orc, ref):
    """BASELINE config 1 shape: 2816 x 2816 q4_0 against a q8_0 activation."""
    W = orc.q40_quant_rows(synth.gaussian(12, (2816, 2816), 0.02))
    xq, sx = orc.quant_act(synth.gaussian(13, (1, 2816)))
    ya, yb = orc.q40_matvec(W, xq[0], sx[0]), ref.q40_matvec(W, xq[0], sx[0])
    assert np.max(np.abs(ya - yb)) <= 1e-5 * np.max(np.abs(yb))


def test_route_topk(orc, ref):
    logits = synth.gaussian(14, (64, 128))
    logits[0, 5] = logits[0, 9] = 9.0                   # tie: lower index first
    a, b = orc.route_topk(logits, 8), ref.route_topk(logits, 8)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert a[0][0, 0] == 5 and a[0][0, 1] == 9


def _q4_blobs(orc, seed, E, D, MI, q80=False):
    quant = orc.q80_quant_rows if q80 else orc.q40_quant_rows
    blobs = []
    for e in range(E):
        g = quant(synth.gaussian(seed + 3 * e, (MI, D), 0.02))
        u = quant(synth.gaussian(seed + 3 * e + 1, (MI, D), 0.02))
        d = quant(synth.gaussian(seed + 3 * e + 2, (D, MI), 0.02))
        blobs.append(np.concatenate([g.ravel(), u.ravel(), d.ravel()]))
    return np.stack(blobs)


def _tq2_blobs(seed, E, D, MI):
    return np.stack([np.concatenate([synth.tq2_tensor(seed + 3 * e, MI, D), synth.tq2_tensor(seed + 3 * e + 1, MI, D),
                                     synth.tq2_tensor(seed + 3 * e + 2, D, MI)]) for e in range(E)])


@pytest.mark.parametrize("S", [1, 7])
def test_moe_layer_gemma_matches_engine(orc, ref, S):
    """batch-union layer vs gemma4.c's own expert_apply (batch path at S>1)"""
    E, D, MI, K = 8, 256, 128, 2
    blobs = _q4_blobs(orc, 100, E, D, MI)
    X = synth.gaussian(15, (S, D))
    eidx, ewt, _ = synth.zipf_routing(16, S, E, K)
    a = orc.moe_layer(0, blobs, X, eidx, ewt, D, MI)
    b = ref.moe_layer(0, blobs, X, eidx, ewt, D, MI)
    assert np.max(np.abs(a - b)) <= 1e-4 * np.max(np.abs(b))


@pytest.mark.parametrize("S", [1, 6])
def test_moe_layer_maple_matches_engine(orc, ref, S):
    E, D, MI, K = 8, 256, 128, 2
    blobs = _tq2_blobs(200, E, D, MI)
    X = synth.gaussian(17, (S, D))
    eidx, ewt, _ = synth.zipf_routing(18, S, E, K)
    a = orc.moe_layer(3, blobs, X, eidx, ewt, D, MI, 7.0)
    b = ref.moe_layer(3, blobs, X, eidx, ewt, D, MI, 7.0)
    assert np.max(np.abs(a - b)) <= 1e-4 * np.max(np.abs(b))


def test_f32_activation_dots_match_reference(orc, ref):
    """the exact-activation dots the GPU backend is checked against (q40_dot_f32,
    q80_dot_f32, tq2_dot_f32, q4a_dot_f32): the same double arithmetic, so equal"""
    import ctypes
    I = 2048
    x = synth.gaussian(60, (I,))
    W4 = orc.q40_quant_rows(synth.gaussian(61, (5, I), 0.02))
    W8 = orc.q80_quant_rows(synth.gaussian(62, (5, I), 0.02))
    T2 = synth.tq2_tensor(63, 5, I)
    A4 = synth.q4a_tensor(64, 5, I)
    P, F, Ii = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
    p = lambda a: np.ascontiguousarray(a).ctypes.data_as(P)  # noqa: E731
    for o in range(5):
        for name, row in [("q40_dot_f32", W4[o]), ("q80_dot_f32", W8[o]), ("q4a_dot_f32", A4.reshape(5, -1)[o])]:
            a = orc.fn(name, F, [P, P, Ii])(p(row), p(x), I)
            b = ref.fn(name, F, [P, P, Ii])(p(row), p(x), I)
            assert a == b, (name, o)
        al = T2[:20].view(np.float32)[o]
        codes = T2[20:].reshape(5, -1)[o]
        a = orc.fn("tq2_dot_f32", F, [P, F, P, Ii])(p(codes), float(al), p(x), I)
        b = ref.fn("tq2_dot_f32", F, [P, F, P, Ii])(p(codes), float(al), p(x), I)
        assert a == b, o


def test_q4a_dot_matches_reference(orc, ref):
    """q4a_dot with q8_0 activations: the restatement (scalar, double) against the
    reference build's AVX2 path (f32 lanes) within 1e-5 of the summand magnitude"""
    import ctypes
    I = 2048
    xq, sx = orc.quant_act(synth.gaussian(65, (1, I)))
    A4 = synth.q4a_tensor(66, 8, I).reshape(8, -1)
    P, F, Ii = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
    p = lambda a: np.ascontiguousarray(a).ctypes.data_as(P)  # noqa: E731
    for o in range(8):
        a = orc.fn("q4a_dot", F, [P, P, P, Ii])(p(A4[o]), p(xq[0]), p(sx[0]), I)
        b = ref.fn("q4a_dot", F, [P, P, P, Ii])(p(A4[o]), p(xq[0]), p(sx[0]), I)
        scale = float(np.sum(np.abs(xq[0].astype(np.float64) * np.repeat(sx[0], 32)))) * 0.1
        assert abs(a - b) <= 1e-5 * scale, o


def test_gemma4_router_matches_reference(orc, ref):
    """route_row (gemma4.c:581-613): identical experts and weights"""
    S, D, E, K = 64, 2816, 128, 8
    res = synth.gaussian(1, (S, D))
    proj, sc = synth.gaussian(2, (E, D), 0.02), synth.gaussian(3, (D,))
    pes = np.abs(synth.gaussian(4, (E,)))
    a, b = orc.gemma4_route(res, proj, sc, pes, K), ref.gemma4_route(res, proj, sc, pes, K)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.parametrize("E,NG,TG,K", [(256, 8, 4, 8), (128, 8, 4, 8), (64, 1, 1, 6)])
def test_ling_router_matches_reference(orc, ref, E, NG, TG, K):
    """ling's grouped route_row (ling.c:705-789): identical experts and weights"""
    S, D = 48, 1536
    xn = synth.gaussian(5, (S, D))
    rt, bi = synth.gaussian(6, (E, D), 0.05), synth.gaussian(7, (E,), 0.01)
    for norm in (0, 1):
        a = orc.ling_route(xn, rt, bi, K, NG, TG, norm, 2.5)
        b = ref.ling_route(xn, rt, bi, K, NG, TG, norm, 2.5)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
