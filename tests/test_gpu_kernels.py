"""CUDA kernels through the C ABI against the oracle: quantizers and per-block integer
sums bit-exact, fp32 matvec outputs within 1e-4 of max|y| (the tolerance BASELINE
states; accumulation order differs), the gpu.h host surface, and declines."""
import ctypes

import numpy as np
import pytest
import torch

import zunzuncito_b200 as zz
from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-4  # max |y - y_ref| / max |y_ref|


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    yield
    torch.cuda.synchronize()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / (np.max(np.abs(b)) + 1e-30))


def q_weights(orc, fmt, seed, O, I):
    if fmt == zz.GPU_FMT_TQ2:
        return synth.tq2_tensor(seed, O, I)
    if fmt == zz.GPU_FMT_Q4A:
        return synth.q4a_tensor(seed, O, I)
    w = synth.gaussian(seed, (O, I), 0.02)
    return (orc.q40_quant_rows(w) if fmt == zz.GPU_FMT_Q40 else orc.q80_quant_rows(w)).reshape(-1)


def oracle_matvec(orc, fmt, Wb, O, I, xq, sx, tot):
    if fmt == zz.GPU_FMT_Q4A:
        return orc.q4a_matvec(Wb, O, xq, sx)
    if fmt == zz.GPU_FMT_Q40:
        return orc.q40_matvec(Wb.reshape(O, -1), xq, sx)
    if fmt == zz.GPU_FMT_Q80:
        return orc.q80_matvec(Wb.reshape(O, -1), xq, sx)
    return orc.tq2_matvec(Wb, O, xq, sx, tot)


def test_quant_act_bit_exact(orc):
    x = synth.gaussian(21, (9, 2816))
    x[1, :64] = 0.0
    x[2, 5] = 1e-30
    x[3, :32] = np.arange(32, dtype=np.float32) - 15.5          # exact .5 ties
    x[4, :32] = np.float32(3.0) * (np.arange(32) % 3 - 1)
    xq, sx, tot = zz.quant_act(dev(x), want_sxtot=True)
    exq, esx, etot = orc.tq2_quant_act(x)
    assert np.array_equal(xq.cpu().numpy(), exq)
    assert np.array_equal(sx.cpu().numpy(), esx)
    assert np.array_equal(tot.cpu().numpy(), etot)


@pytest.mark.parametrize("fmt", [zz.GPU_FMT_Q40, zz.GPU_FMT_Q80])
@pytest.mark.parametrize("scale", [0.02, 1.0, 1e-6])
def test_quant_rows_bit_exact(orc, fmt, scale):
    w = synth.gaussian(22, (37, 704), scale)
    w[0, :32] = 0.0
    w[1, :32] = 0.5; w[1, 7] = -0.5
    got = zz.quant_rows(fmt, dev(w)).cpu().numpy().reshape(37, -1)
    want = orc.q40_quant_rows(w) if fmt == zz.GPU_FMT_Q40 else orc.q80_quant_rows(w)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("fmt,O,I", [(zz.GPU_FMT_Q40, 37, 704), (zz.GPU_FMT_Q80, 19, 96), (zz.GPU_FMT_TQ2, 33, 128)])
def test_repack_roundtrip(orc, fmt, O, I):
    Wb = q_weights(orc, fmt, 23, O, I)
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    assert np.array_equal(t.unpack().cpu().numpy(), Wb)


@pytest.mark.parametrize("fmt,O,I", [(zz.GPU_FMT_Q40, 64, 2816), (zz.GPU_FMT_Q80, 40, 704), (zz.GPU_FMT_TQ2, 48, 2048)])
def test_blocksums_bit_exact(orc, fmt, O, I):
    Wb = q_weights(orc, fmt, 24, O, I)
    x = synth.gaussian(25, (1, I))
    xq, sx = orc.quant_act(x)
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    got = zz.blocksums(t, dev(xq[0])).cpu().numpy()
    Wrows = Wb[4 * O:].reshape(O, -1) if fmt == zz.GPU_FMT_TQ2 else Wb.reshape(O, -1)
    assert np.array_equal(got, orc.blocksums(fmt, Wrows, xq[0]))


@pytest.mark.parametrize("fmt,O,I", [
    (zz.GPU_FMT_Q40, 2816, 2816),
    (zz.GPU_FMT_Q40, 1, 32), (zz.GPU_FMT_Q40, 37, 704), (zz.GPU_FMT_Q40, 5, 8192), (zz.GPU_FMT_Q40, 9, 8224),
    (zz.GPU_FMT_Q80, 2816, 2816), (zz.GPU_FMT_Q80, 3, 96),
    (zz.GPU_FMT_TQ2, 512, 2048), (zz.GPU_FMT_TQ2, 2048, 512), (zz.GPU_FMT_TQ2, 7, 64), (zz.GPU_FMT_TQ2, 3, 8192 + 64),
])
def test_matvec_one_row(orc, fmt, O, I):
    Wb = q_weights(orc, fmt, 26, O, I)
    x = synth.gaussian(27, (1, I))
    xq, sx, tot = orc.tq2_quant_act(x)
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    y = zz.matvec(t, dev(xq), dev(sx), dev(tot)).cpu().numpy()[0]
    assert rel(y, oracle_matvec(orc, fmt, Wb, O, I, xq[0], sx[0], tot[0])) < TOL


@pytest.mark.parametrize("fmt", [zz.GPU_FMT_Q40, zz.GPU_FMT_Q80, zz.GPU_FMT_TQ2])
@pytest.mark.parametrize("S,O,I", [(2, 128, 256), (3, 200, 704), (17, 2816, 2816), (65, 130, 2048), (130, 64, 512)])
def test_matvec_many_rows(orc, fmt, S, O, I):
    Wb = q_weights(orc, fmt, 28, O, I)
    x = synth.gaussian(29, (S, I))
    xq, sx, tot = orc.tq2_quant_act(x)
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    y = zz.matvec(t, dev(xq), dev(sx), dev(tot)).cpu().numpy()
    for s in range(S):
        assert rel(y[s], oracle_matvec(orc, fmt, Wb, O, I, xq[s], sx[s], tot[s])) < TOL, s


@pytest.mark.parametrize("fmt,reps", [(zz.GPU_FMT_Q40, 12), (zz.GPU_FMT_Q80, 12), (zz.GPU_FMT_TQ2, 24)])
def test_matvec_streamed(orc, fmt, reps):
    """Matrices of >= 64 MB take the bulk-copy streamed kernel: 4099 distinct rows tiled
    `reps` times (O not a multiple of the 16-row tile), every row against the oracle."""
    O0, I = 4099, 2816
    W0 = q_weights(orc, fmt, 40, O0, I)
    O = O0 * reps
    if fmt == zz.GPU_FMT_TQ2:  # alpha[O] then codes[O][I/4]
        al, cd = W0[:4 * O0].view(np.float32), W0[4 * O0:].reshape(O0, I // 4)
        Wb = np.concatenate([np.tile(al, reps).view(np.uint8), np.tile(cd, (reps, 1)).reshape(-1)])
    else:
        Wb = np.tile(W0.reshape(O0, -1), (reps, 1)).reshape(-1)
    assert zz.lib.zz_qtensor_bytes(fmt, O, I) >= 64 << 20
    x = synth.gaussian(41, (1, I))
    xq, sx, tot = orc.tq2_quant_act(x)
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    y = zz.matvec(t, dev(xq), dev(sx), dev(tot)).cpu().numpy()[0]
    want = oracle_matvec(orc, fmt, W0, O0, I, xq[0], sx[0], tot[0])
    assert rel(y, np.tile(want, reps)) < TOL


def test_gpu_h_surface(orc):
    """gpu_init / gpu_map / gpu_matmul exactly as an engine calls them (gemma4.c:445):
    by default f32 activations (the reference GPU backend's numerics, checked against
    q40_dot_f32 & co. at 1e-4 like --check-gpu), with zz_gpu_set_act_quant(1) the q8_0
    integer dots; and the q8_0-activation kernel signatures gpu_*_matvec."""
    L = zz.lib
    assert L.gpu_init() == 1, L.gpu_last_error()
    assert L.gpu_ready() == 1
    assert b"B200" in L.gpu_name() or b"sm_10" in L.gpu_name()
    O, I, It = 300, 2816, 2048
    tens = {zz.GPU_FMT_Q40: (q_weights(orc, zz.GPU_FMT_Q40, 30, O, I), I),
            zz.GPU_FMT_Q80: (q_weights(orc, zz.GPU_FMT_Q80, 31, O, I), I),
            zz.GPU_FMT_TQ2: (q_weights(orc, zz.GPU_FMT_TQ2, 32, O, It), It),
            zz.GPU_FMT_Q4A: (q_weights(orc, zz.GPU_FMT_Q4A, 33, O, It), It)}
    # one page-aligned region holding all four tensors, like the dense blob
    total = sum(w.size for w, _ in tens.values())
    region = np.zeros((total // 4096 + 2) * 4096, np.uint8)
    base, off, where = region.ctypes.data, 0, {}
    for fmt, (w, _) in tens.items():
        region[off:off + w.size] = w
        where[fmt] = off
        off += (w.size + 15) // 16 * 16
    assert L.gpu_map(ctypes.c_void_p(base), region.size) == 1, L.gpu_last_error()
    try:
        for S in (1, 3):
            for fmt, (w, In) in tens.items():
                x = synth.gaussian(33 + S + fmt, (S, In))
                Wp = ctypes.c_void_p(base + where[fmt])
                y = np.zeros((S, O), np.float32)
                assert L.zz_gpu_set_act_quant(0) == 1
                call = (L.gpu_q40_matmul(y.ctypes.data, Wp, x.ctypes.data, O, In, S) if fmt == zz.GPU_FMT_Q40
                        else L.gpu_matmul(fmt, y.ctypes.data, Wp, x.ctypes.data, O, In, S))
                assert call == 1, L.gpu_last_error()
                for s in range(S):
                    assert rel(y[s], orc.matvec_f32(fmt, w, O, In, x[s])) < TOL, (fmt, s)
                assert L.zz_gpu_set_act_quant(1) == 1
                y8 = np.zeros((S, O), np.float32)
                assert L.gpu_matmul(fmt, y8.ctypes.data, Wp, x.ctypes.data, O, In, S) == 1, L.gpu_last_error()
                xq, sx, tot = orc.tq2_quant_act(x)
                for s in range(S):
                    assert rel(y8[s], oracle_matvec(orc, fmt, w, O, In, xq[s], sx[s], tot[s])) < TOL, (fmt, s)
                # the kernel-level signatures (q40.h:308, 456; tq2.h:134, 395) on host buffers
                y1 = np.zeros(O, np.float32)
                if fmt == zz.GPU_FMT_TQ2:
                    ok = L.gpu_tq2_matvec(y1.ctypes.data, Wp, xq[0].ctypes.data, sx[0].ctypes.data, float(tot[0]), O, In)
                else:
                    f = {zz.GPU_FMT_Q40: L.gpu_q40_matvec, zz.GPU_FMT_Q80: L.gpu_q80_matvec,
                         zz.GPU_FMT_Q4A: L.gpu_q4a_matvec}[fmt]
                    ok = f(y1.ctypes.data, Wp, xq[0].ctypes.data, sx[0].ctypes.data, O, In)
                assert ok == 1, L.gpu_last_error()
                assert rel(y1, oracle_matvec(orc, fmt, w, O, In, xq[0], sx[0], tot[0])) < TOL, fmt
        L.zz_gpu_set_act_quant(0)
        # declines: bad shape, unmapped pointer
        y = np.zeros(8, np.float32)
        assert L.gpu_matmul(zz.GPU_FMT_Q4A, y.ctypes.data, ctypes.c_void_p(base), y.ctypes.data, 8, 96, 1) == 0
        assert L.gpu_matmul(zz.GPU_FMT_Q40, y.ctypes.data, ctypes.c_void_p(base), y.ctypes.data, 8, 48, 1) == 0
        other = np.zeros(4096, np.uint8)
        assert L.gpu_q40_matmul(y.ctypes.data, other.ctypes.data, y.ctypes.data, 1, 32, 1) == 0
        assert b"gpu_map" in L.gpu_last_error()
    finally:
        L.zz_gpu_set_act_quant(0)
        assert L.gpu_unmap(ctypes.c_void_p(base)) == 1
    assert L.gpu_q40_matmul(y.ctypes.data, ctypes.c_void_p(base), y.ctypes.data, 1, 32, 1) == 0


@pytest.mark.parametrize("fmt,O,I", [(zz.GPU_FMT_Q40, 2816, 2816), (zz.GPU_FMT_Q80, 64, 704), (zz.GPU_FMT_TQ2, 512, 2048),
                                     (zz.GPU_FMT_Q4A, 4096, 2048), (zz.GPU_FMT_Q40, 7, 32 * 1599)])
def test_matvec_f32_activations(orc, fmt, O, I):
    """zz_matvec_f32_dev against q40_dot_f32 / q80_dot_f32 / tq2_dot_f32 / q4a_dot_f32,
    two rows"""
    Wb = q_weights(orc, fmt, 70, O, I)
    x = synth.gaussian(71, (2, I))
    t = zz.QTensorDev(fmt, dev(Wb), O, I)
    y = torch.empty((2, O), device="cuda")
    x_d = dev(x)   # held for the call
    zz.check(zz.lib.zz_matvec_f32_dev(ctypes.byref(t.t), ctypes.c_void_p(x_d.data_ptr()),
                                      ctypes.c_void_p(y.data_ptr()), 2, None), "zz_matvec_f32_dev")
    y = y.cpu().numpy()
    for s in range(2):
        assert rel(y[s], orc.matvec_f32(fmt, Wb, O, I, x[s])) < TOL, s


@pytest.mark.parametrize("O,I", [(4096, 2048), (37, 128)])
def test_q4a_repack_and_matvec(orc, O, I):
    """q4a planes round-trip to the reference layout; the q8_0-activation matvec matches
    q4a_dot (tq2.h:390-408) at 1e-4 for 1 and 3 rows"""
    Wb = q_weights(orc, zz.GPU_FMT_Q4A, 72, O, I)
    t = zz.QTensorDev(zz.GPU_FMT_Q4A, dev(Wb), O, I)
    assert np.array_equal(t.unpack().cpu().numpy(), Wb)
    for S in (1, 3):
        x = synth.gaussian(73 + S, (S, I))
        xq, sx = orc.quant_act(x)
        y = zz.matvec(t, dev(xq), dev(sx)).cpu().numpy()
        for s in range(S):
            assert rel(y[s], orc.q4a_matvec(Wb, O, xq[s], sx[s])) < TOL


@pytest.mark.parametrize("engine", ["gemma4_zz", "maple_zz"])
def test_reference_engine_check_gpu(engine):
    """The reference engines' own source, built with the GPU backend on (-DCOLI_METAL)
    and linked against libzz_cuda.so in place of metal.o (oracle/Makefile), run their
    own --check-gpu: six shapes each (gemma4.c:2315-2361: q4_0 projections and experts;
    maple.c:1756-1800: tq2 projections / experts and the q4a lm_head / centroids), every
    one within their 1e-4 of the exact-activation dot."""
    import os
    import subprocess
    import tempfile
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", engine)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} not built (the reference tree is needed to build it)")
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([exe, d, "--check-gpu"], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    lines = [ln for ln in r.stdout.splitlines() if "max rel err" in ln]
    assert len(lines) == 6, r.stdout + r.stderr
    assert all(ln.rstrip().endswith(" ok") for ln in lines), r.stdout
    assert r.returncode == 0, r.stdout + r.stderr


def test_ep_pack_unpack_layout():
    """zz_ep_pack_dev / zz_ep_unpack_dev against the torch construction of the same
    exchange rows (ep._exchange_torch's layout), with invalid and out-of-range ids."""
    from zunzuncito_b200 import ep
    S, D, K, world, per = 37, 2816, 8, 4, 32
    r = synth.rng(50)
    xq = torch.from_numpy(r.integers(-127, 128, size=(S, D), dtype=np.int8)).cuda()
    xs = torch.from_numpy(r.random((S, D // 32), dtype=np.float32)).cuda()
    e = r.integers(-1, world * per + 3, size=(S, K)).astype(np.int32)
    eidx = torch.from_numpy(e).cuda()
    ewt = torch.from_numpy(r.random((S, K), dtype=np.float32)).cuda()
    pay = zz.ep_pack(xq, xs, eidx, ewt, world, per)
    assert pay.shape == (world, S, zz.lib.zz_ep_row_bytes(D, K))
    got = zz.ep_unpack(pay, D, K)
    for d in range(world):
        sl = slice(d * S, (d + 1) * S)
        assert torch.equal(got[0][sl], xq) and torch.equal(got[1][sl], xs)
        mine = (eidx >= 0) & (torch.div(eidx, per, rounding_mode="floor") == d)
        assert torch.equal(got[2][sl], torch.where(mine, eidx - d * per, torch.full_like(eidx, -1)))
        assert torch.equal(got[3][sl], torch.where(mine, ewt, torch.zeros_like(ewt)))


@pytest.mark.parametrize("O,cap", [(65536, 30.0), (1000, 0.0), (4099, 30.0)])
def test_lm_head_softcap(orc, O, cap):
    """tied lm_head + final-logit softcap (gemma4.c:1270-1274); 65536 x 2816 q4_0 (104 MB)
    takes the streamed kernel with the softcap in its epilogue, the small ones the
    register kernel and a separate pass"""
    I = 2816
    g = torch.Generator(device="cuda").manual_seed(80)
    w = torch.randn((O, I), generator=g, device="cuda") * 0.02
    Wq = zz.quant_rows(zz.GPU_FMT_Q40, w)
    del w
    t = zz.QTensorDev(zz.GPU_FMT_Q40, Wq, O, I)
    x = synth.gaussian(81, (1, I)) * 4
    xq, sx = orc.quant_act(x)
    y = torch.empty(O, device="cuda")
    xq_d, sx_d = dev(xq), dev(sx)   # held for the call
    zz.check(zz.lib.zz_lm_head_dev(ctypes.byref(t.t), ctypes.c_void_p(xq_d.data_ptr()),
                                   ctypes.c_void_p(sx_d.data_ptr()), None, float(cap),
                                   ctypes.c_void_p(y.data_ptr()), None), "zz_lm_head_dev")
    want = orc.q40_matvec(Wq.cpu().numpy().reshape(O, -1), xq[0], sx[0]).astype(np.float64)
    if cap > 0:
        want = np.tanh(want / cap) * cap
    assert rel(y.cpu().numpy(), want) < TOL


def _pow2_inputs(fmt, O, S, seed):
    """one 32-weight block per row with power-of-two scales: q4_0 / q8_0 codes random, every
    fp16 block scale 2^-4; activations k * 2^-3 with each row's block max |x| = 127 * 2^-3,
    so q8_0 gives xq = 8 x and sx = 2^-3 exactly. Then y = 2^-7 * (the block's integer sum),
    exact in fp32 whatever the kernel's arithmetic order."""
    r = synth.rng(seed)
    bb = 18 if fmt == zz.GPU_FMT_Q40 else 34
    W = np.zeros((O, bb), np.uint8)
    W[:, 0:2] = np.frombuffer(np.float16(2.0 ** -4).tobytes(), np.uint8)
    W[:, 2:] = r.integers(0, 256, size=(O, bb - 2), dtype=np.uint8)
    if fmt == zz.GPU_FMT_Q80:
        W[:, 2:][W[:, 2:] == 128] = 129           # q8_0 codes stay in [-127, 127]
    xq = r.integers(-127, 128, size=(S, 32)).astype(np.int8)
    xq[:, 5] = 127
    x = (xq.astype(np.float32) * np.float32(0.125))
    if fmt == zz.GPU_FMT_Q40:
        q = np.concatenate([W[:, 2:] & 15, W[:, 2:] >> 4], axis=1).astype(np.int32) - 8
    else:
        q = W[:, 2:].view(np.int8).astype(np.int32)
    ints = xq.astype(np.int32) @ q.T             # [S, O] block integer sums
    return W.reshape(-1), x, ints


@pytest.mark.parametrize("fmt", [zz.GPU_FMT_Q40, zz.GPU_FMT_Q80])
@pytest.mark.parametrize("O,S", [(1000, 1), (2200000, 1), (300, 5)])
def test_block_integers_exact_on_production_kernels(orc, fmt, O, S):
    """I = 32 with power-of-two scales makes every production matvec output the exact block
    integer times 2^-7: the register GEMV (S=1, small), the streamed GEMV (S=1, >= 64 MB:
    4M rows), the int8 mma.sync GEMM (S>1); all must equal the integers bit for bit"""
    W, x, ints = _pow2_inputs(fmt, O, S, 90 + fmt)
    xq, sx = orc.quant_act(x)
    assert np.all(sx == np.float32(0.125)) and np.array_equal(xq.astype(np.float32), x * 8)
    t = zz.QTensorDev(fmt, dev(W), O, 32)
    y = zz.matvec(t, dev(xq), dev(sx)).cpu().numpy()
    assert np.array_equal(y.astype(np.float64) * 128.0, ints.astype(np.float64))
