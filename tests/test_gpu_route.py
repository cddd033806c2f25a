"""The device routers (zz_route_gemma4_dev, zz_route_ling_dev) against the oracle's
restatement of route_row (pinned to the reference build in tests/test_oracle.py):
identical experts, weights within 1e-6 (CUDA's expf against the C library's); and the
router feeding the batch-union layer on the device with no host round trip."""
import numpy as np
import pytest
import torch

import zunzuncito_b200 as zz
from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("S", [1, 37, 512])
def test_gemma4_router(orc, S):
    D, E, K = synth.GEMMA_D, synth.GEMMA_E, synth.GEMMA_K
    res = synth.gaussian(20 + S, (S, D))
    res[0, :5] = 0.0
    proj, sc = synth.gaussian(21, (E, D), 0.02), synth.gaussian(22, (D,))
    pes = np.abs(synth.gaussian(23, (E,))) + 0.1
    want_i, want_w = orc.gemma4_route(res, proj, sc, pes, K)
    got_i, got_w = zz.route_gemma4(dev(res), dev(proj), dev(sc), dev(pes), K)
    assert np.array_equal(got_i.cpu().numpy(), want_i)
    assert np.max(np.abs(got_w.cpu().numpy() - want_w)) <= 1e-6 * np.max(np.abs(want_w))


@pytest.mark.parametrize("E,NG,TG,K,D", [(128, 8, 4, 8, 1536), (256, 8, 4, 8, 2048), (64, 1, 1, 6, 512)])
def test_ling_router(orc, E, NG, TG, K, D):
    S = 200
    xn = synth.gaussian(30, (S, D))
    rt, bi = synth.gaussian(31, (E, D), 0.05), synth.gaussian(32, (E,), 0.01)
    for norm in (0, 1):
        want_i, want_w = orc.ling_route(xn, rt, bi, K, NG, TG, norm, 2.5)
        got_i, got_w = zz.route_ling(dev(xn), dev(rt), dev(bi), K, NG, TG, norm, 2.5)
        assert np.array_equal(got_i.cpu().numpy(), want_i)
        assert np.max(np.abs(got_w.cpu().numpy() - want_w)) <= 1e-6 * np.max(np.abs(want_w))


def test_router_feeds_layer_on_device(orc):
    """residual -> router -> batch-union FFN, all on the device; the layer output equals
    the layer run on the oracle's routing of the same rows"""
    E, D, MI, K, S = 16, 512, 128, 4, 64
    blobs = np.stack([np.concatenate([orc.q40_quant_rows(synth.gaussian(40 + 3 * e + i, shp, 0.02)).ravel()
                                      for i, shp in enumerate([(MI, D), (MI, D), (D, MI)])]) for e in range(E)])
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, dev(blobs), D, MI)
    res = synth.gaussian(41, (S, D))
    proj, sc, pes = synth.gaussian(42, (E, D), 0.05), synth.gaussian(43, (D,)), np.abs(synth.gaussian(44, (E,)))
    r = dev(res)
    ei, ew = zz.route_gemma4(r, dev(proj), dev(sc), dev(pes), K)
    out = zz.moe_ffn(bank, r, ei, ew, zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    want_i, want_w = orc.gemma4_route(res, proj, sc, pes, K)
    assert np.array_equal(ei.cpu().numpy(), want_i)
    ref = zz.moe_ffn(bank, r, dev(want_i), dev(want_w), zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
    assert np.max(np.abs(out - ref)) <= 1e-5 * np.max(np.abs(ref))
