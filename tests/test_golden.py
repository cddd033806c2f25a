"""The oracle restatement against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). Runs without the reference tree."""
import os

import numpy as np
import pytest

from zunzuncito_b200 import synth

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def test_golden_q40(orc):
    w = synth.gaussian(1001, (64, 2816), 0.02)
    assert np.array_equal(orc.q40_quant_rows(w), G["q40_W"])
    xq, sx = orc.quant_act(G["q40_x"])
    assert np.array_equal(xq, G["q40_xq"]) and np.array_equal(sx, G["q40_sx"])
    y = orc.q40_matvec(G["q40_W"], xq[0], sx[0])
    assert np.max(np.abs(y - G["q40_y"])) <= 1e-5 * np.max(np.abs(G["q40_y"]))


def test_golden_q80(orc):
    w = synth.gaussian(1003, (32, 2048), 0.02)
    assert np.array_equal(orc.q80_quant_rows(w), G["q80_W"])
    y = orc.q80_matvec(G["q80_W"], G["q80_xq"][0], G["q80_sx"][0])
    assert np.max(np.abs(y - G["q80_y"])) <= 1e-5 * np.max(np.abs(G["q80_y"]))


def test_golden_tq2(orc):
    xq, sx, tot = orc.tq2_quant_act(G["tq2_x"])
    assert np.array_equal(xq, G["tq2_xq"]) and np.array_equal(sx, G["tq2_sx"]) and np.array_equal(tot, G["tq2_tot"])
    y = orc.tq2_matvec(G["tq2_T"], 64, xq[0], sx[0], tot[0])
    assert np.max(np.abs(y - G["tq2_y"])) <= 1e-5 * np.max(np.abs(G["tq2_y"]))


@pytest.mark.parametrize("kind,key", [(0, "g4"), (3, "mp")])
def test_golden_moe(orc, kind, key):
    E, D, MI, K, S = (int(v) for v in G["dims"])
    out = orc.moe_layer(kind, G[key + "_blobs"], G[key + "_X"], G[key + "_eidx"], G[key + "_ewt"], D, MI, 7.0)
    ref = G[key + "_out"]
    assert np.max(np.abs(out - ref)) <= 1e-4 * np.max(np.abs(ref))
