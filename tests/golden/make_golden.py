"""Generates tests/golden/golden.npz from the REFERENCE's own code (oracle/_ref,
compiled from the reference sources): its quantizers, its kernels and its engines'
expert_apply. Run where the reference tree exists:  python tests/golden/make_golden.py
The fixture then pins the oracle restatement and the CUDA path on machines without it."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402
from zunzuncito_b200 import synth  # noqa: E402


def main():
    ref = oracle.Reference()
    ref.set_threads(1)
    out = {}
    # config-1 style q4_0 matvec (64 rows of the 2816-wide shape)
    w = synth.gaussian(1001, (64, 2816), 0.02)
    W = ref.q40_quant_rows(w)
    x = synth.gaussian(1002, (1, 2816))
    xq, sx = ref.quant_act(x)
    out.update(q40_W=W, q40_x=x, q40_xq=xq, q40_sx=sx, q40_y=ref.q40_matvec(W, xq[0], sx[0]))
    # q8_0
    W8 = ref.q80_quant_rows(synth.gaussian(1003, (32, 2048), 0.02))
    x8 = synth.gaussian(1004, (1, 2048))
    xq8, sx8 = ref.quant_act(x8)
    out.update(q80_W=W8, q80_x=x8, q80_xq=xq8, q80_sx=sx8, q80_y=ref.q80_matvec(W8, xq8[0], sx8[0]))
    # tq2
    T = synth.tq2_tensor(1005, 64, 2048)
    xt = synth.gaussian(1006, (1, 2048))
    xqt, sxt, tot = ref.tq2_quant_act(xt)
    out.update(tq2_T=T, tq2_x=xt, tq2_xq=xqt, tq2_sx=sxt, tq2_tot=tot,
               tq2_y=ref.tq2_matvec(T, 64, xqt[0], sxt[0], tot[0]))
    # routed-expert layers through the engines' own expert_apply
    E, D, MI, K, S = 4, 128, 64, 2, 5
    blobs = []
    for e in range(E):
        g = ref.q40_quant_rows(synth.gaussian(1100 + 3 * e, (MI, D), 0.02))
        u = ref.q40_quant_rows(synth.gaussian(1101 + 3 * e, (MI, D), 0.02))
        d = ref.q40_quant_rows(synth.gaussian(1102 + 3 * e, (D, MI), 0.02))
        blobs.append(np.concatenate([g.ravel(), u.ravel(), d.ravel()]))
    blobs = np.stack(blobs)
    X = synth.gaussian(1200, (S, D))
    eidx, ewt, _ = synth.zipf_routing(1201, S, E, K)
    out.update(g4_blobs=blobs, g4_X=X, g4_eidx=eidx, g4_ewt=ewt, g4_out=ref.moe_layer(0, blobs, X, eidx, ewt, D, MI))
    mblobs = np.stack([np.concatenate([synth.tq2_tensor(1300 + 3 * e, MI, D), synth.tq2_tensor(1301 + 3 * e, MI, D),
                                       synth.tq2_tensor(1302 + 3 * e, D, MI)]) for e in range(E)])
    Xm = synth.gaussian(1400, (S, D))
    eim, ewm, _ = synth.zipf_routing(1401, S, E, K)
    out.update(mp_blobs=mblobs, mp_X=Xm, mp_eidx=eim, mp_ewt=ewm,
               mp_out=ref.moe_layer(3, mblobs, Xm, eim, ewm, D, MI, 7.0))
    out["dims"] = np.array([E, D, MI, K, S], np.int32)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"), **out)


if __name__ == "__main__":
    main()
