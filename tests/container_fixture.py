"""Writes a small gemma4 container in the reference converter's format
(tools/convert_gemma4.py:133-167, 361-422): manifest.txt (cfg / esz / dense / expert
lines), dense.bin (tensors back to back; container format codes f32 0, q4_0 1) and
experts.bin ([gate | up | down] q4_0 blobs at 4096-aligned offsets). Every dense name
the engine's parser binds is present (gemma4.c:342-395), so the reference's own
manifest() accepts it. Test infrastructure."""
import os

import numpy as np

from zunzuncito_b200 import synth

LAYER_NAMES = ["input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
               "post_feedforward_layernorm", "pre_feedforward_layernorm_2", "post_feedforward_layernorm_1",
               "post_feedforward_layernorm_2", "layer_scalar", "q_proj", "k_proj", "v_proj", "o_proj", "q_norm",
               "k_norm", "mlp_gate", "mlp_up", "mlp_down", "router_proj", "router_scale", "router_pes"]


def write(dst, orc, L=2, E=8, D=256, MI=128, V=512, seed=0):
    """returns {"blobs": [L][E] expert blob bytes, "embed": q4_0 [V, D] bytes, "offsets": {(l, e): off}}"""
    os.makedirs(dst, exist_ok=True)
    dense, off = {}, 0
    with open(os.path.join(dst, "dense.bin"), "wb") as f:
        def add(name, fmt, arr, O, I):
            nonlocal off
            b = np.ascontiguousarray(arr).tobytes()
            f.write(b)
            dense[name] = (off, len(b), fmt, O, I)
            off += len(b)
        embed = orc.q40_quant_rows(synth.gaussian(seed + 1, (V, D), 0.02))
        add("embed_tokens", 1, embed, V, D)
        add("norm", 0, np.ones(D, np.float32), D, 1)
        for li in range(L):
            for n in LAYER_NAMES:
                add(f"layers.{li}.{n}", 0, np.zeros(4, np.float32), 4, 1)
    gb, db = MI * (D // 32) * 18, D * (MI // 32) * 18
    esz = 2 * gb + db
    offsets, blobs, eoff = {}, [], 0
    with open(os.path.join(dst, "experts.bin"), "wb") as f:
        for li in range(L):
            row = []
            for e in range(E):
                blob = np.concatenate([orc.q40_quant_rows(synth.gaussian(seed + 100 + 3 * (li * E + e) + i, shp, 0.02)).ravel()
                                       for i, shp in enumerate([(MI, D), (MI, D), (D, MI)])])
                pad = (-eoff) % 4096
                f.write(b"\0" * pad)
                eoff += pad
                f.write(blob.tobytes())
                offsets[(li, e)] = eoff
                eoff += esz
                row.append(blob)
            blobs.append(row)
    cfg = {"hidden": D, "n_layers": L, "n_heads": 2, "head_dim": 64, "global_head_dim": 64, "n_kv_heads": 1,
           "n_global_kv_heads": 1, "k_eq_v_global": 0, "n_experts": E, "topk": 2, "moe_inter": MI,
           "dense_inter": 256, "vocab": V, "sliding_window": 128, "ctx": 256, "eps": 1e-6,
           "final_logit_softcap": 30.0}
    with open(os.path.join(dst, "manifest.txt"), "w") as m:
        m.write("cfg layer_types " + " ".join("0" for _ in range(L)) + "\n")
        for k, v in cfg.items():
            m.write(f"cfg {k} {v}\n")
        m.write(f"esz {esz} {gb} {db}\n")
        m.write(f"ndense {len(dense)}\n")
        for k, (o, n, fmt, O, I) in dense.items():
            m.write(f"dense {k} {o} {n} {fmt} {O} {I}\n")
        m.write(f"nexpert {L * E}\n")
        for (li, e), o in offsets.items():
            m.write(f"expert {li} {e} {o}\n")
    return {"blobs": blobs, "embed": embed, "offsets": offsets, "esz": (esz, gb, db)}
