"""Seeded synthetic inputs with the shapes and value distributions of the benchmark
configurations (there are no checkpoints here): N(0, 0.02) weights, N(0, 1) hidden
states, ternary codes with P(c)=1/3 each, and Zipf(s=1.1)-skewed top-k routing standing
in for the usage skew the engines learn into usage.bin (gemma4.c:1286-1335).
All generators are numpy PCG64 streams keyed by an explicit seed."""
import numpy as np

# Gemma-4 26B-A4B routed experts (tools/convert_gemma4.py:21-23)
GEMMA_D, GEMMA_MI, GEMMA_E, GEMMA_K = 2816, 704, 128, 8
# Maple ternary experts (reference tests/test_metal_sim.c:158-160 and its README.md:12)
MAPLE_D, MAPLE_MI, MAPLE_E, MAPLE_K, MAPLE_CLAMP = 2048, 512, 256, 8, 7.0


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def gaussian(seed, shape, std=1.0):
    return (rng(seed).standard_normal(shape) * std).astype(np.float32)


def pack_tq2_codes(c):
    """codes c [O, I] in {0,1,2} -> [O, I/4] bytes: in each 64-weight group byte k holds
    weights k, k+16, k+32, k+48 at bits 0, 2, 4, 6 (tq2.h:46-51)."""
    O, I = c.shape
    g = c.reshape(O, I // 64, 4, 16).astype(np.uint8)  # [O, group, quarter, k]
    b = g[:, :, 0] | (g[:, :, 1] << 2) | (g[:, :, 2] << 4) | (g[:, :, 3] << 6)
    return b.reshape(O, I // 4)


def tq2_tensor(seed, O, I):
    """one tq2 tensor: alpha[O] f32 (|N(0,0.02)| + 1e-3) then packed codes"""
    r = rng(seed)
    alpha = (np.abs(r.standard_normal(O)) * 0.02 + 1e-3).astype(np.float32)
    codes = r.integers(0, 3, size=(O, I), dtype=np.uint8)
    return np.concatenate([alpha.view(np.uint8), pack_tq2_codes(codes).reshape(-1)])


def zipf_routing(seed, S, E, K, s=1.1):
    """top-K of N(0,1) logits + log(p_e), p_e ~ rank(e)^-s over a seeded permutation;
    descending order with ties on the lower index, then softmax over the K selected
    (the selection of gemma4.c:597-612 / maple.c:582-601)."""
    r = rng(seed)
    perm = r.permutation(E)
    p = np.empty(E)
    p[perm] = np.arange(1, E + 1, dtype=np.float64) ** -s
    p /= p.sum()
    logits = (r.standard_normal((S, E)) + np.log(p)[None, :]).astype(np.float32)
    idx = np.argsort(-logits, axis=1, kind="stable")[:, :K].astype(np.int32)
    top = np.take_along_axis(logits, idx, axis=1)
    w = np.exp(top - top[:, :1])
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return idx, w, logits


def q4a_tensor(seed, O, I):
    """one q4a tensor [O, I] in the reference layout (tq2.h:268-283): per 64-weight group
    fp16 d = |N(0,1)| * 0.01 + 0.002, fp16 m = N(0,1) * 0.05, uniform 4-bit codes"""
    r = rng(seed)
    g = np.zeros((O, I // 64, 36), np.uint8)
    g[:, :, 4:] = r.integers(0, 256, size=(O, I // 64, 32), dtype=np.uint8)
    d = (np.abs(r.standard_normal((O, I // 64))) * 0.01 + 0.002).astype(np.float16)
    m = (r.standard_normal((O, I // 64)) * 0.05).astype(np.float16)
    g[:, :, 0:2] = d.view(np.uint8).reshape(O, I // 64, 2)
    g[:, :, 2:4] = m.view(np.uint8).reshape(O, I // 64, 2)
    return g.reshape(-1)
