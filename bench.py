"""Benchmark of the quantized matrix hot path on B200.

Headline (one JSON line on rank 0): MoE layer throughput, token-layers per second,
of the batch-union routed-expert FFN over a Gemma-4-shaped 30-layer stack of resident
q4_0 experts (BASELINE configs 3 and 5: 128 experts x 30 layers = 3840 experts,
12.85 GB in HBM; D 2816, inter 704, top-8, Zipf(1.1)-skewed routing, S tokens per step).
One step = every layer of the stack applied to S tokens; each layer reads ~428 MB of
distinct expert weights, far beyond the 126 MB L2, so no L2 flush is needed.
Sub-benchmarks in the same line: the config-1 q4_0 GEMV (HBM GB/s), the config-2
decode experts, the S=4096 prefill layer (int8 TOPS) and the Maple tq2 layer.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl zz|reference]
Under torchrun (N > 1) experts are sharded across ranks (expert parallelism) and the
routed q8_0 activations move with an NCCL all-to-all; see zunzuncito_b200/ep.py.
"""
import argparse
import ctypes
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, MI, E, K = 2816, 704, 128, 8
LAYERS = 30
EXPERT_BYTES = 3345408        # 2*(704*88*18) + 2816*22*18 (q40.h:313)
GEMV_BYTES = 2816 * 1584 + 2816 + 88 * 4 + 2816 * 4   # config 1, per 2816x2816 GEMV
MACS_PER_PAIR = 3 * MI * D    # gate + up + down per (token, expert)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="zz", choices=["zz", "reference"])
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-sub", action="store_true", help="skip the sub-benchmarks")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--profile-case", choices=["moe", "gemv", "decode", "prefill", "maple", "lmhead", "route", "f32",
                                               "ep"],
                    help="run a small case of one kernel family a few times and exit (for ncu)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """NVML samples (read-only) of SM clock and throttle reasons during the timed region."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index, period=0.1):
        self.index, self.period, self.rows, self.stop = index, period, [], threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # noqa: BLE001
            self.nv, self.err = None, str(e)
        return self

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.rows.append((sm, rs, pw))
            except Exception:  # noqa: BLE001
                pass
            self.stop.wait(self.period)

    def __exit__(self, *a):
        self.stop.set()
        if self.nv:
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [r[0] for r in self.rows]
        reasons = sorted({n for r in self.rows for n, bit in self.REASONS.items() if r[1] & bit})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": self.max_sm, "reasons": reasons,
                "samples": len(self.rows), "power_w_max": max(r[2] for r in self.rows)}


# ----------------------------------------------------------------------------- data
def make_stack(zz, torch, layers, seed, keep_host_layer0=False):
    """layers x 128 q4_0 experts quantized on device (bit-exact with q40_quant_row),
    packed into expert banks; optionally a host copy of layer 0's reference blobs."""
    stride = zz.expert_blob_bytes(zz.GPU_FMT_Q40, D, MI)
    gb = zz.ref_tensor_bytes(zz.GPU_FMT_Q40, MI, D)
    g = torch.Generator(device="cuda").manual_seed(seed)
    banks, host0 = [], None
    for layer in range(layers):
        blobs = torch.empty((E, stride), dtype=torch.uint8, device="cuda")
        for i, (O, I) in enumerate([(MI, D), (MI, D), (D, MI)]):
            w = torch.randn((E * O, I), generator=g, device="cuda") * 0.02
            q = zz.quant_rows(zz.GPU_FMT_Q40, w).view(E, -1)
            blobs[:, i * gb:i * gb + q.shape[1]] = q
            del w, q
        banks.append(zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI))
        if keep_host_layer0 and layer == 0:
            host0 = blobs.cpu().numpy()
        del blobs
    torch.cuda.synchronize()
    return banks, host0


def routing(synth, layers, S, seed):
    return [synth.zipf_routing(seed + 17 * l, S, E, K)[:2] for l in range(layers)]


def stack_config(S, L, routes):
    """the headline workload's config (both arms name the same one)"""
    layer_bytes = float(np.mean([len(np.unique(r[0])) for r in routes])) * EXPERT_BYTES
    return {"workload": f"Gemma-4 batch-union MoE stack: {L} layers x 128 q4_0 experts (12.85 GB resident), "
                        f"S={S} tokens/step, top-8 Zipf(1.1) routing, GeGLU",
            "tokens": S, "layers": L, "experts_per_layer": E, "hidden": D, "inter": MI, "topk": K,
            "parallelism": "ep1",
            "l2": "no flush: each layer reads ~{:.0f} MB of distinct experts > 126 MB L2".format(layer_bytes / 1e6)}


def gateup_alg_bytes(S, distinct):
    """algorithmic bytes of one gate/up launch: the distinct experts' gate+up planes
    (2 * 704 * 88 * 18 B each), the gathered q8_0 rows (2816 + 88*4 B per pair) and the
    requantized hidden rows written (704 + 22*4 B per pair)"""
    return distinct * 2 * MI * (D // 32) * 18 + S * K * (D + 4 * D // 32) + S * K * (MI + 4 * MI // 32)


# DRAM bytes (read + write) per gate/up launch measured by ncu on `bench.py --profile-case
# moe` (the same kernel and shapes, routings zipf_routing(88 + l), l = 0, 1; 4 launches):
# the full 30-layer stack is too large to capture, so the bench scales this by the
# algorithmic bytes of its own routing.
PROFILE_GU_TRAFFIC = 206104960.0 + 5479616.0   # mean read + write of the 4 gate/up launches


def timed(torch, fn, steps, warmup, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def profile_case(kind, zz, torch, synth):
    """small cases sized for an ncu capture (a few GB at most on the device); the
    MoE cases run whichever engine ZZ_MOE_KERNEL selects"""
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    if kind == "gemv":
        G = 64  # 64 distinct 2816 x 2816 q4_0 matrices stacked: 285 MB > L2
        w = torch.randn((G * 2816, 2816), device="cuda") * 0.02
        T = zz.QTensorDev(zz.GPU_FMT_Q40, zz.quant_rows(zz.GPU_FMT_Q40, w), G * 2816, 2816)
        del w
        xq, sx, _ = zz.quant_act(torch.randn((1, 2816), device="cuda"))
        for _ in range(3):
            zz.matvec(T, xq, sx)
    elif kind == "lmhead":
        # tied lm_head 262144 x 2816 q4_0 (415 MiB) with the softcap
        V = 262144
        Wl = torch.empty(V * 1584, dtype=torch.uint8, device="cuda")
        for c0 in range(0, V, 32768):
            Wl[c0 * 1584:(c0 + 32768) * 1584] = zz.quant_rows(zz.GPU_FMT_Q40, torch.randn((32768, 2816), device="cuda") * 0.02)
        T = zz.QTensorDev(zz.GPU_FMT_Q40, Wl, V, 2816)
        del Wl
        xq, sx, _ = zz.quant_act(torch.randn((1, 2816), device="cuda"))
        y = torch.empty(V, device="cuda")
        for _ in range(3):
            zz.check(zz.lib.zz_lm_head_dev(ctypes.byref(T.t), ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(sx.data_ptr()),
                                           None, 30.0, ctypes.c_void_p(y.data_ptr()), None), "lm_head")
    elif kind == "f32":
        # f32-activation matvecs (the gpu.h numerics): q4_0 4096 x 2816, q4a 151936 x 2048 (Maple lm_head)
        for fmt, O, I in [(zz.GPU_FMT_Q40, 4096 * 16, 2816), (zz.GPU_FMT_Q4A, 151936, 2048)]:
            src = dev(synth.q4a_tensor(5, O, I)) if fmt == zz.GPU_FMT_Q4A else \
                zz.quant_rows(zz.GPU_FMT_Q40, torch.randn((O, I), device="cuda") * 0.02)
            T = zz.QTensorDev(fmt, src, O, I)
            x = torch.randn((1, I), device="cuda")
            y = torch.empty(O, device="cuda")
            for _ in range(2):
                zz.check(zz.lib.zz_matvec_f32_dev(ctypes.byref(T.t), ctypes.c_void_p(x.data_ptr()),
                                                  ctypes.c_void_p(y.data_ptr()), 1, None), "f32")
            xq, sx, _ = zz.quant_act(x)
            zz.matvec(T, xq, sx)
    elif kind == "route":
        S = 512
        res = torch.randn((S, D), device="cuda")
        proj, sc, pes = torch.randn((E, D), device="cuda") * 0.02, torch.randn(D, device="cuda"), torch.rand(E, device="cuda")
        for _ in range(2):
            zz.route_gemma4(res, proj, sc, pes, K)
        xn = torch.randn((S, 1536), device="cuda")
        rt, bi = torch.randn((256, 1536), device="cuda") * 0.05, torch.randn(256, device="cuda") * 0.01
        for _ in range(2):
            zz.route_ling(xn, rt, bi, 8, 8, 4, 1, 2.5)
    elif kind == "ep":
        S, W = 512, 8
        xq = torch.randint(-127, 128, (S, D), dtype=torch.int8, device="cuda")
        xs = torch.rand((S, D // 32), device="cuda")
        e, w = synth.zipf_routing(5, S, E, K)[:2]
        for _ in range(2):
            rows = zz.ep_pack(xq, xs, dev(e), dev(w), W, E // W)
            zz.ep_unpack(rows, D, K)
    elif kind == "maple":
        gen = torch.Generator(device="cuda").manual_seed(4321)
        bank = tq2_bank_dev(zz, torch, synth.MAPLE_E, synth.MAPLE_D, synth.MAPLE_MI, gen)
        for S in (512, 1):
            r = synth.zipf_routing(31, S, synth.MAPLE_E, synth.MAPLE_K)
            X = torch.randn((S, synth.MAPLE_D), device="cuda")
            for _ in range(2):
                zz.moe_ffn(bank, X, dev(r[0]), dev(r[1]), zz.ZZ_ACT_SWIGLU_CLAMP, synth.MAPLE_CLAMP)
    else:
        banks, _ = make_stack(zz, torch, 2, seed=77)
        S = {"moe": 512, "prefill": 4096}.get(kind, 1)
        for l in range(2):
            r = synth.zipf_routing(88 + l, S, E, K)
            X = torch.randn((S, D), device="cuda")
            for _ in range(2):
                zz.moe_ffn(banks[l], X, dev(r[0]), dev(r[1]), zz.ZZ_ACT_GEGLU_TANH)
    torch.cuda.synchronize()
    print(f"profile case {kind} done")


def graph_timed(torch, fn, steps, warmup):
    """capture fn once into a CUDA graph, replay it; device time per replay (ms)"""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return timed(torch, g.replay, steps, warmup, torch.cuda.current_stream())


# ----------------------------------------------------------------------------- CPU
def cpu_baseline_moe(host_blobs, S, seed, spare=0):
    """The reference's own gemma4.c expert_apply over the batch union (oracle/_ref),
    all host threads but `spare` (left to the other ranks' processes, which poll while
    rank 0 samples), one layer of the same workload."""
    import oracle
    from zunzuncito_b200 import synth
    if oracle.reference_available():
        lib, kind = oracle.Reference(), "reference"
        lib.set_threads(max(1, os.cpu_count() - spare))
        cores = lib.max_threads()
    else:
        lib, kind, cores = oracle.Oracle(), "port", 1
    X = synth.gaussian(7, (S, D))
    eidx, ewt = routing(synth, 1, S, seed=99)[0]     # the timed stack's layer-0 inputs
    lib.moe_layer(0, host_blobs, X, eidx, ewt, D, MI)   # warm-up (threads, pages)
    n, t0 = 0, time.perf_counter()
    while True:   # a bounded sample of about 10 s of CPU work
        lib.moe_layer(0, host_blobs, X, eidx, ewt, D, MI)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= 10.0 or n >= 200:
            break
    return {"value": S * n / dt, "unit": "token-layers/s", "cores": cores, "kind": kind,
            "sample": f"layer 0 of the stack (S={S} tokens, 128 q4_0 experts, top-8) repeated {n} times, "
                      f"{dt:.1f} s", "seconds": dt}


def run_reference_arm(a, rank):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import oracle
    from zunzuncito_b200 import synth
    if not oracle.reference_available():
        oracle.build()
    if oracle.reference_available():
        lib, kind = oracle.Reference(), "reference"
        lib.set_threads(os.cpu_count())
        cores = lib.max_threads()
    else:
        lib, kind, cores = oracle.Oracle(), "port", 1
    S = a.tokens
    stride = 2 * (MI * (D // 32) * 18) + D * (MI // 32) * 18
    r = synth.rng(5)
    # random q4_0 bytes with sane fp16 scales (every byte pattern is a valid block)
    blobs = r.integers(0, 256, size=(E, stride), dtype=np.uint8)
    for off, rows, nb in [(0, 2 * MI, D // 32), (2 * MI * (D // 32) * 18, D, MI // 32)]:
        v = blobs[:, off:off + rows * nb * 18].reshape(E, rows * nb, 18)
        v[:, :, 0:2] = np.frombuffer(np.full(E * rows * nb, 0.002, np.float16).tobytes(), np.uint8).reshape(E, -1, 2)
    # the GPU arm's layer-0 inputs: the same X (seed 7) and the same seeded routing (seed 99)
    X = synth.gaussian(7, (S, D))
    eidx, ewt = routing(synth, 1, S, seed=99)[0]
    times = []
    for i in range(a.warmup + a.steps):
        t = time.perf_counter()
        lib.moe_layer(0, blobs, X, eidx, ewt, D, MI)
        if i >= a.warmup:
            times.append(time.perf_counter() - t)
    ms = 1e3 * float(np.mean(times))
    v = S / (ms / 1e3)
    line = {"metric": "moe_layer_tok_per_s", "value": v, "unit": "token-layers/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": stack_config(S, a.layers, routing(synth, a.layers, S, seed=99)),
            "cpu_baseline": {"value": v, "unit": "token-layers/s", "cores": cores, "kind": kind,
                             "sample": f"each step one layer of the stack (S={S} tokens, the reference's "
                                       "expert_apply over the batch union on all host threads); the throughput "
                                       "is per layer, as the GPU arm's"},
            "e2e": {"value": v, "unit": "token-layers/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.impl == "reference":
        run_reference_arm(a, rank)
        return
    import torch
    if world > 1:
        import zunzuncito_b200 as zz
        from zunzuncito_b200 import ep
        cpu_fn = None
        if not a.no_cpu:
            # the same CPU sample as the one-GPU line: layer 0 of the 128-expert stack
            cpu_fn = lambda: cpu_baseline_moe(make_stack(zz, torch, 1, seed=1234, keep_host_layer0=True)[1],
                                               a.tokens, seed=11, spare=world)
        ep.bench_main(a, rank, world, ClockSampler, cpu_baseline_fn=cpu_fn)
        return
    import zunzuncito_b200 as zz
    from zunzuncito_b200 import synth

    torch.cuda.set_device(0)
    if a.profile_case:
        profile_case(a.profile_case, zz, torch, synth)
        return
    stream = torch.cuda.current_stream()
    S, L = a.tokens, a.layers
    banks, host0 = make_stack(zz, torch, L, seed=1234, keep_host_layer0=not a.no_cpu)
    routes = routing(synth, L, S, seed=99)
    X = torch.from_numpy(synth.gaussian(7, (S, D))).cuda()
    eidx = [torch.from_numpy(r[0]).cuda() for r in routes]
    ewt = [torch.from_numpy(r[1]).cuda() for r in routes]
    out = torch.empty((S, D), device="cuda")
    for b in banks:
        b.workspace(S, K)
    distinct = [len(np.unique(r[0])) for r in routes]

    def step():
        for l in range(L):
            zz.moe_ffn(banks[l], X, eidx[l], ewt[l], zz.ZZ_ACT_GEGLU_TANH, out=out)

    step()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ms = timed(torch, step, a.steps, a.warmup, stream)
        # stage split of the same loop, live CUDA events inside the library
        zz.lib.zz_prof_enable(1)
        for _ in range(max(1, a.steps // 2)):
            step()
        zz.lib.zz_prof_enable(0)
    import ctypes
    st = (ctypes.c_float * 3)()
    calls = ctypes.c_int()
    zz.lib.zz_prof_collect(st, ctypes.byref(calls))
    stage_ms = [st[i] / max(1, calls.value) for i in range(3)]   # per layer call

    value = S * L / (ms / 1e3)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    # dominant kernel: gate/up GEMM; algorithmic bytes = distinct experts' gate+up planes
    # (2 * 704 * 88 * 18 B) + the gathered q8_0 rows (2816 + 88*4 B per pair) + hq/hs out
    gu_bytes = gateup_alg_bytes(S, float(np.mean(distinct)))
    prof_alg = float(np.mean([gateup_alg_bytes(512, len(np.unique(synth.zipf_routing(88 + l, 512, E, K)[0])))
                              for l in range(2)]))
    traffic = PROFILE_GU_TRAFFIC * gu_bytes / prof_alg
    gu_ms = stage_ms[1]
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    layer_bytes = float(np.mean(distinct)) * EXPERT_BYTES
    line = {
        "metric": "moe_layer_tok_per_s", "value": value, "unit": "token-layers/s", "n_gpus": 1,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": stack_config(S, L, routes),
        "layer_ms": ms / L,
        "layer_hbm_gbs": layer_bytes / (ms / L / 1e3) / 1e9,
        "layer_int8_tops": 2 * S * K * MACS_PER_PAIR / (ms / L / 1e3) / 1e12,
        "stage_ms_per_layer": {"quant_route": stage_ms[0], "gate_up": stage_ms[1], "down": stage_ms[2]},
        "roofline": {"kernel": "k_gemm<q4_0, BN=32, EPI_GATEUP, int8 mma.sync, preset accumulators> (gate/up GEMM + GeGLU + requant)",
                     "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "peak_source": peak_src, "traffic": traffic,
                     "traffic_source": "ncu dram bytes of the same kernel (profile case moe), scaled by algorithmic bytes",
                     "algorithmic_bytes_per_launch": gu_bytes},
        "clocks": clk.summary(),
        "gpu_launches": (a.steps) * L * 5,   # route, quantize, gather, gate/up, down per layer
    }
    # ---- e2e: the same stack through the host-buffer plugin path (pinned copies in the timed region)
    Xh = torch.from_numpy(synth.gaussian(7, (S, D))).pin_memory()
    eh = [torch.from_numpy(r[0]).pin_memory() for r in routes]
    wh = [torch.from_numpy(r[1]).pin_memory() for r in routes]
    oh = torch.empty((L, S, D), dtype=torch.float32).pin_memory()
    # Two buffer sets: layer l+1's inputs are copied in (H2D stream) and layer l-1's
    # output copied out (D2H stream) while layer l computes; every layer's copies are
    # inside the timed region, ordered by events.
    Xd = [torch.empty((S, D), device="cuda") for _ in range(2)]
    ed = [torch.empty((S, K), dtype=torch.int32, device="cuda") for _ in range(2)]
    wd = [torch.empty((S, K), device="cuda") for _ in range(2)]
    od = [torch.empty((S, D), device="cuda") for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731

    def step_e2e():
        comp = torch.cuda.current_stream()
        h2d.wait_stream(comp)
        d2h.wait_stream(comp)
        computed, copied_out = [None, None], [None, None]
        for l in range(L):
            b = l % 2
            with torch.cuda.stream(h2d):
                if computed[b] is not None:
                    h2d.wait_event(computed[b])      # layer l-2 has finished reading buffer b
                Xd[b].copy_(Xh, non_blocking=True)
                ed[b].copy_(eh[l], non_blocking=True)
                wd[b].copy_(wh[l], non_blocking=True)
                inp = ev(); inp.record(h2d)
            comp.wait_event(inp)
            if copied_out[b] is not None:
                comp.wait_event(copied_out[b])       # layer l-2's output has left buffer b
            zz.moe_ffn(banks[l], Xd[b], ed[b], wd[b], zz.ZZ_ACT_GEGLU_TANH, out=od[b])
            computed[b] = ev(); computed[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[b])
                oh[l].copy_(od[b], non_blocking=True)
                copied_out[b] = ev(); copied_out[b].record(d2h)
        comp.wait_stream(h2d)
        comp.wait_stream(d2h)

    ms_e2e = timed(torch, step_e2e, max(2, a.steps // 2), 2, stream)
    # the last layer's host copy against the device path's result of the same layer
    step()
    torch.cuda.synchronize()
    chk = float((oh[L - 1] - out.cpu()).abs().max() / out.abs().max().cpu())
    line["e2e"] = {"value": S * L / (ms_e2e / 1e3), "unit": "token-layers/s",
                   "h2d_bytes_per_step": L * (S * D * 4 + S * K * 8), "d2h_bytes_per_step": L * S * D * 4,
                   "copies": "double-buffered: H2D and D2H streams overlap the neighbouring layers' compute",
                   "max_rel_diff_vs_device_path": chk}
    if not a.no_sub:
        line["sub"] = sub_benchmarks(zz, torch, synth, stream, banks, hbm_peak)
    del banks
    if host0 is not None:
        line["cpu_baseline"] = cpu_baseline_moe(host0, S, seed=11)
    print(json.dumps(line), flush=True)


def sub_benchmarks(zz, torch, synth, stream, banks, hbm_peak):
    res = {}
    # config 1: q4_0 2816x2816 GEMV, 64 stacked distinct matrices per launch (285 MB > L2)
    G = 64
    w = torch.randn((G * 2816, 2816), device="cuda") * 0.02
    Wq = zz.quant_rows(zz.GPU_FMT_Q40, w)
    del w
    T = zz.QTensorDev(zz.GPU_FMT_Q40, Wq, G * 2816, 2816)
    del Wq
    xq, sx, _ = zz.quant_act(torch.randn((1, 2816), device="cuda"))
    y = torch.empty((1, G * 2816), device="cuda")
    # launches replayed from a CUDA graph (8 per replay), so the host's per-call cost
    # cannot leave the GPU idle between the ~50 us kernels
    def eight():
        for _ in range(8):
            zz.matvec(T, xq, sx, y=y)
    ms = graph_timed(torch, eight, 5, 3) / 8
    gbs = G * GEMV_BYTES / (ms / 1e3) / 1e9
    res["q40_gemv_2816"] = {"unit": "GB/s", "value": gbs, "frac_hbm": gbs / hbm_peak, "us_per_launch": ms * 1e3,
                            "gemvs_per_launch": G, "bytes_per_gemv": GEMV_BYTES,
                            "launch": "cuda graph, 8 launches per replay"}
    # one 2816 x 2816 GEMV per launch, cycling through the same 64 distinct matrices
    # (285 MB > L2), launches replayed from a CUDA graph
    subs = [zz.QTensor(zz.GPU_FMT_Q40, 2816, 2816, T.t.codes + g * 2816 * 1408,
                       T.t.scale + g * 2816 * 88 * 2) for g in range(G)]
    ys = torch.empty((G, 2816), device="cuda")

    def one_each():
        for g in range(G):
            zz.check(zz.lib.zz_matvec_dev(ctypes.byref(subs[g]), ctypes.c_void_p(xq.data_ptr()),
                                          ctypes.c_void_p(sx.data_ptr()), None,
                                          ctypes.c_void_p(ys[g].data_ptr()), 1,
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))

    ms1 = graph_timed(torch, one_each, 20, 3) / G
    res["q40_gemv_2816_single"] = {"unit": "GB/s", "value": GEMV_BYTES / (ms1 / 1e3) / 1e9,
                                   "us_per_gemv": ms1 * 1e3, "launch": "cuda graph, 64 distinct matrices"}
    del T, subs
    # tied lm_head of a Gemma-4 decode step: 262144 x 2816 q4_0 (415 MiB) + softcap 30
    # (gemma4.c:1270-1274), one launch per token, graph-replayed
    V = 262144
    Wl = torch.empty(V * 2816 // 32 * 18, dtype=torch.uint8, device="cuda")
    for c0 in range(0, V, 32768):
        w = torch.randn((32768, 2816), device="cuda") * 0.02
        Wl[c0 * 1584:(c0 + 32768) * 1584] = zz.quant_rows(zz.GPU_FMT_Q40, w)
        del w
    TL = zz.QTensorDev(zz.GPU_FMT_Q40, Wl, V, 2816)
    del Wl
    yl = torch.empty(V, device="cuda")

    def lm_head():
        zz.check(zz.lib.zz_lm_head_dev(ctypes.byref(TL.t), ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(sx.data_ptr()),
                                       None, 30.0, ctypes.c_void_p(yl.data_ptr()),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "lm_head")
    msl = graph_timed(torch, lm_head, 20, 3)
    lbytes = V * 1584 + 2816 + 88 * 4 + V * 4
    res["lm_head_262144x2816"] = {"unit": "GB/s", "value": lbytes / (msl / 1e3) / 1e9,
                                  "frac_hbm": lbytes / (msl / 1e3) / 1e9 / hbm_peak, "us_per_launch": msl * 1e3,
                                  "bytes": lbytes, "softcap": 30.0}
    del TL
    # config 2: decode, M=1, 8 routed experts per layer, over the 30 resident layers
    L = len(banks)
    r1 = [synth.zipf_routing(300 + l, 1, E, K)[:2] for l in range(L)]
    x1 = torch.randn((1, D), device="cuda")
    e1 = [torch.from_numpy(r[0]).cuda() for r in r1]
    w1 = [torch.from_numpy(r[1]).cuda() for r in r1]
    o1 = torch.empty((1, D), device="cuda")
    for b in banks:
        b.workspace(1, K)

    def dec():
        for l in range(L):
            zz.moe_ffn(banks[l], x1, e1[l], w1[l], zz.ZZ_ACT_GEGLU_TANH, out=o1)

    ms_eager = timed(torch, dec, 10, 3, stream)
    # the same 30 layer calls captured once in a CUDA graph and replayed: decode is
    # launch-bound otherwise (a few microseconds of weight streaming per layer)
    ms = graph_timed(torch, dec, 20, 3)
    res["decode_8_experts"] = {"unit": "us per layer", "value": ms * 1e3 / L,
                               "hbm_gbs": 8 * EXPERT_BYTES / (ms / L / 1e3) / 1e9,
                               "eager_us_per_layer": ms_eager * 1e3 / L, "launch": "cuda graph of 30 layers"}
    # S=4096 prefill layer (compute-bound regime)
    S4 = 4096
    r4 = [synth.zipf_routing(400 + l, S4, E, K)[:2] for l in range(2)]
    X4 = torch.randn((S4, D), device="cuda")
    e4 = [torch.from_numpy(r[0]).cuda() for r in r4]
    w4 = [torch.from_numpy(r[1]).cuda() for r in r4]
    o4 = torch.empty((S4, D), device="cuda")

    def pre():
        for l in range(2):
            zz.moe_ffn(banks[l], X4, e4[l], w4[l], zz.ZZ_ACT_GEGLU_TANH, out=o4)

    ms = timed(torch, pre, 5, 2, stream) / 2
    tops = 2 * S4 * K * MACS_PER_PAIR / (ms / 1e3) / 1e12
    peak = int8_peak_tops(torch)
    res["int8_peak"] = peak
    res["prefill_4096_layer"] = {"unit": "int8 TOPS", "value": tops, "frac_int8_peak": tops / peak["value"],
                                 "frac_int8_spec_4500": tops / 4500.0,
                                 "ms_per_layer": ms, "tok_per_s": S4 / (ms / 1e3)}
    # the same layers on the folded-scale tcgen05 engine (opt-in; fp16 tensor-core work is
    # 3 products per weight-activation pair, reported against the same effective ops)
    prev = os.environ.get("ZZ_MOE_KERNEL")
    os.environ["ZZ_MOE_KERNEL"] = "h3"
    try:
        ms_h3 = timed(torch, pre, 5, 2, stream) / 2
    finally:
        if prev is None:
            del os.environ["ZZ_MOE_KERNEL"]
        else:
            os.environ["ZZ_MOE_KERNEL"] = prev
    tops_h3 = 2 * S4 * K * MACS_PER_PAIR / (ms_h3 / 1e3) / 1e12
    res["prefill_4096_layer_h3"] = {"unit": "int8 TOPS", "value": tops_h3, "frac_int8_peak": tops_h3 / peak["value"],
                                    "ms_per_layer": ms_h3, "engine": "tcgen05 kind::f16, folded block scales"}
    for b in banks[:2]:
        b._ws = None
    res.update(maple_tq2(zz, torch, synth, stream, hbm_peak))
    return res


def int8_peak_tops(torch):
    """dense int8 tensor peak measured here: torch._int_mm (cuBLASLt) at 8192^3, int32
    out, best of 10 CUDA-event timings, timed in isolation (burst)"""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    bt = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = bt.t()   # column-major operand
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        torch._int_mm(a, b)
        t1.record()
        torch.cuda.synchronize()
        best = min(best, t0.elapsed_time(t1))
    del a, bt, b
    return {"unit": "TOPS", "value": 2 * n ** 3 / (best / 1e3) / 1e12, "how": "torch._int_mm 8192^3, best of 10"}


def tq2_bank_dev(zz, torch, E, D, MI, gen):
    """E Maple-shaped tq2 experts generated on the device: codes uniform in {0,1,2}
    (weights -1/0/+1, P(0) = 1/3), alpha |N(0,0.02)| + 1e-3, packed as tq2.h:46-51"""
    def tensor(O, I):
        c = torch.randint(0, 3, (E, O, I // 64, 4, 16), generator=gen, device="cuda", dtype=torch.uint8)
        b = c[:, :, :, 0] | (c[:, :, :, 1] << 2) | (c[:, :, :, 2] << 4) | (c[:, :, :, 3] << 6)
        al = torch.randn((E, O), generator=gen, device="cuda").abs() * 0.02 + 1e-3
        return torch.cat([al.view(torch.uint8).view(E, -1), b.reshape(E, -1)], dim=1)
    blobs = torch.cat([tensor(MI, D), tensor(MI, D), tensor(D, MI)], dim=1).contiguous()
    return zz.ExpertBankDev(zz.GPU_FMT_TQ2, blobs, D, MI)


def maple_tq2(zz, torch, synth, stream, hbm_peak):
    """Maple-shaped ternary MoE layer (256 tq2 experts, D 2048, inter
    512, top-8, clamped SwiGLU), decode (S=1) and S=512."""
    D, MI, E, K, CL = synth.MAPLE_D, synth.MAPLE_MI, synth.MAPLE_E, synth.MAPLE_K, synth.MAPLE_CLAMP
    per_expert = zz.expert_blob_bytes(zz.GPU_FMT_TQ2, D, MI)   # 798,720 B
    gen = torch.Generator(device="cuda").manual_seed(4321)
    banks = [tq2_bank_dev(zz, torch, E, D, MI, gen) for _ in range(4)]  # 4 x 204 MB > L2
    act = zz.ZZ_ACT_SWIGLU_CLAMP
    res = {}
    # S=512 on one bank (each layer call reads its ~200 MB of distinct experts)
    S = 512
    r = synth.zipf_routing(31, S, E, K)
    X = torch.from_numpy(synth.gaussian(32, (S, D))).cuda()
    e, w = torch.from_numpy(r[0]).cuda(), torch.from_numpy(r[1]).cuda()
    out = torch.empty((S, D), device="cuda")
    banks[0].workspace(S, K)
    ms = timed(torch, lambda: zz.moe_ffn(banks[0], X, e, w, act, CL, out=out), 10, 3, stream)
    distinct = len(np.unique(r[0]))
    res["maple_tq2_layer_s512"] = {"unit": "ms per layer", "value": ms, "tok_per_s": S / (ms / 1e3),
                                   "hbm_gbs": distinct * per_expert / (ms / 1e3) / 1e9, "distinct_experts": distinct}
    # decode: one token, 8 of 256 experts per layer, 4 layers (distinct banks) per graph replay
    rs = [synth.zipf_routing(40 + l, 1, E, K) for l in range(4)]
    X1 = torch.from_numpy(synth.gaussian(41, (1, D))).cuda()
    es = [torch.from_numpy(x[0]).cuda() for x in rs]
    ws = [torch.from_numpy(x[1]).cuda() for x in rs]
    o1 = torch.empty((1, D), device="cuda")
    for b in banks:
        b.workspace(1, K)

    def four():
        for l in range(4):
            zz.moe_ffn(banks[l], X1, es[l], ws[l], act, CL, out=o1)
    ms1 = graph_timed(torch, four, 20, 3) / 4
    res["maple_tq2_decode"] = {"unit": "us per layer", "value": ms1 * 1e3,
                               "hbm_gbs": K * per_expert / (ms1 / 1e3) / 1e9, "launch": "cuda graph of 4 layers"}
    del banks
    return res


if __name__ == "__main__":
    main()
