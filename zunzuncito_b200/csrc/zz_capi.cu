// zz_capi.cu -- the reference backend surface (gpu.h:61-84) on CUDA, error reporting,
// and the device-pointer matvec entry points.
//
// gpu_map copies a registered host region into HBM once (the reference wraps the same
// pages without a copy, metal.mm:366-387; a discrete GPU must copy). A matmul on a
// pointer inside a region repacks that tensor into structure-of-arrays planes the
// first time it is named and reuses the planes afterwards, so the hot path reads only
// the SoA copy. Activations and outputs cross as host f32, copied per call as the
// reference's backend does (metal.mm:445, 464).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>
#include "zz_common.cuh"

namespace zz {

static thread_local char g_err[512] = "";

int fail(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return 0;
}
int check_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 1;
    return fail("%s: %s", what, cudaGetErrorString(e));
}

int matvec_impl(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y, int S,
                cudaStream_t st);
int launch_gemv_f32(const zz_qtensor *W, const float *x, int S, float *y, cudaStream_t st);
int launch_blocksums(const zz_qtensor *W, const int8_t *xq, int32_t *out, cudaStream_t st);
size_t ref_tensor_bytes(int fmt, int O, int I);

// ---- backend state (single host thread, like metal.mm:280-296) ----
struct Region {
    const uint8_t *host;
    size_t n;
    uint8_t *dev;
};
struct PackKey {
    const uint8_t *W;
    int fmt, O, I;
    bool operator<(const PackKey &o) const {
        if (W != o.W) return W < o.W;
        if (fmt != o.fmt) return fmt < o.fmt;
        if (O != o.O) return O < o.O;
        return I < o.I;
    }
};
struct Packed {
    void *mem;
    zz_qtensor t;
};
static struct {
    int ready = 0;
    int device = -1;
    char name[320] = "none";
    cudaStream_t stream = nullptr;
    std::vector<Region> regions;
    std::map<PackKey, Packed> packed;
    void *scratch = nullptr;  // activations, quantized rows, outputs, items
    size_t scratch_bytes = 0;
    int act_quant = 0;        // gpu_matmul numerics: 0 f32 activations, 1 q8_0 activations
} G;

static const size_t kMaxRegions = 8192;  // the reference's map capacity (metal.mm:291)

static int ensure_scratch(size_t n) {
    if (n <= G.scratch_bytes) return 1;
    if (G.scratch) cudaFree(G.scratch);
    G.scratch = nullptr;
    G.scratch_bytes = 0;
    if (!check_cuda(cudaMalloc(&G.scratch, n), "scratch alloc")) return 0;
    G.scratch_bytes = n;
    return 1;
}

static const Region *find_region(const uint8_t *p, size_t len) {
    for (const Region &r : G.regions)
        if (p >= r.host && p + len <= r.host + r.n) return &r;
    return nullptr;
}

}  // namespace zz

using namespace zz;

static inline size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

extern "C" const char *gpu_last_error(void) { return g_err; }

extern "C" int gpu_init(void) {
    g_err[0] = 0;
    if (G.ready) return 1;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail("gpu_init: no CUDA device");
    int dev = 0;
    if (!check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return 0;
    cudaDeviceProp prop;
    if (!check_cuda(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties")) return 0;
    if (prop.major != 10) return fail("gpu_init: device %s is sm_%d%d, kernels are built for sm_100a", prop.name, prop.major, prop.minor);
    if (!check_cuda(cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking), "stream create")) return 0;
    G.device = dev;
    snprintf(G.name, sizeof G.name, "%s (CUDA sm_%d%d)", prop.name, prop.major, prop.minor);
    G.ready = 1;
    return 1;
}

extern "C" void gpu_shutdown(void) {
    if (!G.ready) return;
    cudaStreamSynchronize(G.stream);
    for (auto &kv : G.packed) cudaFree(kv.second.mem);
    G.packed.clear();
    for (Region &r : G.regions) cudaFree(r.dev);
    G.regions.clear();
    if (G.scratch) cudaFree(G.scratch);
    G.scratch = nullptr;
    G.scratch_bytes = 0;
    cudaStreamDestroy(G.stream);
    G.stream = nullptr;
    G.ready = 0;
    snprintf(G.name, sizeof G.name, "none");
}

extern "C" int gpu_ready(void) { return G.ready; }
extern "C" const char *gpu_name(void) { return G.name; }

extern "C" int gpu_unmap(const void *p);

extern "C" int gpu_map(const void *p, size_t n) {
    if (!G.ready) return fail("gpu_map: gpu_init has not succeeded");
    if (!p || n == 0) return fail("gpu_map: empty region");
    if (G.regions.size() >= kMaxRegions) return fail("gpu_map: more than %zu regions", kMaxRegions);
    const uint8_t *h = (const uint8_t *)p;
    // A region that overlaps mapped ones means the caller reused that host memory (the
    // reference backend maps pages without copying, so it always sees the current
    // bytes): the older copies are dropped with their packed planes.
    for (size_t i = G.regions.size(); i-- > 0;) {
        const Region &o = G.regions[i];
        if (h < o.host + o.n && o.host < h + n) gpu_unmap(o.host);
    }
    Region r{h, n, nullptr};
    if (!check_cuda(cudaMalloc(&r.dev, n), "gpu_map alloc")) return 0;
    if (!check_cuda(cudaMemcpyAsync(r.dev, h, n, cudaMemcpyHostToDevice, G.stream), "gpu_map copy") ||
        !check_cuda(cudaStreamSynchronize(G.stream), "gpu_map sync")) {
        cudaFree(r.dev);
        return 0;
    }
    G.regions.push_back(r);
    return 1;
}

extern "C" int gpu_unmap(const void *p) {
    if (!G.ready) return fail("gpu_unmap: not initialised");
    for (size_t i = 0; i < G.regions.size(); i++) {
        Region &r = G.regions[i];
        if (r.host != p) continue;
        cudaStreamSynchronize(G.stream);
        for (auto it = G.packed.begin(); it != G.packed.end();) {
            if (it->first.W >= r.host && it->first.W < r.host + r.n) {
                cudaFree(it->second.mem);
                it = G.packed.erase(it);
            } else {
                ++it;
            }
        }
        cudaFree(r.dev);
        G.regions.erase(G.regions.begin() + i);
        return 1;
    }
    return fail("gpu_unmap: %p is not the start of a mapped region", p);
}

// the SoA planes of the tensor at W (inside a mapped region), packed on first use
static const zz_qtensor *packed_tensor(const char *who, int fmt, const uint8_t *W, int O, int I) {
    if (!G.ready) { fail("%s: gpu_init has not succeeded", who); return nullptr; }
    if (fmt != GPU_FMT_Q40 && fmt != GPU_FMT_Q80 && fmt != GPU_FMT_TQ2 && fmt != GPU_FMT_Q4A) {
        fail("%s: unknown fmt %d", who, fmt);
        return nullptr;
    }
    const int grp = fmt == GPU_FMT_TQ2 || fmt == GPU_FMT_Q4A ? 64 : 32;
    if (O <= 0 || I <= 0 || I % grp) { fail("%s: bad shape O=%d I=%d", who, O, I); return nullptr; }
    if (!W) { fail("%s: null W", who); return nullptr; }
    const size_t tb = ref_tensor_bytes(fmt, O, I);
    const Region *reg = find_region(W, tb);
    if (!reg) { fail("%s: W is not inside a gpu_map'd region", who); return nullptr; }
    PackKey key{W, fmt, O, I};
    auto it = G.packed.find(key);
    if (it == G.packed.end()) {
        Packed pk{};
        size_t nb = zz_qtensor_bytes(fmt, O, I);
        if (!check_cuda(cudaMalloc(&pk.mem, nb), "plane alloc")) return nullptr;
        if (!zz_repack_dev(fmt, reg->dev + (W - reg->host), O, I, pk.mem, &pk.t, G.stream)) {
            cudaFree(pk.mem);
            return nullptr;
        }
        it = G.packed.emplace(key, pk).first;
    }
    return &it->second.t;
}

extern "C" int zz_gpu_set_act_quant(int on) {
    G.act_quant = on != 0;
    return 1;
}

extern "C" int gpu_matmul(int fmt, float *y, const uint8_t *W, const float *x, int O, int I, int S) {
    g_err[0] = 0;
    if (S <= 0) return fail("gpu_matmul: bad S=%d", S);
    if (!y || !x) return fail("gpu_matmul: null pointer");
    const zz_qtensor *T = packed_tensor("gpu_matmul", fmt, W, O, I);
    if (!T) return 0;
    // scratch: x f32 | xq | sx | sxtot | y
    const size_t bx = al256((size_t)S * I * 4), bq = al256((size_t)S * I), bs = al256((size_t)S * (I / 32) * 4);
    const size_t bt = al256((size_t)S * 4), by = al256((size_t)S * O * 4);
    if (!ensure_scratch(bx + bq + bs + bt + by)) return 0;
    uint8_t *s = (uint8_t *)G.scratch;
    float *dx = (float *)s;
    int8_t *dq = (int8_t *)(s + bx);
    float *dsx = (float *)(s + bx + bq);
    float *dtot = (float *)(s + bx + bq + bs);
    float *dy = (float *)(s + bx + bq + bs + bt);
    if (!check_cuda(cudaMemcpyAsync(dx, x, (size_t)S * I * 4, cudaMemcpyHostToDevice, G.stream), "x copy")) return 0;
    if (!G.act_quant) {
        // the reference backend's numerics: f32 activations (gpu.h:25-30)
        if (!launch_gemv_f32(T, dx, S, dy, G.stream)) return 0;
    } else {
        if (!zz_quant_act_dev(dx, S, I, dq, dsx, fmt == GPU_FMT_TQ2 ? dtot : nullptr, G.stream)) return 0;
        if (!matvec_impl(T, dq, dsx, dtot, dy, S, G.stream)) return 0;
    }
    if (!check_cuda(cudaMemcpyAsync(y, dy, (size_t)S * O * 4, cudaMemcpyDeviceToHost, G.stream), "y copy")) return 0;
    return check_cuda(cudaStreamSynchronize(G.stream), "gpu_matmul");
}

// q8_0-activation matvec on host buffers: the kernel-level signatures of q40.h / tq2.h
static int host_matvec_q8(const char *who, int fmt, float *y, const uint8_t *W, const int8_t *xq, const float *sx,
                          float sxtot, int O, int I) {
    g_err[0] = 0;
    if (!y || !xq || !sx) return fail("%s: null pointer", who);
    const zz_qtensor *T = packed_tensor(who, fmt, W, O, I);
    if (!T) return 0;
    const size_t bq = al256((size_t)I), bs = al256((size_t)(I / 32) * 4), bt = 256, by = al256((size_t)O * 4);
    if (!ensure_scratch(bq + bs + bt + by)) return 0;
    uint8_t *s = (uint8_t *)G.scratch;
    int8_t *dq = (int8_t *)s;
    float *dsx = (float *)(s + bq), *dtot = (float *)(s + bq + bs), *dy = (float *)(s + bq + bs + bt);
    if (!check_cuda(cudaMemcpyAsync(dq, xq, (size_t)I, cudaMemcpyHostToDevice, G.stream), "xq copy") ||
        !check_cuda(cudaMemcpyAsync(dsx, sx, (size_t)(I / 32) * 4, cudaMemcpyHostToDevice, G.stream), "sx copy"))
        return 0;
    if (fmt == GPU_FMT_TQ2 &&
        !check_cuda(cudaMemcpyAsync(dtot, &sxtot, 4, cudaMemcpyHostToDevice, G.stream), "sxtot copy"))
        return 0;
    if (!matvec_impl(T, dq, dsx, dtot, dy, 1, G.stream)) return 0;
    if (!check_cuda(cudaMemcpyAsync(y, dy, (size_t)O * 4, cudaMemcpyDeviceToHost, G.stream), "y copy")) return 0;
    return check_cuda(cudaStreamSynchronize(G.stream), who);
}

extern "C" int gpu_q40_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    return host_matvec_q8("gpu_q40_matvec", GPU_FMT_Q40, y, W, xq, sx, 0.f, O, I);
}
extern "C" int gpu_q80_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    return host_matvec_q8("gpu_q80_matvec", GPU_FMT_Q80, y, W, xq, sx, 0.f, O, I);
}
extern "C" int gpu_tq2_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, float sxtot, int O,
                              int I) {
    return host_matvec_q8("gpu_tq2_matvec", GPU_FMT_TQ2, y, W, xq, sx, sxtot, O, I);
}
extern "C" int gpu_q4a_matvec(float *y, const uint8_t *W, const int8_t *xq, const float *sx, int O, int I) {
    return host_matvec_q8("gpu_q4a_matvec", GPU_FMT_Q4A, y, W, xq, sx, 0.f, O, I);
}

extern "C" int gpu_q40_matmul(float *y, const uint8_t *W, const float *x, int O, int I, int S) {
    return gpu_matmul(GPU_FMT_Q40, y, W, x, O, I, S);
}

// ---- device-pointer entry points ----

static bool qt_ok(const zz_qtensor *W) {
    if (!W || !W->codes || !W->scale || W->O <= 0) return false;
    if (W->fmt == GPU_FMT_Q40 || W->fmt == GPU_FMT_Q80) return W->I > 0 && W->I % 32 == 0;
    if (W->fmt == GPU_FMT_TQ2 || W->fmt == GPU_FMT_Q4A) return W->I > 0 && W->I % 64 == 0;
    return false;
}

extern "C" int zz_matvec_f32_dev(const zz_qtensor *W, const float *x, float *y, int S, void *stream) {
    if (!qt_ok(W)) return fail("zz_matvec_f32_dev: invalid tensor");
    if (S < 0) return fail("zz_matvec_f32_dev: S < 0");
    if (S == 0) return 1;
    if (!x || !y) return fail("zz_matvec_f32_dev: null pointer");
    return launch_gemv_f32(W, x, S, y, (cudaStream_t)stream);
}

extern "C" int zz_matvec_dev(const zz_qtensor *W, const int8_t *xq, const float *sx, const float *sxtot, float *y,
                             int S, void *stream) {
    if (!qt_ok(W)) return fail("zz_matvec_dev: invalid tensor");
    if (S < 0) return fail("zz_matvec_dev: S < 0");
    if (S == 0) return 1;
    if (!xq || !sx || !y || (W->fmt == GPU_FMT_TQ2 && !sxtot)) return fail("zz_matvec_dev: null pointer");
    return matvec_impl(W, xq, sx, sxtot, y, S, (cudaStream_t)stream);
}

extern "C" int zz_blocksums_dev(const zz_qtensor *W, const int8_t *xq, int32_t *out, void *stream) {
    if (!qt_ok(W) || !xq || !out) return fail("zz_blocksums_dev: invalid arguments");
    return launch_blocksums(W, xq, out, (cudaStream_t)stream);
}
