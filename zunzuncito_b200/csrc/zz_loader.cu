// zz_loader.cu -- the gemma4 container (manifest.txt, dense.bin, experts.bin, written by
// the reference's tools/convert_gemma4.py:361-422 and read by gemma4.c:260-403) loaded
// straight into structure-of-arrays HBM: a layer's expert blobs are read from
// experts.bin at their manifest offsets into pinned staging, copied to the device once
// and repacked into an expert bank; a q4_0 dense tensor (the tied embedding / lm_head,
// projections) is repacked into zz_qtensor planes. No engine-side host copy of the
// experts and no gpu_map of them is needed.
//
// Host code only. The loader allocates its own staging (pinned host and device); it is
// not a hot path.
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <string>
#include <unistd.h>
#include <vector>
#include "zz_common.cuh"

namespace zz {
size_t ref_tensor_bytes(int fmt, int O, int I);
}
using namespace zz;

struct zz_container {
    std::string dir;
    std::map<std::string, std::string> cfg;  // "cfg <key> <value...>" lines
    long long esz = 0, gate_b = 0, down_b = 0;
    struct Dense { long long off, len; int fmt, O, I; };
    std::map<std::string, Dense> dense;
    int n_layers = 0, n_experts = 0, hidden = 0, inter = 0;
    std::vector<long long> eoff;             // [layer * n_experts + expert], -1 = absent
};

// manifest.txt as gemma4.c:260-331 parses it; unknown lines are ignored, as there
static int parse_manifest(zz_container *c) {
    const std::string p = c->dir + "/manifest.txt";
    FILE *f = fopen(p.c_str(), "r");
    if (!f) return fail("zz_container_open: %s: %s", p.c_str(), strerror(errno));
    char line[1024];
    std::vector<std::string> experts;
    while (fgets(line, sizeof line, f)) {
        size_t n = strlen(line);
        while (n && (line[n - 1] == '\n' || line[n - 1] == '\r')) line[--n] = 0;
        char k[96];
        if (sscanf(line, "cfg %95s", k) == 1) {
            const char *v = line + 4 + strlen(k);
            while (*v == ' ') v++;
            c->cfg[k] = v;
            continue;
        }
        long long a, b, cc;
        if (sscanf(line, "esz %lld %lld %lld", &a, &b, &cc) == 3) {
            c->esz = a; c->gate_b = b; c->down_b = cc;
            continue;
        }
        char nm[96];
        long long off, len;
        int fmt, O, I;
        if (sscanf(line, "dense %95s %lld %lld %d %d %d", nm, &off, &len, &fmt, &O, &I) == 6) {
            c->dense[nm] = zz_container::Dense{off, len, fmt, O, I};
            continue;
        }
        int li, e;
        long long eo;
        if (sscanf(line, "expert %d %d %lld", &li, &e, &eo) == 3) {
            experts.push_back(line);
            continue;
        }
    }
    fclose(f);
    auto geti = [&](const char *key) -> int {
        auto it = c->cfg.find(key);
        return it == c->cfg.end() ? 0 : atoi(it->second.c_str());
    };
    c->n_layers = geti("n_layers");
    c->n_experts = geti("n_experts");
    c->hidden = geti("hidden");
    c->inter = geti("moe_inter");
    if (c->n_layers <= 0 || c->n_experts <= 0 || c->hidden <= 0 || c->inter <= 0)
        return fail("zz_container_open: manifest lacks n_layers / n_experts / hidden / moe_inter");
    c->eoff.assign((size_t)c->n_layers * c->n_experts, -1);
    for (const std::string &l : experts) {
        int li, e;
        long long eo;
        sscanf(l.c_str(), "expert %d %d %lld", &li, &e, &eo);
        if (li < 0 || li >= c->n_layers || e < 0 || e >= c->n_experts)
            return fail("zz_container_open: expert line out of range: %s", l.c_str());
        c->eoff[(size_t)li * c->n_experts + e] = eo;
    }
    return 1;
}

static int read_at(int fd, void *dst, size_t n, long long off, const char *what) {
    uint8_t *p = (uint8_t *)dst;
    for (size_t o = 0; o < n;) {
        ssize_t r = pread(fd, p + o, n - o, off + (long long)o);
        if (r <= 0) return fail("%s: read failed at %lld: %s", what, off + (long long)o, r ? strerror(errno) : "EOF");
        o += (size_t)r;
    }
    return 1;
}

extern "C" int zz_container_open(const char *dir, zz_container **out) {
    if (!dir || !out) return fail("zz_container_open: null argument");
    zz_container *c = new zz_container();
    c->dir = dir;
    if (!parse_manifest(c)) {
        delete c;
        return 0;
    }
    *out = c;
    return 1;
}

extern "C" void zz_container_close(zz_container *c) { delete c; }

extern "C" int zz_container_cfg(const zz_container *c, const char *key, double *val) {
    if (!c || !key || !val) return fail("zz_container_cfg: null argument");
    auto it = c->cfg.find(key);
    if (it == c->cfg.end()) return fail("zz_container_cfg: no key %s", key);
    char *end = nullptr;
    *val = strtod(it->second.c_str(), &end);
    if (end == it->second.c_str()) return fail("zz_container_cfg: %s is not numeric", key);
    return 1;
}

extern "C" int zz_container_dense_info(const zz_container *c, const char *name, int *fmt, int *O, int *I,
                                       int64_t *off, int64_t *len) {
    if (!c || !name) return fail("zz_container_dense_info: null argument");
    auto it = c->dense.find(name);
    if (it == c->dense.end()) return fail("zz_container_dense_info: no dense tensor %s", name);
    if (fmt) *fmt = it->second.fmt;
    if (O) *O = it->second.O;
    if (I) *I = it->second.I;
    if (off) *off = it->second.off;
    if (len) *len = it->second.len;
    return 1;
}

extern "C" int64_t zz_container_expert_offset(const zz_container *c, int layer, int expert) {
    if (!c || layer < 0 || layer >= c->n_layers || expert < 0 || expert >= c->n_experts) return -1;
    return c->eoff[(size_t)layer * c->n_experts + expert];
}

extern "C" size_t zz_container_bank_bytes(const zz_container *c) {
    if (!c) return 0;
    return zz_expert_bank_bytes(GPU_FMT_Q40, c->n_experts, c->hidden, c->inter);
}

extern "C" int zz_container_load_bank_dev(zz_container *c, int layer, void *dst, zz_expert_bank *bank, void *stream) {
    if (!c || !dst || !bank) return fail("zz_container_load_bank_dev: null argument");
    if (layer < 0 || layer >= c->n_layers) return fail("zz_container_load_bank_dev: layer %d out of range", layer);
    const int E = c->n_experts, D = c->hidden, MI = c->inter;
    const long long gb = (long long)ref_tensor_bytes(GPU_FMT_Q40, MI, D), db = (long long)ref_tensor_bytes(GPU_FMT_Q40, D, MI);
    if (c->gate_b != gb || c->down_b != db || c->esz != 2 * gb + db)
        return fail("zz_container_load_bank_dev: esz %lld %lld %lld is not the q4_0 [gate|up|down] of %dx%d",
                    c->esz, c->gate_b, c->down_b, D, MI);
    for (int e = 0; e < E; e++)
        if (c->eoff[(size_t)layer * E + e] < 0) return fail("zz_container_load_bank_dev: layer %d expert %d absent", layer, e);
    const std::string p = c->dir + "/experts.bin";
    const int fd = open(p.c_str(), O_RDONLY);
    if (fd < 0) return fail("zz_container_load_bank_dev: %s: %s", p.c_str(), strerror(errno));
    cudaStream_t st = (cudaStream_t)stream;
    const size_t stride = (size_t)(c->esz + 15) / 16 * 16;   // 16-byte-aligned blob stride on the device
    const int CH = 16;                                       // experts per pinned chunk
    uint8_t *dev = nullptr, *pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int ok = check_cuda(cudaMalloc(&dev, stride * E), "loader staging") &&
             check_cuda(cudaMallocHost(&pin[0], stride * CH), "loader pinned") &&
             check_cuda(cudaMallocHost(&pin[1], stride * CH), "loader pinned") &&
             check_cuda(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming), "loader event") &&
             check_cuda(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming), "loader event");
    // double-buffered: the file read of chunk k+1 overlaps the copy of chunk k
    for (int e0 = 0, k = 0; ok && e0 < E; e0 += CH, k++) {
        const int b = k & 1, n = E - e0 < CH ? E - e0 : CH;
        if (k >= 2) ok = check_cuda(cudaEventSynchronize(ev[b]), "loader sync");
        for (int i = 0; ok && i < n; i++)
            ok = read_at(fd, pin[b] + (size_t)i * stride, (size_t)c->esz, c->eoff[(size_t)layer * E + e0 + i],
                         "zz_container_load_bank_dev");
        ok = ok && check_cuda(cudaMemcpyAsync(dev + (size_t)e0 * stride, pin[b], stride * n, cudaMemcpyHostToDevice, st),
                              "loader copy") &&
             check_cuda(cudaEventRecord(ev[b], st), "loader event");
    }
    close(fd);
    ok = ok && zz_expert_bank_pack_dev(GPU_FMT_Q40, E, D, MI, dev, (int64_t)stride, dst, bank, stream) &&
         check_cuda(cudaStreamSynchronize(st), "loader pack");
    for (int i = 0; i < 2; i++) {
        if (pin[i]) cudaFreeHost(pin[i]);
        if (ev[i]) cudaEventDestroy(ev[i]);
    }
    if (dev) cudaFree(dev);
    return ok;
}

extern "C" int zz_container_load_dense_dev(zz_container *c, const char *name, void *dst, zz_qtensor *out, void *stream) {
    if (!c || !name || !dst || !out) return fail("zz_container_load_dense_dev: null argument");
    auto it = c->dense.find(name);
    if (it == c->dense.end()) return fail("zz_container_load_dense_dev: no dense tensor %s", name);
    const zz_container::Dense &d = it->second;
    if (d.fmt != 1) return fail("zz_container_load_dense_dev: %s has container format %d, not q4_0 (1)", name, d.fmt);
    if ((long long)ref_tensor_bytes(GPU_FMT_Q40, d.O, d.I) != d.len)
        return fail("zz_container_load_dense_dev: %s is %lld bytes, not q4_0 %dx%d", name, d.len, d.O, d.I);
    const std::string p = c->dir + "/dense.bin";
    const int fd = open(p.c_str(), O_RDONLY);
    if (fd < 0) return fail("zz_container_load_dense_dev: %s: %s", p.c_str(), strerror(errno));
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t *pin = nullptr, *dev = nullptr;
    int ok = check_cuda(cudaMallocHost(&pin, (size_t)d.len), "loader pinned") &&
             check_cuda(cudaMalloc(&dev, (size_t)d.len), "loader staging") &&
             read_at(fd, pin, (size_t)d.len, d.off, "zz_container_load_dense_dev") &&
             check_cuda(cudaMemcpyAsync(dev, pin, (size_t)d.len, cudaMemcpyHostToDevice, st), "loader copy") &&
             zz_repack_dev(GPU_FMT_Q40, dev, d.O, d.I, dst, out, stream) &&
             check_cuda(cudaStreamSynchronize(st), "loader repack");
    close(fd);
    if (pin) cudaFreeHost(pin);
    if (dev) cudaFree(dev);
    return ok;
}
