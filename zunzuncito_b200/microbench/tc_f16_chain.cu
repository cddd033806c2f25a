// tc_f16_chain.cu -- how fast one thread's chain of tcgen05.mma kind::f16 instructions
// (M = 128, K = 16, A and B from shared memory) runs, by accumulator pattern.
//
// The folded-scale expert engine (zz_moe_h3.cu) issues per 16-wide K step one MMA of
// N = 2 np2 columns (main | cross sums) and one of N = np2 columns into the cross half,
// so consecutive MMAs write overlapping but different TMEM column ranges. This program
// times, one CTA per SM and 4096 MMAs per CTA, the cycles per MMA (max over SMs) of:
//   same N        every MMA into the same columns (a GEMM's K loop)
//   overlap       the engine's pattern: N = 2n into [0, 2n), then N = n into [n, 2n)
//   disjoint      N = 2n into [0, 2n), then N = n into [2n, 3n)
//   W-way         W independent accumulations of N columns each, issued round robin
//   warp:         the same patterns with the whole warp running the loop and one elected
//                 lane issuing each MMA (operands in uniform registers)
//   unrolled      the engine's loop shape: per stage a probe, a fence and a commit around
//                 4 fully unrolled MMA pairs
//   A in TMEM     the same with the A operand read from TMEM ([a-tmem] form)
//   stage=4       plus, every 4 MMA pairs (one 64-weight stage), a probe of a completed
//                 barrier phase and a commit: the engine's per-stage bookkeeping
// against the arithmetic alone (M N K 2 / 8192 flops per SM cycle). Every wait is
// bounded (100 ms of %globaltimer).
//
// build: nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//            -I zunzuncito_b200/csrc -I include zunzuncito_b200/microbench/tc_f16_chain.cu -o tc_f16_chain
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>
#include "zz_common.cuh"
#include "zz_tc.cuh"
using namespace zz;

namespace {
constexpr int NMMA = 4096;
struct Case {
    const char *name;
    int n1, off1, n2, off2;  // first MMA: N, column offset; second (n2 = 0: none)
    int ways;                // > 0: round robin over `ways` chains of n1 columns each
    int warp_issue;          // 1: warp 0 runs the loop, one elected lane issues each MMA
    int stage;               // > 0 (with warp_issue): after every `stage` MMA pairs, a commit
                             // to a second barrier and a probe of a completed barrier phase
    int parts;               // which of those: 1 probe, 2 fence, 4 commit (0 = all)
};
__global__ void __launch_bounds__(128, 1) k_chain(Case c, unsigned long long *cycles, int *err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + 3 * 32768);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 1);  // bar + 2, bar + 3: stage barriers
    const int tid = threadIdx.x, warp = tid >> 5;
    // operands: zeros (the timing does not depend on the values)
    for (int i = tid; i < 3 * 32768 / 16; i += 128) reinterpret_cast<uint4 *>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::mbar_init(bar + 2, 1);
        tc::mbar_init(bar + 3, 1 << 20);  // counts the stage commits, never completes
        tc::mbar_init_fence();
        tc::mbar_arrive(bar + 2);           // phase 0 of bar + 2 completes here
    }
    tc::fence_proxy_async();
    if (warp == 0) tc::tmem_alloc(tslot, 512);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tbase = *tslot;
    if (c.warp_issue == 1 && warp == 0) {
        const uint32_t sa = tc::smem_u32(smem), sb = tc::smem_u32(smem + 32768);
        const uint64_t ad = tc::smem_desc_sw128(sa), bd = tc::smem_desc_sw128(sb);
        const uint32_t id1 = tc::idesc_f16(128, c.n1), id2 = c.n2 ? tc::idesc_f16(128, c.n2) : 0;
        const long long t0 = clock64();
        for (int i = 0; i < NMMA; i += c.n2 ? 2 : 1) {
            const int kk = (i >> 1) & 3;
            if (c.stage && (i >> 1) % c.stage == 0) {
                // the engine's per-stage bookkeeping: probe a barrier (phase 0 completed at
                // set-up) and commit the previous stage's MMAs to another barrier
                const int pm = c.parts ? c.parts : 7;
                if (pm & 1) while (!tc::mbar_test(bar + 2, 0)) {}
                if (pm & 2) tc::tc_fence_after();
                if ((pm & 4) && i) tc::mma_commit_warp(bar + 3);
            }
            tc::mma_f16_ss_warp(tbase + c.off1, ad + 2 * kk, bd + 2 * kk, id1, i != 0);
            if (c.n2) tc::mma_f16_ss_warp(tbase + c.off2, ad + 2 * kk, bd + 2 * kk, id2, 1);
        }
        tc::mma_commit_warp(bar);
        const unsigned long long w0 = tc::global_ns();
        while (!tc::mbar_try(bar, 0))
            if (tc::global_ns() - w0 > 100000000ull) { atomicExch(err, 1); break; }
        const long long t1 = clock64();
        if (tid == 0) atomicMax(cycles, (unsigned long long)(t1 - t0));
    } else if (c.warp_issue >= 2 && warp == 0) {
        // the engine's loop shape: per stage a probe, a fence and a commit, then the stage's
        // 4 MMA pairs fully unrolled with descriptors formed once per stage
        const uint32_t sa = tc::smem_u32(smem), sb = tc::smem_u32(smem + 32768);
        const uint32_t id1 = tc::idesc_f16(128, c.n1), id2 = tc::idesc_f16(128, c.n2);
        const long long t0 = clock64();
        for (int st = 0; st < NMMA / 8; st++) {
            while (!tc::mbar_test(bar + 2, 0)) {}
            tc::tc_fence_after();
            const uint64_t ad = tc::smem_desc_sw128(sa + (st & 1) * 16384), bd = tc::smem_desc_sw128(sb + (st & 1) * 16384);
            if (c.warp_issue == 3) {
                // A from TMEM (columns 256.. of the allocation, packed fp16 pairs)
                const uint32_t at = tbase + 256 + (st & 1) * 64;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    tc::mma_f16_ts_warp(tbase + c.off1, at + 8 * kk, bd + 2 * kk, id1, (st | kk) != 0);
                    tc::mma_f16_ts_warp(tbase + c.off2, at + 32 + 8 * kk, bd + 2 * kk, id2, 1);
                }
            } else {
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    tc::mma_f16_ss_warp(tbase + c.off1, ad + 2 * kk, bd + 2 * kk, id1, (st | kk) != 0);
                    tc::mma_f16_ss_warp(tbase + c.off2, ad + 2 * kk, bd + 2 * kk, id2, 1);
                }
            }
            tc::mma_commit_warp(bar + 3);
        }
        tc::mma_commit_warp(bar);
        const unsigned long long w0 = tc::global_ns();
        while (!tc::mbar_try(bar, 0))
            if (tc::global_ns() - w0 > 100000000ull) { atomicExch(err, 1); break; }
        const long long t1 = clock64();
        if (tid == 0) atomicMax(cycles, (unsigned long long)(t1 - t0));
    } else if (!c.warp_issue && tid == 0) {
        const uint32_t sa = tc::smem_u32(smem), sb = tc::smem_u32(smem + 32768);
        const uint64_t ad = tc::smem_desc_sw128(sa), bd = tc::smem_desc_sw128(sb);
        const uint32_t id1 = tc::idesc_f16(128, c.n1), id2 = c.n2 ? tc::idesc_f16(128, c.n2) : 0;
        const long long t0 = clock64();
        if (c.ways > 0) {
            for (int i = 0; i < NMMA; i += c.ways)
                for (int w = 0; w < c.ways; w++)
                    tc::mma_f16_ss(tbase + w * c.n1, ad + 2 * ((i / c.ways) & 3), bd + 2 * ((i / c.ways) & 3), id1, i != 0);
        } else
        for (int i = 0; i < NMMA; i += c.n2 ? 2 : 1) {
            const int kk = (i >> 1) & 3;
            tc::mma_f16_ss(tbase + c.off1, ad + 2 * kk, bd + 2 * kk, id1, i != 0);
            if (c.n2) tc::mma_f16_ss(tbase + c.off2, ad + 2 * kk, bd + 2 * kk, id2, 1);
        }
        tc::mma_commit(bar);
        const unsigned long long w0 = tc::global_ns();
        while (!tc::mbar_try(bar, 0))
            if (tc::global_ns() - w0 > 100000000ull) { atomicExch(err, 1); break; }
        const long long t1 = clock64();
        atomicMax(cycles, (unsigned long long)(t1 - t0));
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tbase, 512);
    }
}
}  // namespace

int main() {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const int smem = 3 * 32768 + 64 + 1024;  // operands, barriers, alignment slack
    cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    unsigned long long *cyc;
    int *err;
    cudaMalloc(&cyc, 8);
    cudaMalloc(&err, 4);
    cudaMemset(err, 0, 4);
    const Case cases[] = {
        {"same N=256", 256, 0, 0, 0},      {"same N=128", 128, 0, 0, 0},      {"same N=64", 64, 0, 0, 0},
        {"same N=32", 32, 0, 0, 0},        {"same N=16", 16, 0, 0, 0},
        {"overlap 256+128", 256, 0, 128, 128}, {"disjoint 256+128", 256, 0, 128, 256},
        {"overlap 64+32", 64, 0, 32, 32},  {"disjoint 64+32", 64, 0, 32, 64},
        {"overlap 32+16", 32, 0, 16, 16},  {"disjoint 32+16", 32, 0, 16, 32},
        {"overlap 128+64", 128, 0, 64, 64},
        {"2-way N=64", 64, 0, 0, 0, 2},    {"4-way N=64", 64, 0, 0, 0, 4},    {"8-way N=64", 64, 0, 0, 0, 8},
        {"4-way N=32", 32, 0, 0, 0, 4},    {"8-way N=32", 32, 0, 0, 0, 8},    {"4-way N=128", 128, 0, 0, 0, 4},
        {"warp: same N=64", 64, 0, 0, 0, 0, 1},          {"warp: same N=256", 256, 0, 0, 0, 0, 1},
        {"warp: overlap 64+32", 64, 0, 32, 32, 0, 1},    {"warp: overlap 128+64", 128, 0, 64, 64, 0, 1},
        {"warp: overlap 256+128", 256, 0, 128, 128, 0, 1},
        {"warp: 64+32, stage=4", 64, 0, 32, 32, 0, 1, 4},    {"warp: 128+64, stage=4", 128, 0, 64, 64, 0, 1, 4},
        {"warp: 32+16, stage=4", 32, 0, 16, 16, 0, 1, 4},
        {"  probe only", 64, 0, 32, 32, 0, 1, 4, 1}, {"  fence only", 64, 0, 32, 32, 0, 1, 4, 2},
        {"  commit only", 64, 0, 32, 32, 0, 1, 4, 4}, {"  commit, stage=8", 64, 0, 32, 32, 0, 1, 8, 4},
        {"unrolled stage 64+32", 64, 0, 32, 32, 0, 2},    {"unrolled stage 128+64", 128, 0, 64, 64, 0, 2},
        {"unrolled stage 32+16", 32, 0, 16, 16, 0, 2},
        {"A in TMEM 64+32", 64, 0, 32, 32, 0, 3},         {"A in TMEM 128+64", 128, 0, 64, 64, 0, 3},
        {"A in TMEM 32+16", 32, 0, 16, 16, 0, 3},
    };
    printf("%-20s %10s %10s %8s\n", "case", "cyc/MMA", "arith", "ratio");
    for (const Case &c : cases) {
        for (int rep = 0; rep < 2; rep++) {  // the first launch warms up
            cudaMemset(cyc, 0, 8);
            k_chain<<<sms, 128, smem>>>(c, cyc, err);
            cudaDeviceSynchronize();
        }
        unsigned long long h = 0;
        int e = 0;
        cudaMemcpy(&h, cyc, 8, cudaMemcpyDeviceToHost);
        cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost);
        const double per = (double)h / NMMA;
        const double arith = c.n2 && !c.ways ? (128.0 * (c.n1 + c.n2) * 16 * 2 / 8192) / 2 : 128.0 * c.n1 * 16 * 2 / 8192;
        printf("%-20s %10.1f %10.1f %8.2f%s\n", c.name, per, arith, per / arith, e ? "  (wait ran out)" : "");
    }
    const cudaError_t r = cudaGetLastError();
    printf("status: %s\n", cudaGetErrorString(r));
    return r != cudaSuccess;
}
