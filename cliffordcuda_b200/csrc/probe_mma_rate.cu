// probe_mma_rate.cu -- measurement aid (not part of the library): the issue
// rate of tcgen05 kind::tf32 MMAs on one GPU, one CTA per SM (M = 128) and
// CTA pairs (cta_group::2, M = 256), N = 256 and 128, K-major 64-byte-swizzle
// operands resident in shared memory (no loads), fp32 accumulate in TMEM.
// It prints TFLOP/s and SM cycles per 6-MMA iteration (clock64), which give
// the tensor core's tf32 rate per clock: one 128 x 256 x 8 MMA per 128 cycles
// per SM, i.e. 4096 FLOP/clk/SM.
//
//   make -C cliffordcuda_b200/csrc probe && cliffordcuda_b200/csrc/_build/probe_mma_rate [seconds]
// With `seconds`, it also reports the rate over that long a run of
// back-to-back launches (the sustained rate under the power cap).
#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include "common.cuh"
using namespace cb;
__device__ __forceinline__ uint64_t desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(1) << 16; d |= (uint64_t)(512 >> 4) << 32; d |= (uint64_t)1 << 46; d |= (uint64_t)4 << 61;
    return d;
}
constexpr uint32_t idesc(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
template <int PAIR, int N>
__global__ void __launch_bounds__(128, 1) k(int iters, int *err, unsigned long long *cyc) {
    extern __shared__ unsigned char smraw[];
    unsigned char *sm = smraw + ((1024 - (smem_u32(smraw) & 1023)) & 1023);
    __shared__ uint64_t bar; __shared__ uint32_t slot;
    // non-zero operands: tensor-core power (hence the clock under the power
    // cap) depends on the data
    for (int i = threadIdx.x; i < 65536 / 4; i += 128)
        reinterpret_cast<float *>(sm)[i] = (float)((i * 2654435761u) >> 8) * (1.0f / 16777216.0f) - 0.5f;
    if (threadIdx.x == 0) { mbar_init(&bar, 1); fence_barrier_init(); }
    __syncthreads();
    if (PAIR) cluster_sync();
    if (threadIdx.x < 32) {
        if (PAIR) asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&slot)), "r"(256) : "memory");
        else asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&slot)), "r"(256) : "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (PAIR) cluster_sync();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = slot;
    const uint32_t a = smem_u32(sm), b = a + 32768;
    unsigned long long t0 = clock64();
    const bool issuer = threadIdx.x == 0 && (!PAIR || (blockIdx.x & 1) == 0);
    if (issuer) {
        for (int i = 0; i < iters; ++i) {
            #pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                uint64_t da = desc(a + kk * 32), db = desc(b + kk * 32);
                if (PAIR) {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(256, N)), "r"(1) : "memory");
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(256, N)), "r"(1) : "memory");
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(256, N)), "r"(1) : "memory");
                } else {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(128, N)), "r"(1) : "memory");
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(128, N)), "r"(1) : "memory");
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tm), "l"(da), "l"(db), "r"(idesc(128, N)), "r"(1) : "memory");
                }
            }
        }
        if (PAIR) asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(smem_u32(&bar)), "h"((uint16_t)3) : "memory");
        else asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(&bar)) : "memory");
    }
    if (threadIdx.x == 0) {
        mbar_wait_bounded(&bar, 0, err, 1, 4000000000ull);
        cyc[blockIdx.x] = clock64() - t0;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (PAIR) cluster_sync();
    if (threadIdx.x < 32) {
        if (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(256) : "memory");
        else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(256) : "memory");
    }
}
template <int PAIR, int N>
void run(int iters, int *err, unsigned long long *cyc) {
    auto f = k<PAIR, N>;
    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536 + 1024);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(148); cfg.blockDim = dim3(128); cfg.dynamicSmemBytes = 65536 + 1024;
    cudaLaunchAttribute at[1]; at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = PAIR ? 2 : 1; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
    cfg.attrs = at; cfg.numAttrs = 1;
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    for (int w = 0; w < 2; ++w) cudaLaunchKernelEx(&cfg, f, iters, err, cyc);
    cudaEventRecord(e0);
    cudaLaunchKernelEx(&cfg, f, iters, err, cyc);
    cudaEventRecord(e1);
    cudaError_t e = cudaEventSynchronize(e1);
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    int h = 0; cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    unsigned long long c0; cudaMemcpy(&c0, cyc, 8, cudaMemcpyDeviceToHost);
    double macs = 148.0 * 128 * N * 8 * 6.0 * iters;  // per SM: 128 rows x N x K=8, 6 MMAs per iter
    printf("pair=%d N=%d: %.3f ms  %.1f TFLOP/s tf32  err=%d cuda=%d cyc/iter=%.1f\n", PAIR, N, ms, 2 * macs / ms / 1e9, h, (int)e, (double)c0 / iters);
}
// Back-to-back launches for about `seconds` (the power cap settles the clock):
// average rate over the loop.
template <int PAIR, int N>
void sustained(double seconds, int iters, int *err, unsigned long long *cyc) {
    auto f = k<PAIR, N>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(148); cfg.blockDim = dim3(128); cfg.dynamicSmemBytes = 65536 + 1024;
    cudaLaunchAttribute at[1]; at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = PAIR ? 2 : 1; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
    cfg.attrs = at; cfg.numAttrs = 1;
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaLaunchKernelEx(&cfg, f, iters, err, cyc);
    cudaEventRecord(e0);
    cudaLaunchKernelEx(&cfg, f, iters, err, cyc);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    float ms1; cudaEventElapsedTime(&ms1, e0, e1);
    const int reps = (int)(seconds * 1e3 / ms1) + 1;
    cudaEventRecord(e0);
    for (int r = 0; r < reps; ++r) cudaLaunchKernelEx(&cfg, f, iters, err, cyc);
    cudaEventRecord(e1);
    cudaError_t e = cudaEventSynchronize(e1);
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    double macs = 148.0 * 128 * N * 8 * 6.0 * iters * reps;
    printf("sustained pair=%d N=%d: %d launches in %.1f ms  %.1f TFLOP/s tf32  cuda=%d\n", PAIR, N, reps, ms, 2 * macs / ms / 1e9, (int)e);
}
int main(int argc, char **argv) {
    const double seconds = argc > 1 ? atof(argv[1]) : 0.0;
    int *err; unsigned long long *cyc;
    cudaMalloc(&err, 4); cudaMemset(err, 0, 4); cudaMalloc(&cyc, 148 * 8);
    run<0, 256>(4000, err, cyc);
    run<1, 256>(4000, err, cyc);
    run<0, 128>(4000, err, cyc);
    run<1, 128>(4000, err, cyc);
    run<0, 256>(4000, err, cyc);
    if (seconds > 0) sustained<0, 256>(seconds, 4000, err, cyc);
    return 0;
}
