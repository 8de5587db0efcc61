// common.cuh -- shared device helpers for the cliffordcuda_b200 kernels:
// blade sign arithmetic, mbarrier / TMA (cp.async.bulk.tensor) wrappers and
// the library-wide error state.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/cliffordcuda_b200.h"

namespace cb {

// ------------------------------------------------------------ error state --
// Host side: thread-local message returned by cb_last_error().
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);

// Device side: the first failing kernel records a code in the library's
// device error word (bounded waits that ran out; never a trap). Kernels get
// its address as an argument; cb_device_status() reads and clears it.
int device_error_word(int **out);  // address for the current device; cached

// ------------------------------------------------------------ blade signs --
// Bit b of suffix_parity(p) is the parity of popcount(p >> (b + 1)): the
// number of generators of blade p that a generator b has to move past.
__host__ __device__ __forceinline__ uint32_t suffix_parity(uint32_t p) {
    uint32_t s = p >> 1;
    s ^= s >> 1;
    s ^= s >> 2;
    s ^= s >> 4;
    s ^= s >> 8;
    s ^= s >> 16;
    return s;
}

__host__ __device__ __forceinline__ int parity(uint32_t v) {
#ifdef __CUDA_ARCH__
    return __popc(v) & 1;
#else
    return __builtin_popcount(v) & 1;
#endif
}

// Reordering sign of e_p e_q: (-1)^#{(a, b): a > b, a in p, b in q}.
__host__ __device__ __forceinline__ int reorder_parity(uint32_t p, uint32_t q) {
    return parity(q & suffix_parity(p));
}

// Full geometric-product sign of e_p e_q under the metric given as two masks
// (generators squaring to -1 and to 0): +1, -1 or 0.
__host__ __device__ __forceinline__ int blade_sign(uint32_t p, uint32_t q, uint32_t neg,
                                                   uint32_t zero) {
    uint32_t c = p & q;
    if (c & zero) return 0;
    return (reorder_parity(p, q) ^ parity(c & neg)) ? -1 : 1;
}

// Product predicate on the blade pair (p, q) (the pair the sign is taken on).
__host__ __device__ __forceinline__ bool op_mask(int op, uint32_t p, uint32_t q) {
    switch (op) {
    case CB_OP_GP: return true;
    case CB_OP_WEDGE: return (p & q) == 0;
    case CB_OP_INNER: return ((p & ~q) == 0) || ((q & ~p) == 0);
    case CB_OP_LC: return (p & ~q) == 0;
    case CB_OP_RC: return (q & ~p) == 0;
    default: return false;
    }
}

// ------------------------------------------------------- PTX: mbarrier/TMA --
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One poll of the phase with parity `phase`. The thread may be suspended
// inside the instruction until the phase completes or about `hint_ns` pass,
// so a waiting warp takes no issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase,
                                              uint32_t hint_ns = 20000) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, with acquire at cluster scope: for barriers that threads
// of another CTA in the cluster arrive on (their prior writes become visible).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t phase,
                                                      uint32_t hint_ns = 20000) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Arrive on the barrier at the same shared offset as `bar` in CTA `rank` of
// this cluster (the own CTA included). Default (CTA-scope release)
// semantics: a cluster-scope release costs a cluster-wide memory barrier on
// every arrival. Writers of shared data that an async-proxy reader consumes
// fence the proxy (fence.proxy.async) before arriving.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *bar, uint32_t rank) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(rank)
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Full barrier over all threads of all CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: gives up once `timeout_ns` of wall time have passed without
// the phase completing, records `code` in the device error word and returns
// false (the caller then stops issuing work; nothing traps).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, int *err,
                                                  int code,
                                                  uint64_t timeout_ns = 2000000000ull,
                                                  bool cluster = false) {
    auto poll = [&] { return cluster ? mbar_try_wait_cluster(bar, phase) : mbar_try_wait(bar, phase); };
    if (poll()) return true;
    const uint64_t t0 = global_timer_ns();
    while (!poll()) {
        if (global_timer_ns() - t0 > timeout_ns) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int x,
                                             int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(smem_src)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --------------------------------------------------------- host utilities --
struct DeviceInfo {
    int sm_count = 0;
    int max_smem_optin = 0;
};
int device_info(DeviceInfo *out);  // for the current device; cached

// 2-D tensor map over `lines` rows of 32 fp32 (128 B), box 32 x box_lines,
// 128-byte swizzle. Returns CB_OK or an error status.
int make_tmap_lines(CUtensorMap *map, const void *base, uint64_t lines, uint32_t box_lines);

// 2-D fp32 tensor map over `outer` rows of `inner` floats (row pitch
// `row_bytes`), box box_inner x box_outer, 128-byte swizzle.
int make_tmap_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// internal 3xTF32 tcgen05 GEMMs (layer_gemm.cu), D = 128 or 256:
//   Y[rows][D] = A[rows][D] * B^T with B = [N][K] given as tf32 hi/lo parts;
//   partial[p][D][D] = X^T dY over row range p of `parts` ranges;
//   split_mats: M (D x D) -> [M^T hi | M^T lo | M hi | M lo]; M may alias
//   the third quarter (M hi) of `mats`.
int gemm3x_kmajor(int D, const float *A, const float *Bhi, const float *Blo, float *Y,
                  int64_t rows, cudaStream_t s);
int gemm3x_mn_parts(int64_t rows);
int gemm3x_mn(int D, const float *X, const float *dY, float *partial, int64_t rows, int parts,
              cudaStream_t s);
int reduce_partials(const float *partial, int parts, int D, float *G, cudaStream_t s);  // G is D x D
int split_mats(const float *M, float *mats, int D, cudaStream_t s);

// Cl(8,0) geometric product through the 16 x 16 real matrix representation
// (gp_mat16.cu): applicable when use_mat16 holds; mode as in cb_bilinear.
bool use_mat16(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
               const void *o);
int gp_mat16(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s);
// GP layer of Cl(8,0) through the 16 x 16 representation (gp_mat16.cu):
// gp_layer_weight writes [W | W^T] (2 x 288 floats) into mats; gp_layer_apply
// computes out = rho^-1(rho(in) wm) for wm = mats (y) or mats + 288 (dx);
// gp_layer_dw sums rho(x)^T rho(dy) over the batch into gp_layer_dw_parts(batch)
// partials of 256 floats and writes dw.
int gp_layer_weight(const float *w, float *mats, cudaStream_t s);
int gp_layer_apply(const float *wm, const float *in, float *out, int64_t batch, cudaStream_t s);
int gp_layer_dw_parts(int64_t batch);
int gp_layer_dw(const float *x, const float *dy, float *dw, float *partial, int64_t batch,
                cudaStream_t s);
constexpr int kGpLayerWFloats = 288;

// Both backward sums in one pass (grad_a and grad_b non-null and aligned).
int gp_mat16_bwd(const float *a, const float *b, const float *g, float *ga, float *gb,
                 int64_t batch, cudaStream_t s);

// Cl(9,0,1) geometric product through Cl(8,0) matrix products (pga10.cu),
// applicable when use_pga10 holds; pga10_sum (gp_mat16.cu) is one sum of it.
bool use_pga10(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
               const void *o);
int pga10(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s);
int pga10_sum(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s);

// internal bilinear dispatcher (bilinear.cu)
// direct: always the blade-by-blade kernels (never the matrix representation).
int bilinear(int op, int mode, const float *x, const float *y, float *out, int64_t batch, int n,
             uint32_t neg, uint32_t zero, cudaStream_t stream, bool direct = false);

}  // namespace cb
