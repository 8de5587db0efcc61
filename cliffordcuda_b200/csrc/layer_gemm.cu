// layer_gemm.cu -- shared-weight product layers on the 5th-generation tensor
// cores (tcgen05, TMEM accumulators, TMA operands), fp32 accuracy by 3xTF32.
//
// A product layer computes y = op(x, w) with one weight row w for the whole
// batch (reference layers.py:43-47, which materialised w.expand_as(x) and ran
// the batch-by-batch kernel). Because op is bilinear, y = x M(w) with
//     M(w)[i][:] = op(e_i, w)            (D x D, D = 2^n)
// and the backward pass is
//     dX = dY M^T,   G = X^T dY,   dw[k] = sum_i grad_b(e_i, G[i][:])[k]
// where grad_b is the product's own second-operand backward sum. M and the
// fold are built with the batch-by-batch bilinear kernel on identity rows, so
// every product (the regressive one included) uses this path unchanged.
//
// GEMMs (D = 128 or 256):
//   * gemm_kmajor_kernel: Y[rows][D] = A[rows][D] B^T with B given as [N][K]
//     (Y = X M uses B = M^T, dX = dY M^T uses B = M). Persistent CTA pairs
//     (cluster of 2, tcgen05 cta_group::2, M = 256): each CTA of a pair holds
//     128 rows of the 256-row tile and half of B's N rows, so B streams from
//     L2 once per 256 rows. K in 16-float chunks (64-byte swizzle rows),
//     six-stage TMA pipeline (eight at D = 128), two TMEM accumulators so the
//     epilogue of one tile overlaps the MMAs of the next.
//   * gemm_mn_kernel: G[D][D] = X^T dY with K = rows, split over CTAs (CTA
//     pairs at D = 256, gemm_mn_pair_kernel); both
//     operands are MN-major in shared memory (128-byte swizzle on 32-byte
//     atoms, the layout the tf32 MMA requires for MN-major operands); each
//     CTA writes a D x D partial.
// Warp roles: warp 0 issues TMA loads, warp 1 allocates TMEM and issues the
// MMAs (one lane; in the K-major kernel only in the even CTA of the pair),
// warps 2-3 split each landed A tile (both tiles in the MN kernel) into tf32
// hi and lo parts in place, warps 4-7 drain TMEM (tcgen05.ld); the K-major
// kernel stages 32x32 chunks of Y in 128B-swizzled shared buffers and
// TMA-stores them. The CTA-pair MN kernel has six converter warps (2-7) and
// its epilogue in warps 8-11. The MN kernels restart their TMEM accumulation
// every 256 rows and add the segments into their partial in fp32.
//
// 3xTF32: every operand v is split as hi = v with the low 13 mantissa bits
// cleared (exactly representable in tf32) and lo = v - hi (exact in fp32);
// each k-step issues hi*hi + hi*lo + lo*hi into one fp32 accumulator, which
// leaves an error near 2^-21 |a||b| per product.
//
// All waits are bounded (mbar_wait_bounded): on expiry the kernel records a
// code in the device error word, stops issuing work, and still frees TMEM.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "tcgen05.cuh"

namespace cb {
namespace {

constexpr int kThreads = 256;
constexpr int BM = 128;  // MMA M
constexpr int BK = 16;   // K chunk of the K-major kernel (64 bytes of fp32)
constexpr int BKR = 16;  // K chunk (rows) of the MN-major kernel

using namespace tc;

// Split fp32 values in place into tf32 hi (low 13 mantissa bits cleared) and
// lo = v - hi.
__device__ __forceinline__ void split_tf32(float4 *hi, float4 *lo, int count, int t, int nt) {
    for (int e = t; e < count; e += nt) {
        float4 v = hi[e];
        float4 h;
        h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
        h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
        h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
        h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
        hi[e] = h;
        lo[e] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    }
}

// ------------------------------------------------- K-major GEMM (Y = A B^T) --
// Runs on CTA pairs (clusters of 2, tcgen05 cta_group::2). A pair owns
// 256-row tiles: CTA r loads rows 128r..128r+127 of the tile and rows
// (D/2)r..(D/2)r+D/2-1 of B (the N rows of B^T), so B streams from L2 once per
// 256 output rows and each SM's tensor core reads only half of B from its own
// shared memory. The even CTA issues M = 256 MMAs that read both CTAs' tiles
// and write each CTA's 128 accumulator rows into that CTA's TMEM.
// Barriers: full (local TMA bytes), conv (in the even CTA: one arrival per
// converter warp of both CTAs), empty and accfull (in both CTAs, signalled by
// a multicast tcgen05.commit), accempty (in the even CTA: one arrival per
// epilogue warp of both CTAs).
template <int D>
struct KMajorSmem {
    static constexpr int A_BYTES = BM * BK * 4;                // 8 KB (128 rows)
    static constexpr int B_BYTES = (D / 2) * BK * 4;           // 8 KB at D = 256
    static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;    // hi + lo of both
    static constexpr int NSTAGE = D == 256 ? 6 : 8;
    // epilogue staging: 4 warps x 2 buffers of 32 rows x 32 floats (128B swizzle)
    static constexpr int OUT_BUF = 32 * 32 * 4;
    static constexpr int OUT_BYTES = 4 * 2 * OUT_BUF;
    static constexpr int BYTES = 1024 + NSTAGE * STAGE + OUT_BYTES + 256;
    static constexpr int TMEM_COLS = (2 * D <= 256) ? 256 : 512;
};

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_kmajor_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mBhi,
                       const __grid_constant__ CUtensorMap mBlo, const __grid_constant__ CUtensorMap mY,
                       int num_tiles, int *err) {
    using S = KMajorSmem<D>;
    constexpr int NK = D / BK;
    constexpr int NS = S::NSTAGE;
    extern __shared__ unsigned char smem_raw[];
    // 1 KB-aligned start, derived by pointer arithmetic on the shared array so
    // the compiler keeps the shared address space (32-bit LDS/STS addressing).
    // Both CTAs of a pair get the same layout, which the pair MMA relies on.
    unsigned char *const base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char *stage0 = base;
    unsigned char *outbuf = stage0 + NS * S::STAGE;
    uint64_t *bars = reinterpret_cast<uint64_t *>(outbuf + S::OUT_BYTES);
    uint64_t *full = bars, *conv = bars + NS, *empty = bars + 2 * NS, *accfull = bars + 3 * NS,
             *accempty = bars + 3 * NS + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * NS + 4);
    auto Ahi = [&](int s) { return stage0 + s * S::STAGE; };
    auto Alo = [&](int s) { return stage0 + s * S::STAGE + S::A_BYTES; };
    auto Bhi = [&](int s) { return stage0 + s * S::STAGE + 2 * S::A_BYTES; };
    auto Blo = [&](int s) { return stage0 + s * S::STAGE + 2 * S::A_BYTES + S::B_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 4);  // converter warps of both CTAs
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 8);  // epilogue warps of both CTAs
        }
        fence_barrier_init();
        prefetch_tensormap(&mA);
        prefetch_tensormap(&mBhi);
        prefetch_tensormap(&mBlo);
        prefetch_tensormap(&mY);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM of both allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int my_tiles = (num_tiles - pair + npairs - 1) / npairs;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                const int tile = pair + lt * npairs;
                for (int kc = 0; kc < NK && ok; ++kc, ++it) {
                    const int s = it % NS;
                    if (!(ok = mbar_wait_bounded(&empty[s], ((it / NS) + 1) & 1, err, 0x201))) break;
                    mbar_arrive_expect_tx(&full[s], S::A_BYTES + 2 * S::B_BYTES);
                    tma_load_2d(Ahi(s), &mA, kc * BK, tile * (2 * BM) + (int)rank * BM, &full[s]);
                    tma_load_2d(Bhi(s), &mBhi, kc * BK, (int)rank * (D / 2), &full[s]);
                    tma_load_2d(Blo(s), &mBlo, kc * BK, (int)rank * (D / 2), &full[s]);
                }
            }
            // The last commits arrive on this CTA's empty barriers from the
            // even CTA; take them before the CTA may exit.
            for (int j = it - NS < 0 ? 0 : it - NS; j < it && ok; ++j)
                ok = mbar_wait_bounded(&empty[j % NS], (j / NS) & 1, err, 0x206);
        }
    } else if (warp == 1) {
        if (leader) {
            constexpr uint32_t idesc = idesc_tf32(2 * BM, D, false, false);
            int it = 0;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                const int b = lt & 1;
                if (lane == 0)
                    ok = mbar_wait_bounded(&accempty[b], ((lt >> 1) + 1) & 1, err, 0x202,
                                           2000000000ull, true);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                const uint32_t dcol = tmem + b * D;
                for (int kc = 0; kc < NK && ok; ++kc, ++it) {
                    const int s = it % NS;
                    if (lane == 0)
                        ok = mbar_wait_bounded(&conv[s], (it / NS) & 1, err, 0x203, 2000000000ull, true);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t ah = smem_u32(Ahi(s)), al = smem_u32(Alo(s));
                        const uint32_t bh = smem_u32(Bhi(s)), bl = smem_u32(Blo(s));
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            const uint32_t off = kk * 32;  // 8 fp32 along K within a 64-byte row
                            const uint64_t dah = kmajor_desc(ah + off);
                            const uint64_t dal = kmajor_desc(al + off);
                            const uint64_t dbh = kmajor_desc(bh + off);
                            const uint64_t dbl = kmajor_desc(bl + off);
                            mma_tf32_pair(dcol, dah, dbh, idesc, (kc | kk) ? 1u : 0u);
                            mma_tf32_pair(dcol, dah, dbl, idesc, 1u);
                            mma_tf32_pair(dcol, dal, dbh, idesc, 1u);
                        }
                        mma_commit_pair(&empty[s]);
                        if (kc == NK - 1) mma_commit_pair(&accfull[b]);
                    }
                    __syncwarp();
                }
            }
        }
    } else if (warp < 4) {
        const int t = threadIdx.x - 64;
        int it = 0;
        for (int lt = 0; lt < my_tiles && ok; ++lt) {
            for (int kc = 0; kc < NK && ok; ++kc, ++it) {
                const int s = it % NS;
                if (!(ok = mbar_wait_bounded(&full[s], (it / NS) & 1, err, 0x204))) break;
                split_tf32(reinterpret_cast<float4 *>(Ahi(s)), reinterpret_cast<float4 *>(Alo(s)),
                           S::A_BYTES / 16, t, 64);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(&conv[s], 0);
            }
        }
    } else {
        // Each warp drains its 32 TMEM lanes (rows) in 32-column chunks into a
        // 128B-swizzled 32x32 staging buffer (lane = row; the swizzle spreads
        // the 8 float4 of a row over all banks) and one lane TMA-stores it.
        // The tensor map clips rows past the end of the batch.
        const int q = warp & 3;  // TMEM lane quarter of this warp
        unsigned char *mybuf = outbuf + q * 2 * S::OUT_BUF;
        int chunk = 0;
        for (int lt = 0; lt < my_tiles && ok; ++lt) {
            const int tile = pair + lt * npairs;
            const int b = lt & 1;
            if (!(ok = mbar_wait_bounded(&accfull[b], (lt >> 1) & 1, err, 0x205))) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * D;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c, ++chunk) {
                float v[32];
                tmem_ld32(taddr + c * 32, v);
                if (c == D / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(&accempty[b], 0);
                }
                unsigned char *buf = mybuf + (chunk & 1) * S::OUT_BUF;
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
                float4 *rowp = reinterpret_cast<float4 *>(buf + lane * 128);
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    rowp[u ^ (lane & 7)] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&mY, buf, c * 32, tile * (2 * BM) + (int)rank * BM + q * 32);
                    bulk_commit();
                }
            }
        }
        if (lane == 0) bulk_wait_all();
    }
    tc_fence_before();
    cluster_sync();  // no MMA of the pair still reads this CTA's tiles or TMEM
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, S::TMEM_COLS);
}

// ------------------------------------------ MN-major GEMM (G = X^T dY, split-K) --
// Shared tile of one operand chunk: D/32 boxes of 32 floats (MN) x BKR rows
// (K), box g (MN elements 32g..32g+31) at g * BKR * 128 bytes.
constexpr int MN_BOX_BYTES = BKR * 128;  // 2 KB
constexpr int MN_NSTAGE = 3;
template <int D>
struct MNSmem {
    static constexpr int OP_BYTES = D * BKR * 4;    // 16 KB at D = 256
    static constexpr int STAGE = 4 * OP_BYTES;      // X hi, X lo, dY hi, dY lo
    static constexpr int BYTES = 1024 + MN_NSTAGE * STAGE + 256;
    static constexpr int HALVES = D / BM;           // M = D split into 128-row MMAs
    static constexpr int ACC_COLS = HALVES * D;     // one D x D accumulator
    static constexpr int NACC = (2 * ACC_COLS <= 512) ? 2 : 1;
    static constexpr int TMEM_COLS = (NACC * ACC_COLS < 32) ? 32 : NACC * ACC_COLS;
};

// Rows of K accumulated in one TMEM accumulator before the epilogue adds it
// into the CTA's partial in global memory. The tensor core rounds its fp32
// accumulator at every MMA (three per 8 rows with 3xTF32), so a long K range
// in one accumulator loses accuracy with the square root of its length or
// faster; short segments summed in fp32 by the epilogue, then across CTAs in
// double, keep G at fp32 accuracy for millions of rows. Two accumulators
// alternate so the epilogue of one segment overlaps the MMAs of the next.
constexpr int kSegChunks = 16;  // 16 chunks of BKR = 16 rows: 256 rows per segment

// Storage order of a D x D partial of G: for each block of 128 rows, column
// groups of four, then the 128 rows, then the four columns:
//     off(row, col) = (row / 128) * 128 * D + ((col / 4) * 128 + row % 128) * 4 + col % 4
// so that the 32 lanes of an epilogue warp (32 consecutive rows, the TMEM
// lanes) touch 512 contiguous bytes with each float4 access.
__host__ __device__ __forceinline__ size_t partial_off(int D, int row, int col) {
    return (size_t)(row >> 7) * 128 * D + ((size_t)(col >> 2) * 128 + (row & 127)) * 4 + (col & 3);
}

// Epilogue of one segment for the 32 TMEM lanes of this warp: add columns
// [0, D) of accumulator row `row` (TMEM address taddr) into the partial, or
// store them for the first segment.
__device__ __forceinline__ void drain_segment(uint32_t taddr, float *part, int D, int row,
                                              bool first) {
    float4 *base = reinterpret_cast<float4 *>(part + partial_off(D, row, 0));
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        float4 *dst = base + (size_t)c * 8 * 128;  // column group 8c, this row
        float4 old[8];
        if (!first) {
#pragma unroll
            for (int u = 0; u < 8; ++u) old[u] = dst[u * 128];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            float4 a = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
            if (!first) {
                a.x += old[u].x;
                a.y += old[u].y;
                a.z += old[u].z;
                a.w += old[u].w;
            }
            dst[u * 128] = a;
        }
    }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_mn_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mG,
                   float *__restrict__ partial, int64_t rows, int64_t rows_per_cta, int *err) {
    using S = MNSmem<D>;
    constexpr int MN_OP_BYTES = S::OP_BYTES;
    constexpr int MN_STAGE = S::STAGE;
    extern __shared__ unsigned char smem_raw[];
    // 1 KB-aligned start, derived by pointer arithmetic on the shared array so
    // the compiler keeps the shared address space (32-bit LDS/STS addressing).
    unsigned char *const base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char *stage0 = base;
    uint64_t *bars = reinterpret_cast<uint64_t *>(stage0 + MN_NSTAGE * MN_STAGE);
    uint64_t *full = bars, *conv = bars + MN_NSTAGE, *empty = bars + 2 * MN_NSTAGE,
             *accfull = bars + 3 * MN_NSTAGE, *accempty = bars + 3 * MN_NSTAGE + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * MN_NSTAGE + 4);
    auto op = [&](int s, int which) { return stage0 + s * MN_STAGE + which * MN_OP_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    const int64_t r1 = std::min<int64_t>(rows, r0 + rows_per_cta);
    const int nchunks = r1 > r0 ? (int)((r1 - r0 + BKR - 1) / BKR) : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < MN_NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 64);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&accfull[a], 1);
            mbar_init(&accempty[a], 4);  // the four epilogue warps
        }
        fence_barrier_init();
        prefetch_tensormap(&mX);
        prefetch_tensormap(&mG);
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            for (int c = 0; c < nchunks && ok; ++c) {
                const int s = c % MN_NSTAGE;
                if (!(ok = mbar_wait_bounded(&empty[s], ((c / MN_NSTAGE) + 1) & 1, err, 0x211)))
                    break;
                mbar_arrive_expect_tx(&full[s], 2 * MN_OP_BYTES);
                const int row = (int)(r0 + (int64_t)c * BKR);
                for (int g = 0; g < D / 32; ++g) {
                    tma_load_2d(op(s, 0) + g * MN_BOX_BYTES, &mX, g * 32, row, &full[s]);
                    tma_load_2d(op(s, 2) + g * MN_BOX_BYTES, &mG, g * 32, row, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        constexpr uint32_t idesc = idesc_tf32(BM, D, true, true);
        for (int c = 0; c < nchunks && ok; ++c) {
            const int s = c % MN_NSTAGE;
            const int seg = c / kSegChunks, a = seg % S::NACC;
            const bool seg_first = (c % kSegChunks) == 0;
            const bool seg_last = (c % kSegChunks) == kSegChunks - 1 || c == nchunks - 1;
            // accumulator a is free once the epilogue drained its previous segment
            if (lane == 0 && seg_first && seg >= S::NACC)
                ok = mbar_wait_bounded(&accempty[a], (seg / S::NACC - 1) & 1, err, 0x215);
            if (lane == 0 && ok) ok = mbar_wait_bounded(&conv[s], (c / MN_NSTAGE) & 1, err, 0x212);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t xh = smem_u32(op(s, 0)), xl = smem_u32(op(s, 1));
                const uint32_t gh = smem_u32(op(s, 2)), gl = smem_u32(op(s, 3));
#pragma unroll
                for (int kk = 0; kk < BKR / 8; ++kk) {
                    const uint32_t koff = kk * 1024;  // next 8 rows of K
                    const uint64_t dgh = mnmajor_desc(gh + koff, MN_BOX_BYTES);
                    const uint64_t dgl = mnmajor_desc(gl + koff, MN_BOX_BYTES);
#pragma unroll
                    for (int h = 0; h < S::HALVES; ++h) {  // i in [128h, 128h + 128)
                        const uint32_t moff = h * 4 * MN_BOX_BYTES + koff;
                        const uint64_t dxh = mnmajor_desc(xh + moff, MN_BOX_BYTES);
                        const uint64_t dxl = mnmajor_desc(xl + moff, MN_BOX_BYTES);
                        const uint32_t dcol = tmem + a * S::ACC_COLS + h * D;
                        mma_tf32(dcol, dxh, dgh, idesc, (seg_first && kk == 0) ? 0u : 1u);
                        mma_tf32(dcol, dxh, dgl, idesc, 1u);
                        mma_tf32(dcol, dxl, dgh, idesc, 1u);
                    }
                }
                mma_commit(&empty[s]);
                if (seg_last) mma_commit(&accfull[a]);
            }
            __syncwarp();
        }
    } else if (warp < 4) {
        const int t = threadIdx.x - 64;
        for (int c = 0; c < nchunks && ok; ++c) {
            const int s = c % MN_NSTAGE;
            if (!(ok = mbar_wait_bounded(&full[s], (c / MN_NSTAGE) & 1, err, 0x213))) break;
            split_tf32(reinterpret_cast<float4 *>(op(s, 0)), reinterpret_cast<float4 *>(op(s, 1)),
                       MN_OP_BYTES / 16, t, 64);
            split_tf32(reinterpret_cast<float4 *>(op(s, 2)), reinterpret_cast<float4 *>(op(s, 3)),
                       MN_OP_BYTES / 16, t, 64);
            fence_proxy_async_smem();
            mbar_arrive(&conv[s]);
        }
    } else {
        const int q = warp & 3;
        float *dst0 = partial + (size_t)blockIdx.x * D * D;
        const int nseg = (nchunks + kSegChunks - 1) / kSegChunks;
        for (int seg = 0; seg < nseg && ok; ++seg) {
            const int a = seg % S::NACC;
            if (!(ok = mbar_wait_bounded(&accfull[a], (seg / S::NACC) & 1, err, 0x214))) break;
            tc_fence_after();
            for (int h = 0; h < S::HALVES; ++h) {
                const int i = h * 128 + q * 32 + lane;
                const uint32_t taddr =
                    tmem + ((uint32_t)(q * 32) << 16) + a * S::ACC_COLS + h * D;
                drain_segment(taddr, dst0, D, i, seg == 0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[a]);
        }
        if (nchunks == 0) {
            for (int h = 0; h < S::HALVES; ++h) {
                const int i = h * 128 + q * 32 + lane;
                for (int k = 0; k < D; ++k) dst0[partial_off(D, i, k)] = 0.0f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, S::TMEM_COLS);
}

// ---------------------------------------------------------- small helpers --
__global__ void fill_identity_kernel(float *I, int D) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e < D * D) I[e] = (e / D == e % D) ? 1.0f : 0.0f;
}

__global__ void repeat_row_kernel(const float *w, float *W, int D) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e < D * D) W[e] = w[e % D];
}

// mats = [Bf_hi | Bf_lo | Bd_hi | Bd_lo], Bf[k][i] = M[i][k], Bd[i][k] = M[i][k].
// Each thread reads only M[e] before writing, so M may be the Bd_hi quarter.
__global__ void split_mats_kernel(const float *M, float *mats, int D) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= D * D) return;
    const int i = e / D, k = e % D;
    const float v = M[e];
    const float hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    const float lo = v - hi;
    const size_t DD = (size_t)D * D;
    mats[(size_t)k * D + i] = hi;
    mats[DD + (size_t)k * D + i] = lo;
    mats[2 * DD + e] = hi;
    mats[3 * DD + e] = lo;
}

// G[row][col] = sum over partials (stored in partial_off order), accumulated
// in double in a fixed order.
__global__ void reduce_partials_kernel(const float *partial, int parts, int D, float *G) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= D * D) return;
    double s = 0.0;
    for (int p = 0; p < parts; ++p) s += (double)partial[(size_t)p * D * D + e];
    const int h = e / (128 * D), rem = e % (128 * D);
    const int row = h * 128 + (rem & 511) / 4, col = (rem / 512) * 4 + (rem & 3);
    G[row * D + col] = (float)s;
}

__global__ void column_sum_kernel(const float *A, int D, float *out) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= D) return;
    float s = 0.0f;
    for (int i = 0; i < D; ++i) s += A[(size_t)i * D + k];
    out[k] = s;
}

bool gemm_supported(int n) { return n == 7 || n == 8; }

int check_layer(int op, int n, uint32_t neg, uint32_t zero) {
    if (op < CB_OP_GP || op > CB_OP_REG) {
        set_error("layer: op %d out of range", op);
        return CB_ERR_INVALID;
    }
    if (!gemm_supported(n)) {
        set_error("layer GEMM path supports n = 7 and 8; got n = %d", n);
        return CB_ERR_UNSUPPORTED;
    }
    const uint32_t nmask = (1u << n) - 1;
    if ((neg & ~nmask) || (zero & ~nmask) || (neg & zero) || (op == CB_OP_REG && zero)) {
        set_error("layer: invalid metric masks for op %d", op);
        return CB_ERR_INVALID;
    }
    return CB_OK;
}

// CTA-pair form of the MN-major kernel for D = 256 (tcgen05 cta_group::2,
// M = 256): both CTAs of a pair read the same rows; CTA r loads features
// 128r..128r+127 of X (its half of M) and of dY (its half of N), so each SM
// splits and feeds the tensor core half of every operand chunk. Converters
// write only lo = v - hi next to the raw values, which serve as hi: the tf32
// MMA reads the top 19 bits of each fp32 operand (sign, exponent, 10 mantissa
// bits) and ignores the rest, so the raw value is read as exactly
// hi = v & 0xFFFFE000. The fp32-accuracy tests of the layer and rotor
// backward passes fail if that does not hold. CTA r's TMEM holds rows
// 128r..128r+127 of the pair's D x D partial.
struct MNPairSmem {
    static constexpr int HALF = 128;                    // features per CTA
    static constexpr int OP_BYTES = HALF * BKR * 4;     // 8 KB
    static constexpr int STAGE = 4 * OP_BYTES;          // X raw, X lo, dY raw, dY lo
    static constexpr int NSTAGE = 6;
    static constexpr int BYTES = 1024 + NSTAGE * STAGE + 256;
    static constexpr int ACC_COLS = 256;                // one 128 x 256 accumulator per CTA
    static constexpr int TMEM_COLS = 2 * ACC_COLS;      // two, alternating per segment
    static constexpr int CONV_WARPS = 6;                // warps 2-7
};
// Warps of gemm_mn_pair_kernel: 0 TMA, 1 TMEM allocation + MMA issue (even
// CTA), 2-7 converters, 8-11 epilogue. The epilogue drains one segment while
// the converters and the MMA work on the next, so it needs warps of its own.
constexpr int kPairMNThreads = 384;

// lo = v - (v with the low 13 mantissa bits cleared), v read from `raw`.
__device__ __forceinline__ void split_lo(const float4 *raw, float4 *lo, int count, int t, int nt) {
    for (int e = t; e < count; e += nt) {
        const float4 v = raw[e];
        lo[e] = make_float4(v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u),
                            v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u),
                            v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u),
                            v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
    }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairMNThreads, 1)
    gemm_mn_pair_kernel(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mG,
                        float *__restrict__ partial, int64_t rows, int64_t rows_per_part, int *err) {
    using S = MNPairSmem;
    constexpr int D = 256;
    constexpr int NS = S::NSTAGE;
    extern __shared__ unsigned char smem_raw[];
    // 1 KB-aligned start, derived by pointer arithmetic on the shared array so
    // the compiler keeps the shared address space; identical in both CTAs.
    unsigned char *const base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    unsigned char *stage0 = base;
    uint64_t *bars = reinterpret_cast<uint64_t *>(stage0 + NS * S::STAGE);
    uint64_t *full = bars, *conv = bars + NS, *empty = bars + 2 * NS, *accfull = bars + 3 * NS,
             *accempty = bars + 3 * NS + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * NS + 4);
    auto op = [&](int s, int which) { return stage0 + s * S::STAGE + which * S::OP_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int part = blockIdx.x >> 1;
    const int64_t r0 = (int64_t)part * rows_per_part;
    const int64_t r1 = std::min<int64_t>(rows, r0 + rows_per_part);
    const int nchunks = r1 > r0 ? (int)((r1 - r0 + BKR - 1) / BKR) : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 2 * S::CONV_WARPS);  // converter warps of both CTAs
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&accfull[a], 1);
            mbar_init(&accempty[a], 8);  // the epilogue warps of both CTAs (even CTA's counts)
        }
        fence_barrier_init();
        prefetch_tensormap(&mX);
        prefetch_tensormap(&mG);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            const int f0 = (int)rank * S::HALF;
            for (int c = 0; c < nchunks && ok; ++c) {
                const int s = c % NS;
                if (!(ok = mbar_wait_bounded(&empty[s], ((c / NS) + 1) & 1, err, 0x221))) break;
                mbar_arrive_expect_tx(&full[s], 2 * S::OP_BYTES);
                const int row = (int)(r0 + (int64_t)c * BKR);
                for (int g = 0; g < S::HALF / 32; ++g) {
                    tma_load_2d(op(s, 0) + g * MN_BOX_BYTES, &mX, f0 + g * 32, row, &full[s]);
                    tma_load_2d(op(s, 2) + g * MN_BOX_BYTES, &mG, f0 + g * 32, row, &full[s]);
                }
            }
            // The last commits arrive on this CTA's empty barriers from the
            // even CTA; take them before the CTA may exit.
            for (int j = nchunks - NS < 0 ? 0 : nchunks - NS; j < nchunks && ok; ++j)
                ok = mbar_wait_bounded(&empty[j % NS], (j / NS) & 1, err, 0x226);
        }
    } else if (warp == 1) {
        if (leader) {
            constexpr uint32_t idesc = idesc_tf32(2 * BM, D, true, true);
            for (int c = 0; c < nchunks && ok; ++c) {
                const int s = c % NS;
                const int seg = c / kSegChunks, a = seg & 1;
                const bool seg_first = (c % kSegChunks) == 0;
                const bool seg_last = (c % kSegChunks) == kSegChunks - 1 || c == nchunks - 1;
                // accumulator a is free once both CTAs drained its previous segment
                if (lane == 0 && seg_first && seg >= 2)
                    ok = mbar_wait_bounded(&accempty[a], (seg / 2 - 1) & 1, err, 0x225,
                                           2000000000ull, true);
                if (lane == 0 && ok)
                    ok = mbar_wait_bounded(&conv[s], (c / NS) & 1, err, 0x222, 2000000000ull, true);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t xh = smem_u32(op(s, 0)), xl = smem_u32(op(s, 1));
                    const uint32_t gh = smem_u32(op(s, 2)), gl = smem_u32(op(s, 3));
#pragma unroll
                    for (int kk = 0; kk < BKR / 8; ++kk) {
                        const uint32_t koff = kk * 1024;  // next 8 rows of K
                        const uint64_t dxh = mnmajor_desc(xh + koff, MN_BOX_BYTES);
                        const uint64_t dxl = mnmajor_desc(xl + koff, MN_BOX_BYTES);
                        const uint64_t dgh = mnmajor_desc(gh + koff, MN_BOX_BYTES);
                        const uint64_t dgl = mnmajor_desc(gl + koff, MN_BOX_BYTES);
                        const uint32_t acc = tmem + a * S::ACC_COLS;
                        mma_tf32_pair(acc, dxh, dgh, idesc, (seg_first && kk == 0) ? 0u : 1u);
                        mma_tf32_pair(acc, dxh, dgl, idesc, 1u);
                        mma_tf32_pair(acc, dxl, dgh, idesc, 1u);
                    }
                    mma_commit_pair(&empty[s]);
                    if (seg_last) mma_commit_pair(&accfull[a]);
                }
                __syncwarp();
            }
        }
    } else if (warp < 2 + S::CONV_WARPS) {
        const int t = threadIdx.x - 64;
        for (int c = 0; c < nchunks && ok; ++c) {
            const int s = c % NS;
            if (!(ok = mbar_wait_bounded(&full[s], (c / NS) & 1, err, 0x223))) break;
            split_lo(reinterpret_cast<const float4 *>(op(s, 0)), reinterpret_cast<float4 *>(op(s, 1)),
                     S::OP_BYTES / 16, t, 32 * S::CONV_WARPS);
            split_lo(reinterpret_cast<const float4 *>(op(s, 2)), reinterpret_cast<float4 *>(op(s, 3)),
                     S::OP_BYTES / 16, t, 32 * S::CONV_WARPS);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(&conv[s], 0);
        }
    } else {
        {  // epilogue warps 8-11: TMEM lane quarter warp % 4
            const int q = warp & 3;
            const int i = (int)rank * S::HALF + q * 32 + lane;
            float *dst0 = partial + (size_t)part * D * D;
            const int nseg = (nchunks + kSegChunks - 1) / kSegChunks;
            for (int seg = 0; seg < nseg && ok; ++seg) {
                const int a = seg & 1;
                if (!(ok = mbar_wait_bounded(&accfull[a], (seg / 2) & 1, err, 0x224))) break;
                tc_fence_after();
                drain_segment(tmem + ((uint32_t)(q * 32) << 16) + a * S::ACC_COLS, dst0, D, i,
                              seg == 0);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(&accempty[a], 0);
            }
            if (nchunks == 0) {
                for (int k = 0; k < D; ++k) dst0[partial_off(D, i, k)] = 0.0f;
            }
        }
    }
    tc_fence_before();
    cluster_sync();  // no MMA of the pair still reads this CTA's tiles or TMEM
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, S::TMEM_COLS);
}


// Split of the batch for G = X^T dY: about 512 rows per partial, at most 8
// partials per SM (the partials are summed in double; within a partial the
// TMEM accumulation restarts every kSegChunks chunks).
constexpr int kRowsPerPart = 512;
int mn_parts(const DeviceInfo &di, int64_t batch) {
    const int64_t want = (batch + kRowsPerPart - 1) / kRowsPerPart;
    return (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)8 * di.sm_count, want));
}

// workspace: I | Wrep | M | fold | G | partials (floats)
size_t layer_ws_floats(int n, int parts) {
    const size_t DD = (size_t)1 << (2 * n);
    return 5 * DD + (size_t)parts * DD;
}

template <int D>
int launch_kmajor(const float *A, const float *Bhi, const float *Blo, float *Y, int64_t rows,
                  cudaStream_t s) {
    if (rows == 0) return CB_OK;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    CUtensorMap mA, mBh, mBl, mY;
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
    if ((st = make_tmap_2d(&mY, Y, D, rows, D * 4, 32, 32))) return st;
    if ((st = make_tmap_2d(&mA, A, D, rows, D * 4, BK, BM, sw))) return st;
    if ((st = make_tmap_2d(&mBh, Bhi, D, D, D * 4, BK, D / 2, sw))) return st;
    if ((st = make_tmap_2d(&mBl, Blo, D, D, D * 4, BK, D / 2, sw))) return st;
    using S = KMajorSmem<D>;
    auto kern = gemm_kmajor_kernel<D>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_kmajor)");
    const int64_t tiles = (rows + 2 * BM - 1) / (2 * BM);  // 256-row pair tiles
    if (rows >= ((int64_t)1 << 31)) {  // TMA row coordinates are 32-bit signed
        set_error("layer: batch too large");
        return CB_ERR_UNSUPPORTED;
    }
    static int max_pairs[64] = {};  // per device: co-resident CTA pairs
    int dev = 0;
    cudaGetDevice(&dev);
    int &mp = max_pairs[dev & 63];
    if (mp == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (di.sm_count / 2));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = S::BYTES;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = di.sm_count / 2;
        }
        mp = n;
    }
    const int grid = 2 * (int)std::min<int64_t>(tiles, mp);
    kern<<<grid, kThreads, S::BYTES, s>>>(mA, mBh, mBl, mY, (int)tiles, err);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gemm_kmajor_kernel");
}

template <int D>
int launch_mn(const float *x, const float *dy, float *partial, int64_t batch, int parts,
              cudaStream_t s) {
    int *err = nullptr;
    int st = device_error_word(&err);
    if (st) return st;
    CUtensorMap mX, mG;
    if ((st = make_tmap_2d(&mX, x, D, batch, D * 4, 32, BKR, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
        return st;
    if ((st = make_tmap_2d(&mG, dy, D, batch, D * 4, 32, BKR, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)))
        return st;
    const int64_t chunks = (batch + BKR - 1) / BKR;
    const int64_t rows_per_part = ((chunks + parts - 1) / parts) * BKR;
    cudaError_t e;
    if constexpr (D == 256) {  // one CTA pair per partial
        e = cudaFuncSetAttribute(gemm_mn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 MNPairSmem::BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_mn_pair)");
        gemm_mn_pair_kernel<<<2 * parts, kPairMNThreads, MNPairSmem::BYTES, s>>>(mX, mG, partial, batch,
                                                                             rows_per_part, err);
    } else {
        auto kern = gemm_mn_kernel<D>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MNSmem<D>::BYTES);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_mn)");
        kern<<<parts, kThreads, MNSmem<D>::BYTES, s>>>(mX, mG, partial, batch, rows_per_part, err);
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gemm_mn_kernel");
}

}  // namespace

int gemm3x_kmajor(int D, const float *A, const float *Bhi, const float *Blo, float *Y,
                  int64_t rows, cudaStream_t s) {
    if (D == 256) return launch_kmajor<256>(A, Bhi, Blo, Y, rows, s);
    if (D == 128) return launch_kmajor<128>(A, Bhi, Blo, Y, rows, s);
    set_error("gemm3x_kmajor: D = %d unsupported", D);
    return CB_ERR_UNSUPPORTED;
}

int gemm3x_mn_parts(int64_t rows) {
    DeviceInfo di;
    if (device_info(&di)) return -1;
    return mn_parts(di, std::max<int64_t>(rows, 1));
}

int gemm3x_mn(int D, const float *X, const float *dY, float *partial, int64_t rows, int parts,
              cudaStream_t s) {
    if (D == 256) return launch_mn<256>(X, dY, partial, rows, parts, s);
    if (D == 128) return launch_mn<128>(X, dY, partial, rows, parts, s);
    set_error("gemm3x_mn: D = %d unsupported", D);
    return CB_ERR_UNSUPPORTED;
}

int reduce_partials(const float *partial, int parts, int D, float *G, cudaStream_t s) {
    reduce_partials_kernel<<<(D * D + 255) / 256, 256, 0, s>>>(partial, parts, D, G);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch reduce_partials_kernel");
}

int split_mats(const float *M, float *mats, int D, cudaStream_t s) {
    split_mats_kernel<<<(D * D + 255) / 256, 256, 0, s>>>(M, mats, D);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch split_mats_kernel");
}

}  // namespace cb

using namespace cb;

extern "C" int cb_layer_workspace_bytes(int n, int64_t batch, int64_t *bytes) {
    if (!gemm_supported(n)) {
        set_error("layer GEMM path supports n = 7 and 8; got n = %d", n);
        return CB_ERR_UNSUPPORTED;
    }
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    *bytes = (int64_t)layer_ws_floats(n, mn_parts(di, std::max<int64_t>(batch, 1))) * 4;
    return CB_OK;
}

extern "C" int cb_layer_prepare(int op, const float *w, int n, uint32_t neg_mask,
                                uint32_t zero_mask, float *mats, void *workspace,
                                int64_t workspace_bytes, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = check_layer(op, n, neg_mask, zero_mask);
    if (st) return st;
    const int D = 1 << n;
    const size_t DD = (size_t)D * D;
    if (!w || !mats || !workspace || workspace_bytes < (int64_t)(3 * DD * 4)) {
        set_error("layer_prepare: invalid arguments or workspace too small");
        return CB_ERR_INVALID;
    }
    float *I = static_cast<float *>(workspace), *W = I + DD, *M = W + DD;
    const int blocks = (int)((DD + 255) / 256);
    fill_identity_kernel<<<blocks, 256, 0, s>>>(I, D);
    repeat_row_kernel<<<blocks, 256, 0, s>>>(w, W, D);
    if ((st = bilinear(op, CB_MODE_FWD, I, W, M, D, n, neg_mask, zero_mask, s))) return st;
    split_mats_kernel<<<blocks, 256, 0, s>>>(M, mats, D);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch layer prepare kernels");
}

extern "C" int cb_layer_forward(const float *mats, const float *x, float *y, int64_t batch, int n,
                                void *stream) {
    if (!gemm_supported(n)) {
        set_error("layer GEMM path supports n = 7 and 8; got n = %d", n);
        return CB_ERR_UNSUPPORTED;
    }
    if (batch < 0 || (batch > 0 && (!mats || !x || !y || x == y))) {
        set_error("layer_forward: invalid arguments");
        return CB_ERR_INVALID;
    }
    const size_t DD = (size_t)1 << (2 * n);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return n == 8 ? launch_kmajor<256>(x, mats, mats + DD, y, batch, s)
                  : launch_kmajor<128>(x, mats, mats + DD, y, batch, s);
}

extern "C" int cb_layer_backward(int op, const float *mats, const float *x, const float *dy,
                                 float *dx, float *dw, int64_t batch, int n, uint32_t neg_mask,
                                 uint32_t zero_mask, void *workspace, int64_t workspace_bytes,
                                 void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = check_layer(op, n, neg_mask, zero_mask);
    if (st) return st;
    if (batch < 0 || !mats || (batch > 0 && (!x || !dy))) {
        set_error("layer_backward: invalid arguments");
        return CB_ERR_INVALID;
    }
    const int D = 1 << n;
    const size_t DD = (size_t)D * D;
    if (dx && batch > 0) {
        st = n == 8 ? launch_kmajor<256>(dy, mats + 2 * DD, mats + 3 * DD, dx, batch, s)
                    : launch_kmajor<128>(dy, mats + 2 * DD, mats + 3 * DD, dx, batch, s);
        if (st) return st;
    }
    if (!dw) return CB_OK;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const int parts = mn_parts(di, batch);
    if (!workspace || workspace_bytes < (int64_t)layer_ws_floats(n, parts) * 4) {
        set_error("layer_backward: workspace of %lld bytes needed",
                  (long long)layer_ws_floats(n, parts) * 4);
        return CB_ERR_INVALID;
    }
    float *I = static_cast<float *>(workspace);
    float *fold = I + 3 * DD, *G = I + 4 * DD, *partial = I + 5 * DD;
    const int blocks = (int)((DD + 255) / 256);
    cudaError_t e;
    if (batch > 0) {
        st = n == 8 ? launch_mn<256>(x, dy, partial, batch, parts, s)
                    : launch_mn<128>(x, dy, partial, batch, parts, s);
        if (st) return st;
        reduce_partials_kernel<<<blocks, 256, 0, s>>>(partial, parts, D, G);
    } else {
        e = cudaMemsetAsync(G, 0, DD * 4, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(G)");
    }
    fill_identity_kernel<<<blocks, 256, 0, s>>>(I, D);
    if ((st = bilinear(op, CB_MODE_GRAD_B, I, G, fold, D, n, neg_mask, zero_mask, s))) return st;
    column_sum_kernel<<<(D + 255) / 256, 256, 0, s>>>(fold, D, dw);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch layer fold kernels");
}

// ----------------------------------------- GP layer of Cl(8,0), matrix route --
namespace {
int gp8_aligned(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" int cb_layer_gp8_prepare(const float *w, float *mats, void *stream) {
    if (!w || !mats || !gp8_aligned(mats)) {
        set_error("layer_gp8_prepare: null or unaligned pointer");
        return CB_ERR_INVALID;
    }
    return gp_layer_weight(w, mats, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_layer_gp8_forward(const float *mats, const float *x, float *y, int64_t batch,
                                    void *stream) {
    if (batch < 0 || (batch > 0 && (!mats || !x || !y || x == y))) {
        set_error("layer_gp8_forward: invalid arguments");
        return CB_ERR_INVALID;
    }
    if (batch > 0 && (!gp8_aligned(mats) || !gp8_aligned(x) || !gp8_aligned(y))) {
        set_error("layer_gp8_forward: rows must be 16-byte aligned");
        return CB_ERR_INVALID;
    }
    return gp_layer_apply(mats, x, y, batch, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_layer_gp8_backward(const float *mats, const float *x, const float *dy,
                                     float *dx, float *dw, int64_t batch, void *workspace,
                                     int64_t workspace_bytes, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (batch < 0 || !mats || (batch > 0 && (!x || !dy)) || (dx && (dx == dy || dx == x))) {
        set_error("layer_gp8_backward: invalid arguments");
        return CB_ERR_INVALID;
    }
    if (batch > 0 && (!gp8_aligned(x) || !gp8_aligned(dy) || (dx && !gp8_aligned(dx)))) {
        set_error("layer_gp8_backward: rows must be 16-byte aligned");
        return CB_ERR_INVALID;
    }
    int st;
    if (dx && (st = gp_layer_apply(mats + kGpLayerWFloats, dy, dx, batch, s))) return st;
    if (!dw) return CB_OK;
    const int parts = gp_layer_dw_parts(batch);
    if (parts <= 0 || !workspace || workspace_bytes < (int64_t)parts * 256 * 4) {
        set_error("layer_gp8_backward: workspace of %lld bytes needed",
                  (long long)(parts > 0 ? parts : 0) * 256 * 4);
        return CB_ERR_INVALID;
    }
    return gp_layer_dw(x, dy, dw, static_cast<float *>(workspace), batch, s);
}
