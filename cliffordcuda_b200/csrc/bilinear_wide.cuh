// bilinear_wide.cuh -- the batch-by-batch bilinear sums for large algebras,
// 11 <= n <= 16 (rows of 8 KB to 256 KB), instantiated per sum in
// bilinear_wide_{fwd,ga,gb}.cu. Reference: the tiled fused product the
// reference switches to past its standard kernel's limit
// (extensions/ga/geom_prod_tiled.py:370-398, kernels/ga/geom_prod_tiled.cu:29-163;
// dispatch geom_prod.py:253-275).
//
// Same arithmetic as bilinear_tiled.cuh (read its header first): blade
// indices split into high bits (5..n-1, the 128-byte line of a row) and low
// bits (0..4, the float within the line); a thread owns the 32 outputs of one
// line k_h of one row and sweeps the lines i_h, each step up to 1024 FFMAs
// with compile-time +-1 coefficients, the runtime high-part sign folded into
// y. What changes with n is the data movement:
//
//   * a row has NH = 2^(n-5) lines (64 .. 2048). The output lines of a row are
//     cut into blocks KB of 128 lines (64 at n = 11, where a tile holds two
//     rows); one CTA of 128 threads owns one block of one row;
//   * for an input block IB of 128 lines of x, the y lines a step reads,
//     i_h ^ k_h with i_h in IB and k_h in KB, are exactly the block IB ^ KB.
//     So the CTA streams pairs (x block IB, y block IB ^ KB), 16 KB each, by
//     2-D TMA (128-byte swizzle) through a two-stage mbarrier pipeline, and
//     sweeps the 128 lines of each pair: 128 x 128 x 1024 FFMAs per 32 KB;
//     a unit's sums leave from registers (float4 stores, or float atomics
//     into the zeroed output where several units add into one block);
//   * the high-part factor of a step is computed from popcounts (no per-CTA
//     table: it would take 4^(n-5) entries);
//   * when rows x blocks is too small to fill the GPU (a few rows of a large
//     algebra), the input blocks of each output block are split over several
//     CTAs that add their sums into the zeroed output with float atomics
//     (summation order, so the last bits, may then differ between runs).
//
// Inner product: left + right contraction minus the doubly counted P == Q
// terms, as in the tiled kernel; the forward sum's correction out[0] -=
// sum_i s(i, i) x_i y_i is accumulated by the CTAs of block KB = 0 (whose y
// block equals the x block), reduced per warp and added atomically; the backward
// sums' out[k] -= s(k, k) x_k y_0 are applied at the step IB == KB (whose
// x block holds line k_h and whose y block holds line 0).
#pragma once
#include "bilinear_tiled.cuh"

namespace cb {
namespace wide {

using tiled::kBlk;
using tiled::kLow;
using tiled::OPK_GP;
using tiled::OPK_INNER;
using tiled::OPK_LC;
using tiled::OPK_RC;
using tiled::OPK_WEDGE;

constexpr int kThreads = 128;                 // four warps, one output line each
constexpr int kLines = 128;                   // lines per streamed block
constexpr int kBlockFloats = kLines * kBlk;   // 4096 floats, 16 KB
constexpr int kBlockBytes = kBlockFloats * 4;
constexpr int kStages = 2;
constexpr int kMinN = 11, kMaxN = 16;

__host__ __device__ inline size_t smem_bytes() {
    return 1024 /* alignment slack */ + 2 * kStages * size_t(kBlockBytes) + 128;
}

// Layout of one launch: lines per row NH, lines of a row inside a block NHt
// (= min(NH, 128)), rows per block rpt (= 128 / NHt), input steps per output
// block nb (= NH / NHt), output blocks per row nbk (= nb), and the split of
// each output block's nb steps into `splits` units of `spu` steps.
struct Plan {
    int n, lgNH, NHt, rpt, nb, nbk, splits, spu;
    int64_t tiles, units;  // tiles = row groups of rpt rows; units = tiles * nbk * splits
};

template <int MODE, int OPK>
__device__ __forceinline__ void wide_sweep(float (&acc)[kBlk], const float *xt, const float *yt,
                                           int rowl, int NHt, uint32_t ih0, uint32_t kh, int khl,
                                           uint32_t negH, uint32_t zeroH, bool skip_zero) {
    using namespace tiled;
#pragma unroll 1
    for (int ihl = 0; ihl < NHt; ++ihl) {
        const uint32_t ih = ih0 + ihl;
        float2 sg, sg2 = make_float2(0.0f, 0.0f);
        if (OPK == OPK_INNER) {
            sg = high_factor(MODE, OPK_LC, ih, kh, negH, zeroH);
            sg2 = high_factor(MODE, OPK_RC, ih, kh, negH, zeroH);
        } else {
            sg = high_factor(MODE, OPK, ih, kh, negH, zeroH);
        }
        // warp-uniform skip of steps whose high-part factor is zero for every
        // lane (a null generator in both high parts, or the product's predicate)
        if (skip_zero &&
            __all_sync(0xffffffffu, sg.x == 0.0f && sg.y == 0.0f && sg2.x == 0.0f && sg2.y == 0.0f))
            continue;
        float xv[kBlk], yv[kBlk];
        load_block(xt, rowl + ihl, xv);
        load_block(yt, rowl + (ihl ^ khl), yv);
        if (MODE == CB_MODE_GRAD_B) {  // x side of the cross term
            const float sx = parity(ih) ? -1.0f : 1.0f;
#pragma unroll
            for (int e = 0; e < kBlk; ++e)
                if (popcl(e) & 1) xv[e] *= sx;
        }
        if (OPK == OPK_INNER) {
            float y2[kBlk];
#pragma unroll
            for (int e = 0; e < kBlk; ++e) y2[e] = yv[e];
            apply_sign(yv, sg);
            apply_sign(y2, sg2);
            block_fma<MODE, OPK_LC>(acc, xv, yv);
            block_fma<MODE, OPK_RC>(acc, xv, y2);
        } else {
            apply_sign(yv, sg);
            block_fma<MODE, OPK>(acc, xv, yv);
        }
    }
}

// s_L(e, e) (-1)^(popc(k_h) popc(e)) for the diagonal terms of line k_h.
__device__ __forceinline__ float diag_low_sign(int e, uint32_t kh) {
    using namespace tiled;
    return (reorderl(e, e) ^ ((popcl(e) & 1) & parity(kh))) ? -1.0f : 1.0f;
}

template <int MODE, int OPK>
__global__ void __launch_bounds__(kThreads, 3)
    bilinear_wide_kernel(const __grid_constant__ CUtensorMap mx,
                         const __grid_constant__ CUtensorMap my, float *__restrict__ out,
                         const Plan P, int64_t batch, uint32_t neg, uint32_t zero, int *err,
                         bool skip_zero) {
    using namespace tiled;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *const base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    float *xs = reinterpret_cast<float *>(base);  // [kStages][kBlockFloats]
    float *ys = xs + kStages * kBlockFloats;      // [kStages][kBlockFloats]
    uint64_t *full = reinterpret_cast<uint64_t *>(ys + kStages * kBlockFloats);
    int *done_count = reinterpret_cast<int *>(full + kStages);  // [kStages]
    // Sums are added into a zeroed output when units share an output block
    // and for the inner product's forward diagonal correction.
    const bool atomic_out = P.splits > 1 || (OPK == OPK_INNER && MODE == CB_MODE_FWD);

    const int tid = threadIdx.x, lane = tid & 31;
    const int NH = 1 << P.lgNH;
    const uint32_t negH = neg >> kLow, zeroH = zero >> kLow;
    const int r = tid / P.NHt;        // row of the block (0 unless n = 11)
    const int khl = tid % P.NHt;      // output line within the block
    const int rowl = r * P.NHt;       // first local line of this thread's row

    // step f of this CTA -> unit u, input block IB; the loads of step f
    auto step_unit = [&](int64_t f) { return (int64_t)blockIdx.x + (f / P.spu) * gridDim.x; };
    auto issue = [&](int64_t f, int s) {
        const int64_t u = step_unit(f);
        const int split = (int)(u % P.splits);
        const int64_t ob = u / P.splits;  // output block index
        const int64_t tile = ob / P.nbk;
        const int KB = (int)(ob % P.nbk);
        const int IB = split * P.spu + (int)(f % P.spu);
        const int64_t line0 = tile * (int64_t)kLines * (P.rpt > 1 ? 1 : P.nb);
        mbar_arrive_expect_tx(&full[s], 2 * kBlockBytes);
        tma_load_2d(xs + s * kBlockFloats, &mx, 0, (int)(line0 + (int64_t)IB * kLines), &full[s]);
        tma_load_2d(ys + s * kBlockFloats, &my, 0, (int)(line0 + (int64_t)(IB ^ KB) * kLines),
                    &full[s]);
    };
    const int64_t my_units = P.units > blockIdx.x
                                 ? (P.units - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int64_t nsteps = my_units * P.spu;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            done_count[s] = 0;
        }
        fence_barrier_init();
        prefetch_tensormap(&mx);
        prefetch_tensormap(&my);
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kStages && s < nsteps; ++s) issue(s, s);

    float acc[kBlk];
    float dsum = 0.0f;  // inner forward: this thread's share of sum_i s(i,i) x_i y_i
    for (int64_t f = 0; f < nsteps; ++f) {
        const int s = (int)(f % kStages);
        const int64_t u = step_unit(f);
        const int split = (int)(u % P.splits);
        const int64_t ob = u / P.splits;
        const int64_t tile = ob / P.nbk;
        const int KB = (int)(ob % P.nbk);
        const int fs = (int)(f % P.spu);
        const int IB = split * P.spu + fs;
        const uint32_t kh = (uint32_t)(KB * P.NHt + khl);
        if (fs == 0) {
#pragma unroll
            for (int e = 0; e < kBlk; ++e) acc[e] = 0.0f;
            dsum = 0.0f;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (f / kStages) & 1, err, 0x141)))
            break;
        const float *xt = xs + s * kBlockFloats;
        const float *yt = ys + s * kBlockFloats;
        wide_sweep<MODE, OPK>(acc, xt, yt, rowl, P.NHt, (uint32_t)(IB * P.NHt), kh, khl, negH,
                              zeroH, skip_zero);
        if (OPK == OPK_INNER) {
            if (MODE == CB_MODE_FWD && KB == 0) {
                // line i_h = IB * NHt + khl of x and of y (the y block is IB here)
                const uint32_t ih = (uint32_t)(IB * P.NHt + khl);
                const int sh = blade_sign(ih, ih, negH, zeroH);
                if (sh != 0) {
                    float xv[kBlk], yv[kBlk];
                    load_block(xt, rowl + khl, xv);
                    load_block(yt, rowl + khl, yv);
#pragma unroll
                    for (int e = 0; e < kBlk; ++e)
                        dsum = fmaf((float)sh * diag_low_sign(e, ih) * xv[e], yv[e], dsum);
                }
            } else if (MODE != CB_MODE_FWD && IB == KB) {
                // out[k] -= s(k, k) x_k y_0: x line k_h is local line khl, y line 0 local line 0.
                // grad_a negates the odd-parity outputs of odd lines at the end
                // (the x side of the cross term); the correction is not part of
                // that sign, so it enters pre-negated there.
                const int shh = blade_sign(kh, kh, negH, zeroH);
                if (shh != 0) {
                    float xv[kBlk];
                    load_block(xt, rowl + khl, xv);
                    const float y0 = yt[swz_index(rowl << 5)];
                    const bool flip = MODE == CB_MODE_GRAD_A && parity(kh);
#pragma unroll
                    for (int e = 0; e < kBlk; ++e) {
                        const float f = (flip && (popcl(e) & 1)) ? -1.0f : 1.0f;
                        acc[e] = fmaf(-(float)shh * f * diag_low_sign(e, kh) * xv[e], y0, acc[e]);
                    }
                }
            }
        }
        // release the stage: the last warp done reloads it
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&done_count[s], 1) == kThreads / 32 - 1) {
                done_count[s] = 0;
                if (f + kStages < nsteps) issue(f + kStages, s);
            }
        }
        __syncwarp();

        if (fs == P.spu - 1) {  // the unit's last step: finish and write its sums
            if (MODE == CB_MODE_GRAD_A && parity(kh)) {
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    if (popcl(e) & 1) acc[e] = -acc[e];
            }
            const int64_t row = tile * P.rpt + r;
            const int64_t D = (int64_t)NH * kBlk;
            if (OPK == OPK_INNER && MODE == CB_MODE_FWD && KB == 0) {
                // the warp's lanes are 32 lines of one row: one atomic per warp
                for (int m = 16; m > 0; m >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, m);
                if (lane == 0 && row < batch) atomicAdd(out + row * D, -dsum);
            }
            if (row < batch) {
                float *o = out + row * D + (int64_t)kh * kBlk;
                if (!atomic_out) {
                    float4 *o4 = reinterpret_cast<float4 *>(o);
#pragma unroll
                    for (int t = 0; t < kBlk / 4; ++t)
                        o4[t] = make_float4(acc[4 * t], acc[4 * t + 1], acc[4 * t + 2],
                                            acc[4 * t + 3]);
                } else {
#pragma unroll
                    for (int e = 0; e < kBlk; ++e) atomicAdd(o + e, acc[e]);
                }
            }
        }
    }
}

template <int MODE, int OPK>
int launch_wide(const float *x, const float *y, float *out, int64_t batch, int n, uint32_t neg,
                uint32_t zero, cudaStream_t stream) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    Plan P;
    P.n = n;
    P.lgNH = n - kLow;
    const int NH = 1 << P.lgNH;
    P.NHt = NH < kLines ? NH : kLines;
    P.rpt = kLines / P.NHt;
    P.nb = NH / P.NHt;
    P.nbk = P.nb;
    P.tiles = (batch + P.rpt - 1) / P.rpt;
    const size_t smem = smem_bytes();
    auto kern = bilinear_wide_kernel<MODE, OPK>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bilinear_wide)");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (per_sm < 1) {
        set_error("bilinear wide kernel does not fit an SM (smem %zu)", smem);
        return CB_ERR_UNSUPPORTED;
    }
    const int64_t slots = (int64_t)per_sm * di.sm_count;
    const int64_t blocks = P.tiles * P.nbk;
    // split each output block's input steps when the blocks cannot fill the GPU
    P.splits = 1;
    while (blocks * P.splits < slots && P.splits < P.nb) P.splits <<= 1;
    P.spu = P.nb / P.splits;
    P.units = blocks * P.splits;
    if (P.splits > 1 || (OPK == OPK_INNER && MODE == CB_MODE_FWD)) {
        e = cudaMemsetAsync(out, 0, (size_t)batch * (1u << n) * sizeof(float), stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(out)");
    }
    // x and y as lines of 128 bytes; the rows past the batch in the last
    // block of two rows (n = 11) are read as zeros (TMA out-of-bounds fill)
    CUtensorMap mx, my;
    if ((st = make_tmap_lines(&mx, x, (uint64_t)batch * NH, kLines))) return st;
    if ((st = make_tmap_lines(&my, y, (uint64_t)batch * NH, kLines))) return st;
    const int grid = (int)std::min<int64_t>(P.units, slots);
    const bool skip_zero = true;
    kern<<<grid, kThreads, smem, stream>>>(mx, my, out, P, batch, neg, zero, err, skip_zero);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch bilinear_wide_kernel");
    return CB_OK;
}

}  // namespace wide

// Explicitly instantiated per mode in bilinear_wide_{fwd,ga,gb}.cu.
template <int MODE>
int bilinear_wide(int op, const float *x, const float *y, float *out, int64_t batch, int n,
                  uint32_t neg, uint32_t zero, cudaStream_t stream) {
    using namespace wide;
    switch (op) {
    case CB_OP_GP: return launch_wide<MODE, OPK_GP>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_WEDGE: return launch_wide<MODE, OPK_WEDGE>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_LC: return launch_wide<MODE, OPK_LC>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_RC: return launch_wide<MODE, OPK_RC>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_INNER: return launch_wide<MODE, OPK_INNER>(x, y, out, batch, n, neg, zero, stream);
    }
    set_error("op %d has no wide kernel", op);
    return CB_ERR_INVALID;
}

}  // namespace cb
