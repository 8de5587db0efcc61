// gp_mat16.cu -- the geometric product of Cl(8,0) and both of its backward
// sums through the real 16 x 16 matrix representation of the algebra.
//
// Cl(8,0) is isomorphic to the algebra of real 16 x 16 matrices. With 16 x 16
// generator matrices G_i (G_i^2 = 1, G_i G_j = -G_j G_i) the blade e_I maps to
// E_I = G_i1 G_i2 ... (i1 < i2 < ...), a signed permutation matrix, and the
// map rho(a) = sum_I a_I E_I turns the geometric product into a matrix
// product: rho(a * b) = rho(a) rho(b). The E_I are orthogonal with
// <E_I, E_J>_F = 16 delta_IJ, so rho / 4 is an isometry and the backward sums
// of the reference's autograd (grad_a = d<g, a*b>/da, grad_b = d<g, a*b>/db,
// reference extensions/ga/geom_prod.py:241-250) are
//     grad_a = rho^-1(rho(g) rho(b)^T),   grad_b = rho^-1(rho(a)^T rho(g)).
// Per product that is one 16 x 16 x 16 matrix product (4096 FMA) plus the
// basis changes, against 65,536 FMA per sum for the blade-by-blade sum; the
// kernel is bound by HBM instead of the FP32 pipe.
//
// Generators: tensor products of four real 2 x 2 Pauli factors
//   I, X = [[0,1],[1,0]], Z = [[1,0],[0,-1]], W = XZ = [[0,-1],[1,0]]
// (W^2 = -1), G_0 = I(x)I(x)I(x)X, G_1 = I(x)I(x)I(x)Z, and
// G_{2+i} = P_i (x) W with P_0..P_5 six mutually anticommuting 3-factor
// strings that square to -1 (kP below). A product of such strings is +-one
// string, so the coefficient vector of rho(a) in the string basis is a signed
// permutation of a, and the change from string coefficients to matrix entries
// factorises over the four factors into 2-term butterflies:
//   per factor, (c_I, c_Z) -> (m_00, m_11) = (c_I + c_Z, c_I - c_Z) and
//               (c_X, c_W) -> (m_01, m_10) = (c_X - c_W, c_X + c_W).
//
// Work split: a warp handles 8 products, 4 lanes each. Lane q of a product
// holds the 64 string coefficients whose last factor has code q; factors 1-3
// are transformed in registers, factor 4 by one shuffle with lane q ^ 2,
// after which lane q holds one 8 x 8 quadrant of the matrix (row parity
// q >> 1, column parity (q >> 1) ^ (q & 1)). Lanes store their quadrants to
// shared memory in the layout the product reads, each lane computes its
// quadrant of the 16 x 16 product by 16 outer-product steps, and the inverse
// transform runs the same way back. Rows come in and go out by bulk copies
// (1 KB each) into padded per-product regions of shared memory; each warp is
// its own CTA with one buffer.
#include <algorithm>
#include <utility>

#include "common.cuh"
#include "mat16_rep.cuh"

namespace cb {
namespace {

using namespace mat16;

// Shared layout of one product's row region: the raw 256-float row, then in
// place the four 8 x 8 quadrant blocks at a 72-float stride (their 16-byte
// chunks fall on bank groups 0, 2, 4, 6 mod 8). The region is 284 floats (71
// chunks, odd): the next product's blocks take bank groups 1, 3, 5, 7, so a
// quarter-warp's float4 block accesses (two products, four lanes each) are
// conflict-free, and the scalar gather of 8 products spreads over all 32 banks.
// 284 = 3 * 72 + 64 (the last block needs no padding) keeps a warp at 18.2 KB:
// 12 one-warp CTAs per SM.
constexpr int kRowFloats = 284;
constexpr int kBlockFloats = 72;
constexpr int kRegion = 8 * kRowFloats;      // 8 products
constexpr int kBufFloats = 2 * kRegion;      // U and V
constexpr int kSmemBytes = kBufFloats * 4 + 64;

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_store(void *gdst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}

// r[slot(k)] = sign(E_I) * lane factor * row[I] for all 64 k, where the
// blade I of register k in lane q has bits 2..7 = k and bits 0..1 = q, or
// q ^ 3 when k has odd parity (the W factors of G_2..G_7 also carry the
// last-factor code).
template <int K>
__device__ __forceinline__ void gather1(float (&r)[64], const float *row, int qx0, int qx3,
                                        const float (&S)[4]) {
    constexpr int m = popc8(K);
    const float v = row[4 * K + ((m & 1) ? qx3 : qx0)] * S[m & 3];
    r[slot_of(K)] = sig1_of(K) > 0 ? v : -v;
}
template <int... K>
__device__ __forceinline__ void gather(float (&r)[64], const float *row, int q, const float (&S)[4],
                                       std::integer_sequence<int, K...>) {
    (gather1<K>(r, row, q, q ^ 3, S), ...);
}
template <int K>
__device__ __forceinline__ void scatter1(const float (&r)[64], float *row, int qx0, int qx3,
                                         const float (&S)[4]) {
    constexpr int m = popc8(K);
    const float v = r[slot_of(K)] * S[m & 3];
    row[4 * K + ((m & 1) ? qx3 : qx0)] = sig1_of(K) > 0 ? v : -v;
}
template <int... K>
__device__ __forceinline__ void scatter(const float (&r)[64], float *row, int q, const float (&S)[4],
                                        std::integer_sequence<int, K...>) {
    (scatter1<K>(r, row, q, q ^ 3, S), ...);
}

// String coefficients -> matrix entries over factors 1-3 (in registers).
__device__ __forceinline__ void to_matrix3(float (&r)[64]) {
#pragma unroll
    for (int f = 0; f < 3; ++f) {
        const int tb = 5 - 2 * f, sb = 4 - 2 * f;
#pragma unroll
        for (int s = 0; s < 64; ++s) {
            if ((s >> tb) & 1) continue;
            const float p0 = r[s], p1 = r[s | 1 << tb];
            if ((s >> sb) & 1) {
                r[s] = p0 - p1;
                r[s | 1 << tb] = p0 + p1;
            } else {
                r[s] = p0 + p1;
                r[s | 1 << tb] = p0 - p1;
            }
        }
    }
}
// Matrix entries -> string coefficients over factors 1-3 (times 2 per factor).
__device__ __forceinline__ void from_matrix3(float (&r)[64]) {
#pragma unroll
    for (int f = 0; f < 3; ++f) {
        const int tb = 5 - 2 * f, sb = 4 - 2 * f;
#pragma unroll
        for (int s = 0; s < 64; ++s) {
            if ((s >> tb) & 1) continue;
            const float m0 = r[s], m1 = r[s | 1 << tb];
            r[s] = m0 + m1;
            r[s | 1 << tb] = ((s >> sb) & 1) ? m1 - m0 : m0 - m1;
        }
    }
}
// Factor 4 across the lane pair (q, q ^ 2): r += c * partner's r.
__device__ __forceinline__ void factor4(float (&r)[64], float c) {
#pragma unroll
    for (int s = 0; s < 64; ++s) r[s] = fmaf(c, __shfl_xor_sync(0xffffffffu, r[s], 2), r[s]);
}

// Store this lane's quadrant (row parity a, column parity b) into the matrix
// layout the product reads: block (row parity, column parity) of 64 floats;
// the A operand column-major within a block (columns of A contiguous), the B
// operand row-major. TRANS stores the transpose (block and entry swapped).
template <bool A_OPERAND, bool TRANS>
__device__ __forceinline__ void store_quadrant(float *mat, int a, int b, const float (&r)[64]) {
    const int blk = TRANS ? b * 2 + a : a * 2 + b;
    float *base = mat + blk * kBlockFloats;
    // entry (i, j) of the quadrant goes to base + (J_MAJOR ? j * 8 + i : i * 8 + j)
    constexpr bool J_MAJOR = A_OPERAND != TRANS;
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float4 v;
            if (J_MAJOR)  // u = j, consecutive i
                v = make_float4(r[slot_ij(4 * h + 0, u)], r[slot_ij(4 * h + 1, u)],
                                r[slot_ij(4 * h + 2, u)], r[slot_ij(4 * h + 3, u)]);
            else  // u = i, consecutive j
                v = make_float4(r[slot_ij(u, 4 * h + 0)], r[slot_ij(u, 4 * h + 1)],
                                r[slot_ij(u, 4 * h + 2)], r[slot_ij(u, 4 * h + 3)]);
            *reinterpret_cast<float4 *>(base + u * 8 + 4 * h) = v;
        }
}

// acc(i, j) = sum_k A[(i, r4)][k] B[k][(j, c4)] for this lane's quadrant.
// A_ROWMAJOR: A's blocks are stored row-major (the B-operand layout of the
// same matrix) and its columns are read with 8 strided loads.
// ACCUMULATE: add to acc instead of starting from zero.
template <bool A_ROWMAJOR = false, bool ACCUMULATE = false>
__device__ __forceinline__ void quadrant_product(float (&acc)[64], const float *A, const float *B,
                                                 int r4, int c4) {
    if (!ACCUMULATE) {
#pragma unroll
        for (int s = 0; s < 64; ++s) acc[s] = 0.0f;
    }
#pragma unroll
    for (int k4 = 0; k4 < 2; ++k4)
#pragma unroll 2
        for (int kp = 0; kp < 8; ++kp) {
            float av[8];
            if (A_ROWMAJOR) {
                const float *pa = A + (r4 * 2 + k4) * kBlockFloats + kp;
#pragma unroll
                for (int i = 0; i < 8; ++i) av[i] = pa[i * 8];
            } else {
                const float4 *pa =
                    reinterpret_cast<const float4 *>(A + (r4 * 2 + k4) * kBlockFloats + kp * 8);
                const float4 a0 = pa[0], a1 = pa[1];
                av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
                av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
            }
            const float4 *pb =
                reinterpret_cast<const float4 *>(B + (k4 * 2 + c4) * kBlockFloats + kp * 8);
            const float4 b0 = pb[0], b1 = pb[1];
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[slot_ij(i, j)] = fmaf(av[i], bv[j], acc[slot_ij(i, j)]);
        }
}

// store_quadrant with the layout chosen at run time (the two layouts the
// fused backward needs): J_MAJOR stores entry (i, j) at j * 8 + i.
__device__ __forceinline__ void store_quadrant_rt(float *mat, int blk, bool j_major,
                                                  const float (&r)[64]) {
    float *base = mat + blk * kBlockFloats;
    if (j_major) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                *reinterpret_cast<float4 *>(base + u * 8 + 4 * h) =
                    make_float4(r[slot_ij(4 * h + 0, u)], r[slot_ij(4 * h + 1, u)],
                                r[slot_ij(4 * h + 2, u)], r[slot_ij(4 * h + 3, u)]);
    } else {
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                *reinterpret_cast<float4 *>(base + u * 8 + 4 * h) =
                    make_float4(r[slot_ij(u, 4 * h + 0)], r[slot_ij(u, 4 * h + 1)],
                                r[slot_ij(u, 4 * h + 2)], r[slot_ij(u, 4 * h + 3)]);
    }
}

// out = rho^-1(op(U) op(V)): FWD U = x, V = y; GRAD_A (x = b, y = g) U = g,
// V = b transposed; GRAD_B (x = a, y = g) U = a transposed, V = g.
// One buffer per warp; the load latency of one warp's batch is hidden by the
// other warps of the SM (12 per SM; a second, prefetching buffer per warp
// halves that count and measured 20% slower).
template <int MODE>
__global__ void __launch_bounds__(32)
    gp_mat16_kernel(const float *__restrict__ x, const float *__restrict__ y,
                    float *__restrict__ out, int64_t batch, int64_t nbatches, int *err) {
    constexpr bool SWAP = MODE == CB_MODE_GRAD_A;
    constexpr bool TU = MODE == CB_MODE_GRAD_B, TV = MODE == CB_MODE_GRAD_A;
    const float *gu = SWAP ? y : x;
    const float *gv = SWAP ? x : y;
    extern __shared__ __align__(16) float sm[];
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + kBufFloats);
    const int lane = threadIdx.x, p = lane >> 2, q = lane & 3;
    const int r4 = q >> 1, c4 = r4 ^ (q & 1);
    if (lane == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
    }
    __syncwarp();
    // Lane factors: sign of the last string factor for each m mod 4, with the
    // factor-4 butterfly's lane sign folded in (forward: -1 on lane 2; inverse:
    // -1 on lane 2 and the 1/16 of the three in-register and one shuffled
    // half-steps).
    float s_in[4], s_out[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float s = (float)last_sign(q, m);
        s_in[m] = q == 2 ? -s : s;
        s_out[m] = (q == 2 ? -s : s) * 0.0625f;
    }
    const float c_fwd = r4 ? 1.0f : -1.0f;  // factor 4, forward
    const float c_inv = r4 ? -1.0f : 1.0f;  // factor 4, inverse

    bool ok = true;
    int64_t bt = blockIdx.x;
    for (int it = 0; bt < nbatches && ok; bt += gridDim.x, ++it) {
        const int64_t r0 = bt * 8;
        const int nv = (int)std::min<int64_t>(8, batch - r0);
        if (lane == 0) {
            bulk_wait_read<0>();  // the previous batch's store has read the buffer
            mbar_arrive_expect_tx(full, (uint32_t)nv * 2048u);
            for (int i = 0; i < nv; ++i) {
                bulk_load(sm + i * kRowFloats, gu + (r0 + i) * 256, 1024, full);
                bulk_load(sm + kRegion + i * kRowFloats, gv + (r0 + i) * 256, 1024, full);
            }
        }
        ok = mbar_wait_bounded(full, it & 1, err, 0x301);
        if (!__all_sync(0xffffffffu, ok)) break;
        float *U = sm + p * kRowFloats;
        float *V = U + kRegion;
        float r[64];
        // U -> op(rho(U)) as the A operand, V -> op(rho(V)) as the B operand:
        // one loop body (a single copy of the conversion code, see the fused
        // backward kernel below)
#pragma unroll 1
        for (int t = 0; t < 2; ++t) {
            float *R = t == 0 ? U : V;
            gather(r, R, q, s_in, std::make_integer_sequence<int, 64>{});
            __syncwarp();  // every lane of the product has read its row
            to_matrix3(r);
            factor4(r, c_fwd);
            const bool trans = t == 0 ? TU : TV;
            store_quadrant_rt(R, trans ? c4 * 2 + r4 : r4 * 2 + c4, t == 0 ? !TU : TV, r);
        }
        __syncwarp();
        quadrant_product(r, U, V, r4, c4);
        __syncwarp();  // all reads of the matrices done before U is overwritten
        factor4(r, c_inv);
        from_matrix3(r);
        scatter(r, U, q, s_out, std::make_integer_sequence<int, 64>{});
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            for (int i = 0; i < nv; ++i) bulk_store(out + (r0 + i) * 256, sm + i * kRowFloats, 1024);
            bulk_commit();
        }
    }
    if (lane == 0) bulk_wait_all();
}

// quadrant_product with A's layout chosen at run time.
__device__ __forceinline__ void quadrant_product_rt(float (&acc)[64], const float *A,
                                                    const float *B, int r4, int c4,
                                                    bool a_rowmajor) {
#pragma unroll
    for (int s = 0; s < 64; ++s) acc[s] = 0.0f;
#pragma unroll 1
    for (int k4 = 0; k4 < 2; ++k4)
#pragma unroll 2
        for (int kp = 0; kp < 8; ++kp) {
            float av[8];
            const float *pa = A + (r4 * 2 + k4) * kBlockFloats;
            if (a_rowmajor) {
#pragma unroll
                for (int i = 0; i < 8; ++i) av[i] = pa[kp + i * 8];
            } else {
                const float4 a0 = *reinterpret_cast<const float4 *>(pa + kp * 8);
                const float4 a1 = *reinterpret_cast<const float4 *>(pa + kp * 8 + 4);
                av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
                av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
            }
            const float4 *pb =
                reinterpret_cast<const float4 *>(B + (k4 * 2 + c4) * kBlockFloats + kp * 8);
            const float4 b0 = pb[0], b1 = pb[1];
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[slot_ij(i, j)] = fmaf(av[i], bv[j], acc[slot_ij(i, j)]);
        }
}

// ------------------------------------------------ Cl(9,0) blocks --
// The same sums for Cl(9,0) = Cl(8,0) + Cl(8,0): a 512-float block [u | v]
// (x = u + v e8) is the pair (u + v w, u - v w), w = e0 ... e7, multiplied
// componentwise; back, u = (P + Q)/2 and v = (P - Q) w / 2, which is also the
// adjoint map for the backward sums. Used by the Cl(9,0,1) product (pga10.cu).
__device__ __forceinline__ float wsign9(uint32_t j) { return (__popc(j & 0xAAu) & 1) ? -1.0f : 1.0f; }

// As gather, for component cs (+1 / -1) of the block [u | v] (optionally of
// its grade involution, folded into S and C by the caller):
//   row[idx] = u[idx] + sign_K * C * v[255 - idx]
// with the compile-time part of w(255 - idx) in sign_K and its lane part,
// the component sign and the involution's v sign in C (C0 / C3 for the two
// lane codes q, q ^ 3).
template <int K>
__device__ __forceinline__ void gather9_1(float (&r)[64], const float *u, const float *v, int qx0,
                                          int qx3, const float (&S)[4], float C0, float C3) {
    constexpr int m = popc8(K);
    constexpr int wk = popc8((~K) & 0x2A) & 1;  // bits 3, 5, 7 of ~(4K + q')
    const int idx = 4 * K + ((m & 1) ? qx3 : qx0);
    const float c = ((m & 1) ? C3 : C0) * (wk ? -1.0f : 1.0f);
    const float val = fmaf(c, v[255 - idx], u[idx]) * S[m & 3];
    r[slot_of(K)] = sig1_of(K) > 0 ? val : -val;
}
template <int... K>
__device__ __forceinline__ void gather9(float (&r)[64], const float *u, const float *v, int q,
                                        const float (&S)[4], float C0, float C3,
                                        std::integer_sequence<int, K...>) {
    (gather9_1<K>(r, u, v, q, q ^ 3, S, C0, C3), ...);
}

// One whole sum of the Cl(9,0,1) product (pga10.cu) in three stages over the
// same shared slots, 4 rows per warp and batch (product slot p = 2 * row +
// component; u of a block loads into the slot of component +, v into that of
// component -):
//   stage 0: U and V load, acc = U V;
//   stage 1: U and V load, acc += U V, then the output block h1 leaves through
//            the V slots (U keeps its converted operand);
//   stage 2: V loads, acc = U V, and the output block h2 leaves through U.
// U is the A operand's tensor (y for grad_a, x otherwise), V the other one;
// ub / vb are their blocks per stage and ug / vg whether the block's grade
// involution is used.
struct Pga10Plan {
    int ub[2], ug[2];
    int vb[3], vg[3];
    int h1, h2;
};

// In place on the output slots of a region: slot 2r holds P (component +),
// slot 2r + 1 holds Q; u = (P + Q)/2, v = (P - Q) w / 2. Lanes 8r..8r+7 take
// the blade pairs (k, ~k), so every lane reads and writes its own places.
__device__ __forceinline__ void merge9(float *region, int lane, int nv) {
    const int mrow = lane >> 3, j8 = lane & 7;
    if (mrow >= nv) return;
    float *Pz = region + (2 * mrow) * kRowFloats, *Qz = Pz + kRowFloats;
#pragma unroll 4
    for (int t = 0; t < 16; ++t) {
        const uint32_t k = j8 + 8 * t, nk = 255 - k;
        const float P = Pz[k], Q = Qz[k], Pr = Pz[nk], Qr = Qz[nk];
        Pz[k] = 0.5f * (P + Q);
        Pz[nk] = 0.5f * (Pr + Qr);
        Qz[k] = 0.5f * wsign9(nk) * (Pr - Qr);
        Qz[nk] = 0.5f * wsign9(k) * (P - Q);
    }
}

template <int MODE>
__global__ void __launch_bounds__(32, 12)
    pga10_kernel(const float *__restrict__ x, const float *__restrict__ y, float *__restrict__ out,
                 const Pga10Plan P, int64_t batch, int64_t nbatches, int *err) {
    constexpr bool SWAP = MODE == CB_MODE_GRAD_A;
    constexpr bool TU = MODE == CB_MODE_GRAD_B, TV = MODE == CB_MODE_GRAD_A;
    const float *gu = SWAP ? y : x, *gv = SWAP ? x : y;
    extern __shared__ __align__(16) float sm[];
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + kBufFloats);
    float *const RU = sm, *const RV = sm + kRegion;
    const int lane = threadIdx.x, p = lane >> 2, q = lane & 3;
    const int r4 = q >> 1, c4 = r4 ^ (q & 1);
    const int prow = p >> 1;                         // row of this slot in the batch
    const float cs = (p & 1) ? -1.0f : 1.0f;         // component
    if (lane == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
    }
    __syncwarp();
    // Lane factors (see gp_mat16_kernel), per operand with the grade
    // involution folded in: it multiplies u[idx] by (-1)^popc(idx), whose
    // parity is popc(K) + popc(q), and turns v into -g(v), i.e. flips C.
    float s_l[4], s_g[4], s_out[4];
    const int qpar = (q ^ (q >> 1)) & 1;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float s = (float)last_sign(q, m);
        const float sl = q == 2 ? -s : s;
        const float gi = ((m & 1) ^ qpar) ? -1.0f : 1.0f;
        s_l[m] = sl;
        s_g[m] = sl * gi;
        s_out[m] = sl * 0.0625f;
    }
    // lane part of w(~idx): bit 1 of ~q' (q' = q, or q ^ 3 for odd K)
    const float w0 = ((q >> 1) & 1) ? 1.0f : -1.0f, w3 = ((q >> 1) & 1) ? -1.0f : 1.0f;
    const float c_fwd = r4 ? 1.0f : -1.0f;
    const float c_inv = r4 ? -1.0f : 1.0f;
    float *const U = RU + p * kRowFloats, *const V = RV + p * kRowFloats;
    bool ok = true;
    int ph = 0;  // load rounds so far (mbarrier phase)
    for (int64_t bt = blockIdx.x; bt < nbatches && ok; bt += gridDim.x) {
        const int64_t r0 = bt * 4;
        const int nv = (int)std::min<int64_t>(4, batch - r0);
        float acc[64];
#pragma unroll 1
        for (int st = 0; st < 3; ++st, ++ph) {
            const bool loadU = st < 2;
            const int hu = st == 0 ? P.ub[0] : P.ub[1];
            const bool giu = st == 0 ? P.ug[0] : P.ug[1];
            const int hv = st == 0 ? P.vb[0] : st == 1 ? P.vb[1] : P.vb[2];
            const bool giv = st == 0 ? P.vg[0] : st == 1 ? P.vg[1] : P.vg[2];
            if (st > 0) fence_proxy_async_smem();  // earlier reads of the slots before the loads
            __syncwarp();
            if (lane == 0) {
                // stage 0: the previous batch's store from U; stage 2: this batch's from V
                if (st != 1) bulk_wait_read<0>();
                mbar_arrive_expect_tx(full, (uint32_t)nv * (loadU ? 4096u : 2048u));
                for (int i = 0; i < nv; ++i) {
                    if (loadU) {
                        const float *bu = gu + (r0 + i) * 1024 + hu * 512;
                        bulk_load(RU + (2 * i) * kRowFloats, bu, 1024, full);
                        bulk_load(RU + (2 * i + 1) * kRowFloats, bu + 256, 1024, full);
                    }
                    const float *bv = gv + (r0 + i) * 1024 + hv * 512;
                    bulk_load(RV + (2 * i) * kRowFloats, bv, 1024, full);
                    bulk_load(RV + (2 * i + 1) * kRowFloats, bv + 256, 1024, full);
                }
            }
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(full, ph & 1, err, 0x311));
            if (!ok) break;
            float r[64];
#pragma unroll 1
            for (int t = loadU ? 0 : 1; t < 2; ++t) {
                const float *raw = (t == 0 ? RU : RV) + (2 * prow) * kRowFloats;
                const bool gi = t == 0 ? giu : giv;
                const float c = gi ? -cs : cs;
                gather9(r, raw, raw + kRowFloats, q, gi ? s_g : s_l, c * w0, c * w3,
                        std::make_integer_sequence<int, 64>{});
                __syncwarp();  // both components of the row have read the raw block
                to_matrix3(r);
                factor4(r, c_fwd);
                const bool trans = t == 0 ? TU : TV;
                store_quadrant_rt(t == 0 ? U : V, trans ? c4 * 2 + r4 : r4 * 2 + c4,
                                  t == 0 ? !TU : TV, r);
            }
            __syncwarp();
            if (st == 1)
                quadrant_product<false, true>(acc, U, V, r4, c4);
            else
                quadrant_product(acc, U, V, r4, c4);
            __syncwarp();
            if (st == 0) continue;
            // an output block leaves: through V after stage 1, through U after stage 2
            float *region = st == 1 ? RV : RU;
            factor4(acc, c_inv);
            from_matrix3(acc);
            scatter(acc, region + p * kRowFloats, q, s_out, std::make_integer_sequence<int, 64>{});
            __syncwarp();
            merge9(region, lane, nv);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                const int h = st == 1 ? P.h1 : P.h2;
                for (int i = 0; i < nv; ++i) {
                    float *o = out + (r0 + i) * 1024 + h * 512;
                    bulk_store(o, region + (2 * i) * kRowFloats, 1024);
                    bulk_store(o + 256, region + (2 * i + 1) * kRowFloats, 1024);
                }
                bulk_commit();
            }
        }
    }
    if (lane == 0) bulk_wait_all();
}

template <int MODE>
int launch_pga10(const float *x, const float *y, float *out, const Pga10Plan &P, int64_t batch,
                 cudaStream_t s) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    auto kern = pga10_kernel<MODE>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pga10)");
    int ps = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ps, kern, 32, kSmemBytes) != cudaSuccess ||
        ps < 1) {
        cudaGetLastError();
        ps = 1;
    }
    const int64_t nb = (batch + 3) / 4;
    const int grid = (int)std::min<int64_t>(nb, (int64_t)ps * di.sm_count);
    kern<<<grid, 32, kSmemBytes, s>>>(x, y, out, P, batch, nb, err);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch pga10_kernel");
}

// Both backward sums in one pass over a, b, g (5 KB per product instead of 6 KB
// for two launches), in two phases that run the same code:
//   phase 0: a and g load; rho(a)^T (the A operand) and rho(g) (the B
//            operand, row-major) are formed; grad_b = rho^-1(rho(a)^T rho(g));
//   phase 1: b loads into a's region once grad_b has left it; rho(b)^T is
//            formed; grad_a = rho^-1(rho(g) rho(b)^T), reading the columns of
//            rho(g) from its row-major copy.
// The phases and their input conversions are loops, not unrolled copies: the
// eleven warps of an SM run at different points of the kernel, and one copy
// of each piece keeps the instruction working set small. Two regions per
// product: 12 CTAs per SM (against 8 with all three rows resident).
__global__ void __launch_bounds__(32)
    gp_mat16_bwd_kernel(const float *__restrict__ a, const float *__restrict__ b,
                        const float *__restrict__ g, float *__restrict__ ga,
                        float *__restrict__ gb, int64_t batch, int64_t nbatches, int *err) {
    extern __shared__ __align__(16) float sm[];
    float *const RA = sm, *const RG = sm + kRegion;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + 2 * kRegion);
    const int lane = threadIdx.x, p = lane >> 2, q = lane & 3;
    const int r4 = q >> 1, c4 = r4 ^ (q & 1);
    if (lane == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
    }
    __syncwarp();
    float s_in[4], s_out[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float s = (float)last_sign(q, m);
        s_in[m] = q == 2 ? -s : s;
        s_out[m] = (q == 2 ? -s : s) * 0.0625f;
    }
    const float c_fwd = r4 ? 1.0f : -1.0f;
    const float c_inv = r4 ? -1.0f : 1.0f;
    float *const A = RA + p * kRowFloats, *const G = RG + p * kRowFloats;
    bool ok = true;
    uint32_t ph_count = 0;  // completed phases of `full`
    for (int64_t bt = blockIdx.x; bt < nbatches && ok; bt += gridDim.x) {
        const int64_t r0 = bt * 8;
        const int nv = (int)std::min<int64_t>(8, batch - r0);
#pragma unroll 1
        for (int ph = 0; ph < 2; ++ph) {
            if (lane == 0) {
                bulk_wait_read<0>();  // earlier stores have read region A
                mbar_arrive_expect_tx(full, (uint32_t)nv * (ph == 0 ? 2048u : 1024u));
                for (int i = 0; i < nv; ++i) {
                    bulk_load(RA + i * kRowFloats, (ph == 0 ? a : b) + (r0 + i) * 256, 1024, full);
                    if (ph == 0) bulk_load(RG + i * kRowFloats, g + (r0 + i) * 256, 1024, full);
                }
            }
            ok = mbar_wait_bounded(full, ph_count++ & 1, err, ph == 0 ? 0x302 : 0x304);
            if (!__all_sync(0xffffffffu, ok)) break;
            float r[64];
#pragma unroll 1
            for (int t = 0; t < (ph == 0 ? 2 : 1); ++t) {
                // phase 0: a -> rho(a)^T (A operand), g -> rho(g) (B operand);
                // phase 1: b -> rho(b)^T (B operand)
                float *R = t == 1 ? G : A;
                gather(r, R, q, s_in, std::make_integer_sequence<int, 64>{});
                __syncwarp();  // every lane of the product has read its row
                to_matrix3(r);
                factor4(r, c_fwd);
                const bool trans = (t == 0);
                store_quadrant_rt(R, trans ? c4 * 2 + r4 : r4 * 2 + c4, ph == 1, r);
            }
            __syncwarp();
            quadrant_product_rt(r, ph == 0 ? A : G, ph == 0 ? G : A, r4, c4, ph == 1);
            __syncwarp();  // all reads of the matrices done before A is overwritten
            factor4(r, c_inv);
            from_matrix3(r);
            scatter(r, A, q, s_out, std::make_integer_sequence<int, 64>{});
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                float *out = ph == 0 ? gb : ga;
                for (int i = 0; i < nv; ++i)
                    bulk_store(out + (r0 + i) * 256, RA + i * kRowFloats, 1024);
                bulk_commit();
            }
        }
    }
    if (lane == 0) bulk_wait_all();
}

// ------------------------------------------------ GP layer of Cl(8,0) --
// y = x * w with one weight row for the batch (reference layers.py:43-47) is
// rho(y) = rho(x) W with W = rho(w): per row one 16 x 16 x 16 product with a
// fixed matrix. Backward: dx = rho^-1(rho(dy) W^T) and, rho / 4 being an
// isometry, dw = rho^-1(sum over rows of rho(x)^T rho(dy)).
// Weight operands (mats): W and W^T, each as the B operand in the padded
// block layout of the shared tiles (4 blocks of kBlockFloats floats).
constexpr int kWFloats = 4 * kBlockFloats;
static_assert(kWFloats == kGpLayerWFloats, "weight operand size");

__device__ __forceinline__ void lane_signs(int q, float (&s_in)[4], float (&s_out)[4]) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float s = (float)last_sign(q, m);
        s_in[m] = q == 2 ? -s : s;
        s_out[m] = (q == 2 ? -s : s) * 0.0625f;
    }
}

// One warp: lanes 0-3 convert w (lanes 4-31 repeat the work on the same row
// so that the shuffles stay full-warp) and write W and W^T.
__global__ void __launch_bounds__(32) gp_layer_weight_kernel(const float *__restrict__ w,
                                                             float *__restrict__ mats) {
    const int lane = threadIdx.x, q = lane & 3, r4 = q >> 1, c4 = r4 ^ (q & 1);
    float s_in[4], s_out[4];
    lane_signs(q, s_in, s_out);
    float r[64];
    gather(r, w, q, s_in, std::make_integer_sequence<int, 64>{});
    to_matrix3(r);
    factor4(r, r4 ? 1.0f : -1.0f);
    if (lane < 4) {
        store_quadrant<false, false>(mats, r4, c4, r);
        store_quadrant<false, true>(mats + kWFloats, r4, c4, r);
    }
}

// out = rho^-1(rho(in) wm), wm a B operand (W for y, W^T for dx).
__global__ void __launch_bounds__(32)
    gp_layer_apply_kernel(const float *__restrict__ in, float *__restrict__ out,
                          const float *__restrict__ wm, int64_t batch, int64_t nbatches, int *err) {
    extern __shared__ __align__(16) float sm[];
    float *const WM = sm, *const RX = sm + kWFloats;
    uint64_t *full = reinterpret_cast<uint64_t *>(RX + kRegion);
    const int lane = threadIdx.x, p = lane >> 2, q = lane & 3;
    const int r4 = q >> 1, c4 = r4 ^ (q & 1);
    for (int e = lane; e < kWFloats; e += 32) WM[e] = wm[e];
    if (lane == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
    }
    __syncwarp();
    float s_in[4], s_out[4];
    lane_signs(q, s_in, s_out);
    const float c_fwd = r4 ? 1.0f : -1.0f, c_inv = r4 ? -1.0f : 1.0f;
    bool ok = true;
    int64_t bt = blockIdx.x;
    for (int it = 0; bt < nbatches && ok; bt += gridDim.x, ++it) {
        const int64_t r0 = bt * 8;
        const int nv = (int)std::min<int64_t>(8, batch - r0);
        if (lane == 0) {
            bulk_wait_read<0>();
            mbar_arrive_expect_tx(full, (uint32_t)nv * 1024u);
            for (int i = 0; i < nv; ++i) bulk_load(RX + i * kRowFloats, in + (r0 + i) * 256, 1024, full);
        }
        ok = mbar_wait_bounded(full, it & 1, err, 0x311);
        if (!__all_sync(0xffffffffu, ok)) break;
        float *X = RX + p * kRowFloats;
        float r[64];
        gather(r, X, q, s_in, std::make_integer_sequence<int, 64>{});
        __syncwarp();
        to_matrix3(r);
        factor4(r, c_fwd);
        store_quadrant<true, false>(X, r4, c4, r);
        __syncwarp();
        quadrant_product(r, X, WM, r4, c4);
        __syncwarp();
        factor4(r, c_inv);
        from_matrix3(r);
        scatter(r, X, q, s_out, std::make_integer_sequence<int, 64>{});
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            for (int i = 0; i < nv; ++i) bulk_store(out + (r0 + i) * 256, RX + i * kRowFloats, 1024);
            bulk_commit();
        }
    }
    if (lane == 0) bulk_wait_all();
}

// Per CTA: sum over the CTA's rows of rho(x)^T rho(dy), written as a
// row-major 16 x 16 partial at partial[blockIdx.x * 256] (the 8 product
// slots of the warp are summed by shuffles at the end).
__global__ void __launch_bounds__(32)
    gp_layer_dw_kernel(const float *__restrict__ x, const float *__restrict__ dy,
                       float *__restrict__ partial, int64_t batch, int64_t nbatches, int *err) {
    extern __shared__ __align__(16) float sm[];
    float *const RX = sm, *const RG = sm + kRegion;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + 2 * kRegion);
    const int lane = threadIdx.x, p = lane >> 2, q = lane & 3;
    const int r4 = q >> 1, c4 = r4 ^ (q & 1);
    if (lane == 0) {
        mbar_init(full, 1);
        fence_barrier_init();
    }
    __syncwarp();
    float s_in[4], s_out[4];
    lane_signs(q, s_in, s_out);
    const float c_fwd = r4 ? 1.0f : -1.0f;
    float acc[64];
#pragma unroll
    for (int s = 0; s < 64; ++s) acc[s] = 0.0f;
    bool ok = true;
    int64_t bt = blockIdx.x;
    for (int it = 0; bt < nbatches && ok; bt += gridDim.x, ++it) {
        const int64_t r0 = bt * 8;
        const int nv = (int)std::min<int64_t>(8, batch - r0);
        if (lane == 0) {
            bulk_wait_read<0>();
            mbar_arrive_expect_tx(full, (uint32_t)nv * 2048u);
            for (int i = 0; i < nv; ++i) {
                bulk_load(RX + i * kRowFloats, x + (r0 + i) * 256, 1024, full);
                bulk_load(RG + i * kRowFloats, dy + (r0 + i) * 256, 1024, full);
            }
        }
        ok = mbar_wait_bounded(full, it & 1, err, 0x312);
        if (!__all_sync(0xffffffffu, ok)) break;
        float *X = RX + p * kRowFloats, *G = RG + p * kRowFloats;
        const bool valid = p < nv;  // slots past the end of the batch add nothing
        float r[64];
        gather(r, X, q, s_in, std::make_integer_sequence<int, 64>{});
        __syncwarp();
        to_matrix3(r);
        factor4(r, c_fwd);
        if (!valid) {
#pragma unroll
            for (int s = 0; s < 64; ++s) r[s] = 0.0f;
        }
        store_quadrant<true, true>(X, r4, c4, r);  // rho(x)^T as the A operand
        gather(r, G, q, s_in, std::make_integer_sequence<int, 64>{});
        __syncwarp();
        to_matrix3(r);
        factor4(r, c_fwd);
        if (!valid) {  // stale shared memory may hold non-finite values: zero both operands
#pragma unroll
            for (int s = 0; s < 64; ++s) r[s] = 0.0f;
        }
        store_quadrant<false, false>(G, r4, c4, r);  // rho(dy) as the B operand
        __syncwarp();
        quadrant_product<false, true>(acc, X, G, r4, c4);
        __syncwarp();
    }
#pragma unroll
    for (int s = 0; s < 64; ++s)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) acc[s] += __shfl_xor_sync(0xffffffffu, acc[s], o);
    if (p == 0) {
        // entry (i, j) of quadrant (r4, c4) is matrix entry (2i + r4, 2j + c4)
        float *dst = partial + (size_t)blockIdx.x * 256;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[(2 * i + r4) * 16 + 2 * j + c4] = acc[slot_ij(i, j)];
    }
}

// dW = sum of the partials (fp64), then dw = rho^-1(dW) by warp 0.
__global__ void __launch_bounds__(256)
    gp_layer_dw_finish_kernel(const float *__restrict__ partial, int nparts, float *__restrict__ dw) {
    __shared__ float W[256];
    {
        const int e = threadIdx.x;
        double s = 0.0;
        for (int k = 0; k < nparts; ++k) s += (double)partial[(size_t)k * 256 + e];
        W[e] = (float)s;
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x, q = lane & 3, r4 = q >> 1, c4 = r4 ^ (q & 1);
    float s_in[4], s_out[4];
    lane_signs(q, s_in, s_out);
    float r[64];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) r[slot_ij(i, j)] = W[(2 * i + r4) * 16 + 2 * j + c4];
    factor4(r, r4 ? -1.0f : 1.0f);
    from_matrix3(r);
    if (lane < 4) scatter(r, dw, q, s_out, std::make_integer_sequence<int, 64>{});
}

int occupancy_grid(const void *kern, int smem, int64_t nbatches, const DeviceInfo &di) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32, smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    return (int)std::max<int64_t>(1, std::min<int64_t>(nbatches, (int64_t)per_sm * di.sm_count));
}

template <int MODE>
int launch_mat16(const float *x, const float *y, float *out, int64_t batch, cudaStream_t s) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    auto kern = gp_mat16_kernel<MODE>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gp_mat16)");
    static int per_sm[3] = {0, 0, 0};
    int &ps = per_sm[MODE];
    if (ps == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ps, kern, 32, kSmemBytes) != cudaSuccess ||
            ps < 1) {
            cudaGetLastError();
            ps = 1;
        }
    }
    const int64_t nb = (batch + 7) / 8;
    const int grid = (int)std::min<int64_t>(nb, (int64_t)ps * di.sm_count);
    kern<<<grid, 32, kSmemBytes, s>>>(x, y, out, batch, nb, err);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gp_mat16_kernel");
}

}  // namespace

bool use_mat16(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
               const void *o) {
    if (op != CB_OP_GP || n != 8 || neg || zero) return false;
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return al(x) && al(y) && al(o);
}

int gp_mat16(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s) {
    if (batch == 0) return CB_OK;
    switch (mode) {
    case CB_MODE_FWD: return launch_mat16<CB_MODE_FWD>(x, y, out, batch, s);
    case CB_MODE_GRAD_A: return launch_mat16<CB_MODE_GRAD_A>(x, y, out, batch, s);
    default: return launch_mat16<CB_MODE_GRAD_B>(x, y, out, batch, s);
    }
}

int gp_mat16_bwd(const float *a, const float *b, const float *g, float *ga, float *gb,
                 int64_t batch, cudaStream_t s) {
    if (batch == 0) return CB_OK;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    constexpr int kBwdSmem = 2 * kRegion * 4 + 64;
    auto kern = gp_mat16_bwd_kernel;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gp_mat16_bwd)");
    static int per_sm = 0;
    if (per_sm == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32, kBwdSmem) != cudaSuccess ||
            per_sm < 1) {
            cudaGetLastError();
            per_sm = 1;
        }
    }
    const int64_t nb = (batch + 7) / 8;
    const int grid = (int)std::min<int64_t>(nb, (int64_t)per_sm * di.sm_count);
    kern<<<grid, 32, kBwdSmem, s>>>(a, b, g, ga, gb, batch, nb, err);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gp_mat16_bwd_kernel");
}

constexpr int kApplySmem = (kWFloats + kRegion) * 4 + 64;
constexpr int kDwSmem = 2 * kRegion * 4 + 64;

int gp_layer_apply(const float *wm, const float *in, float *out, int64_t batch, cudaStream_t s) {
    if (batch == 0) return CB_OK;
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    static int grid_cap = 0;
    if (grid_cap == 0) grid_cap = occupancy_grid((const void *)gp_layer_apply_kernel, kApplySmem, 1 << 30, di);
    const int64_t nb = (batch + 7) / 8;
    const int grid = (int)std::min<int64_t>(nb, grid_cap);
    gp_layer_apply_kernel<<<grid, 32, kApplySmem, s>>>(in, out, wm, batch, nb, err);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gp_layer_apply_kernel");
}

int gp_layer_dw_parts(int64_t batch) {
    DeviceInfo di;
    if (device_info(&di)) return -1;
    static int grid_cap = 0;
    if (grid_cap == 0) grid_cap = occupancy_grid((const void *)gp_layer_dw_kernel, kDwSmem, 1 << 30, di);
    const int64_t nb = std::max<int64_t>(1, (batch + 7) / 8);
    return (int)std::min<int64_t>(nb, grid_cap);
}

int gp_layer_dw(const float *x, const float *dy, float *dw, float *partial, int64_t batch,
                cudaStream_t s) {
    int *err = nullptr;
    int st = device_error_word(&err);
    if (st) return st;
    const int parts = gp_layer_dw_parts(batch);
    if (parts <= 0) return cuda_fail(cudaGetLastError(), "gp layer dw sizing");
    const int64_t nb = (batch + 7) / 8;
    cudaError_t e = cudaSuccess;
    if (batch > 0)
        gp_layer_dw_kernel<<<parts, 32, kDwSmem, s>>>(x, dy, partial, batch, nb, err);
    else
        e = cudaMemsetAsync(partial, 0, (size_t)parts * 256 * sizeof(float), s);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch gp_layer_dw_kernel");
    gp_layer_dw_finish_kernel<<<1, 256, 0, s>>>(partial, parts, dw);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gp_layer_dw_finish_kernel");
}

int gp_layer_weight(const float *w, float *mats, cudaStream_t s) {
    gp_layer_weight_kernel<<<1, 32, 0, s>>>(w, mats);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch gp_layer_weight_kernel");
}

// One sum of the Cl(9,0,1) product (see pga10_kernel); mode and (x, y) as in
// cb_bilinear. The stage plans (blocks and involutions per stage, output
// blocks): forward (x = a, y = b) c1 = a1 g(b0) + a0 b1, then c0 = a0 b0;
// grad_a (x = b, y = g; U = g) ga0 = gA(b0; g0) + gA(b1; g1), then
// ga1 = gA(g(b0); g1); grad_b (x = a, y = g; U = a) gb0 = gB(g(a1); g(g1)) +
// gB(a0; g0), then gb1 = gB(a0; g1).
int pga10_sum(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s) {
    switch (mode) {
    case CB_MODE_FWD: {
        const Pga10Plan P{{1, 0}, {0, 0}, {0, 1, 0}, {1, 0, 0}, 1, 0};
        return launch_pga10<CB_MODE_FWD>(x, y, out, P, batch, s);
    }
    case CB_MODE_GRAD_A: {
        const Pga10Plan P{{0, 1}, {0, 0}, {0, 1, 0}, {0, 0, 1}, 0, 1};
        return launch_pga10<CB_MODE_GRAD_A>(x, y, out, P, batch, s);
    }
    default: {
        const Pga10Plan P{{1, 0}, {1, 0}, {1, 0, 1}, {1, 0, 0}, 0, 1};
        return launch_pga10<CB_MODE_GRAD_B>(x, y, out, P, batch, s);
    }
    }
}

}  // namespace cb
