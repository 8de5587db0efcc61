// rotor.cu -- learnable rotors: compile a bivector into the blade-minor
// matrices of its rotation, apply the sandwich R~ x R, and the backward pass
// to x and to the bivector.
//
// Reference path (CliffordCUDA): compile_bivector (algebra.py:343-352) builds
// Rm = expm(B), B = 2 (M - M^T), M[p][q] = beta_pq (p < q, lex order,
// algebra.py:127) through linalg_eigh and a closed form (eigh_exp.cu:270-322),
// factors Rm into C(n,2) Givens rotations (givens_factor.cu:7-59) and applies
// the rotation chain to every multivector (givens_apply_mb_perm_packed.cu:8-70).
// The chain composes to the outermorphism of Rm^T:
//     y[J] = sum_{|I| = |J|} det(Rm[I, J]) x[I]
// (rows I and columns J in increasing generator order). The metric is not used,
// as in the reference. This file evaluates that map directly:
//
//   compile:  fp64 -- Rm by scaling and squaring of a Taylor series
//             (||B / 2^s||_1 <= 1/8, 20 terms), then every equal-grade minor
//             C_k[I][J] = det(Rm[I, J]) by Gaussian elimination with partial
//             pivoting, spread over CTAs that each recompute Rm. Per grade
//             k the C(n,k) x C(n,k) matrix is stored
//             row-major, grades concatenated (C(2n, n) entries in total).
//   apply:    y = x C_full with C_full the D x D matrix holding every C_k at
//             its blades' (bit-pattern) positions and zeros between grades;
//             for n = 7, 8 this runs on the tensor cores as the 3xTF32
//             tcgen05 GEMM of layer_gemm.cu, whose tf32 hi/lo operands
//             (C_full and its transpose) the compile step appends to cs.
//             Other n use a generic kernel.
//   backward: dx = g C_full^T by the same GEMM, and dC_k = x_k^T g_k gathered
//             from G = x^T g (the split-K tensor-core GEMM, partials summed in
//             double). The no-allocation variant instead runs a fused
//             CUDA-core pass (dx and per-CTA partial sums of dC) over a fixed
//             in-library array. The chain to the
//             bivector runs in one 1024-thread CTA in fp64 (one warp per
//             entry of dRm, no atomics):
//               dRm[p][q] = sum_{I, J} dC[I][J] (-1)^(a+b) det(Rm[I\p, J\q])
//             (a, b = positions of p in I and q in J; the cofactors are the
//             grade k-1 minors already computed), then the adjoint Frechet
//             derivative of expm, dB = L(B^T, dRm), read off the upper-right
//             block of expm([[B^T, dRm], [0, B^T]]), and
//             dbeta_pq = 2 (dB[p][q] - dB[q][p]).
//             The reference returned no gradient for x
//             (mb_perm_packed.py:42); this path does.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace cb {
namespace {

constexpr int kMaxN = 10;  // blade tables of 2^n ints live in static shared memory

__host__ __device__ inline int binom(int n, int k) {
    if (k < 0 || k > n) return 0;
    int r = 1;
    for (int i = 1; i <= k; ++i) r = r * (n - k + i) / i;
    return r;
}

// Per-n layout of the compiled rotor. cs holds the grade blocks (total
// entries) followed, for the tensor-core sizes, by the GEMM operands
// [C_full^T hi | C_full^T lo | C_full hi | C_full lo] (4 D^2 entries) from
// mats_off on.
struct Layout {
    int n, D;
    int ck[kMaxN + 1];       // C(n, k)
    int goff[kMaxN + 2];     // first grade-sorted index of grade k
    int coff[kMaxN + 2];     // first matrix entry of grade k (sum of C(n,j)^2)
    int padoff[kMaxN + 2];   // first slot of grade k in a 4-padded sorted row
    int total, rowlen;
    bool tensor;             // n = 7, 8: apply and backward on the tensor cores
    int mats_off;            // first GEMM operand entry (256-byte aligned for TMA)
    int64_t cs_floats;       // mats_off + 4 D^2, or total
};

__host__ __device__ inline Layout make_layout(int n) {
    Layout L{};
    L.n = n;
    L.D = 1 << n;
    L.goff[0] = L.coff[0] = L.padoff[0] = 0;
    for (int k = 0; k <= n; ++k) {
        L.ck[k] = binom(n, k);
        L.goff[k + 1] = L.goff[k] + L.ck[k];
        L.coff[k + 1] = L.coff[k] + L.ck[k] * L.ck[k];
        L.padoff[k + 1] = L.padoff[k] + ((L.ck[k] + 3) & ~3);
    }
    L.total = L.coff[n + 1];
    L.rowlen = L.padoff[n + 1];
    L.tensor = (n == 7 || n == 8);
    L.mats_off = (L.total + 63) & ~63;
    L.cs_floats = L.tensor ? L.mats_off + 4 * (int64_t)L.D * L.D : L.total;
    return L;
}

// Rank of blade bp among the blades of its grade in increasing order
// (colexicographic rank of its set of generators), and the inverse.
__host__ __device__ inline int blade_rank(uint32_t bp) {
    int r = 0, i = 0;
    for (int c = 0; bp; ++c, bp >>= 1)
        if (bp & 1u) r += binom(c, ++i);
    return r;
}

__host__ __device__ inline uint32_t blade_unrank(int n, int k, int r) {
    uint32_t bp = 0;
    for (int c = n - 1; c >= 0 && k > 0; --c) {
        const int b = binom(c, k);
        if (b <= r) {
            bp |= 1u << c;
            r -= b;
            --k;
        }
    }
    return bp;
}

__device__ inline int popc(uint32_t v) { return __popc(v); }

// Fills, for every blade bp: rank[bp] (position among blades of its grade in
// increasing order) and blades[goff[k] + rank] = bp.
__device__ void build_blade_tables(const Layout &L, int *rank, int *blades) {
    if (threadIdx.x == 0) {
        int cnt[kMaxN + 1];
        for (int k = 0; k <= L.n; ++k) cnt[k] = 0;
        for (int bp = 0; bp < L.D; ++bp) {
            const int k = popc(bp);
            rank[bp] = cnt[k];
            blades[L.goff[k] + cnt[k]] = bp;
            ++cnt[k];
        }
    }
    __syncthreads();
}

// C = A * B for n x n row-major fp64 matrices in shared memory (all threads).
__device__ void mat_mul(int n, const double *A, const double *B, double *C) {
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
        const int i = e / n, j = e % n;
        double s = 0.0;
        for (int k = 0; k < n; ++k) s += A[i * n + k] * B[k * n + j];
        C[e] = s;
    }
    __syncthreads();
}

// E = expm(A) for an m x m fp64 matrix in shared memory; T, W are scratch.
// Scaling and squaring: A / 2^s with ||A / 2^s||_1 <= 1/8, Taylor to degree 20.
__device__ void expm(int m, double *A, double *E, double *T, double *W) {
    __shared__ int s_sh;
    __shared__ double scale_sh;
    if (threadIdx.x == 0) {
        double nrm = 0.0;
        for (int j = 0; j < m; ++j) {
            double c = 0.0;
            for (int i = 0; i < m; ++i) c += fabs(A[i * m + j]);
            nrm = fmax(nrm, c);
        }
        int s = 0;
        while (nrm > 0.125 && s < 60) {
            nrm *= 0.5;
            ++s;
        }
        s_sh = s;
        scale_sh = ldexp(1.0, -s);
    }
    __syncthreads();
    const int s = s_sh;
    const double scale = scale_sh;
    for (int e = threadIdx.x; e < m * m; e += blockDim.x) {
        A[e] *= scale;
        const double id = (e / m == e % m) ? 1.0 : 0.0;
        E[e] = id;
        T[e] = id;
    }
    __syncthreads();
    for (int k = 1; k <= 20; ++k) {
        mat_mul(m, T, A, W);
        for (int e = threadIdx.x; e < m * m; e += blockDim.x) {
            T[e] = W[e] / (double)k;
            E[e] += T[e];
        }
        __syncthreads();
    }
    for (int k = 0; k < s; ++k) {
        mat_mul(m, E, E, W);
        for (int e = threadIdx.x; e < m * m; e += blockDim.x) E[e] = W[e];
        __syncthreads();
    }
}

// det of the k x k matrix Rm[I rows, J cols] (generators in increasing order).
__device__ double minor_det(int n, const double *Rm, uint32_t I, uint32_t J, int k) {
    if (k == 0) return 1.0;
    double A[kMaxN * kMaxN];
    int ri[kMaxN], ci[kMaxN];
    int a = 0, b = 0;
    for (int t = 0; t < n; ++t) {
        if ((I >> t) & 1u) ri[a++] = t;
        if ((J >> t) & 1u) ci[b++] = t;
    }
    for (int r = 0; r < k; ++r)
        for (int c = 0; c < k; ++c) A[r * k + c] = Rm[ri[r] * n + ci[c]];
    double det = 1.0;
    for (int c = 0; c < k; ++c) {
        int piv = c;
        for (int r = c + 1; r < k; ++r)
            if (fabs(A[r * k + c]) > fabs(A[piv * k + c])) piv = r;
        const double pv = A[piv * k + c];
        if (pv == 0.0) return 0.0;
        if (piv != c) {
            for (int t = 0; t < k; ++t) {
                const double tmp = A[c * k + t];
                A[c * k + t] = A[piv * k + t];
                A[piv * k + t] = tmp;
            }
            det = -det;
        }
        det *= pv;
        for (int r = c + 1; r < k; ++r) {
            const double f = A[r * k + c] / pv;
            for (int t = c + 1; t < k; ++t) A[r * k + t] -= f * A[c * k + t];
        }
    }
    return det;
}

// State (fp64) layout: Bm [n*n], Rm [n*n], C64 [total].
// Each CTA computes Rm = expm(B) itself (a few microseconds at n <= 10) and
// then the minors e = blockIdx.x * 256 + threadIdx.x, ... of its slice; CTA 0
// also stores B and Rm.
__global__ void __launch_bounds__(256)
    rotor_compile_kernel(const float *__restrict__ beta, int n, float *__restrict__ cs,
                         double *__restrict__ state) {
    const Layout L = make_layout(n);
    __shared__ double Bm[kMaxN * kMaxN], Rm[kMaxN * kMaxN], T[kMaxN * kMaxN],
        W[kMaxN * kMaxN];
    __shared__ int rank[1 << kMaxN], blades[1 << kMaxN];
    const int nn = n * n;
    for (int e = threadIdx.x; e < nn; e += blockDim.x) Bm[e] = 0.0;
    __syncthreads();
    if (threadIdx.x == 0) {
        int idx = 0;
        for (int p = 0; p < n - 1; ++p)
            for (int q = p + 1; q < n; ++q, ++idx) {
                Bm[p * n + q] = 2.0 * (double)beta[idx];
                Bm[q * n + p] = -2.0 * (double)beta[idx];
            }
    }
    __syncthreads();
    if (blockIdx.x == 0)
        for (int e = threadIdx.x; e < nn; e += blockDim.x) state[e] = Bm[e];  // B (unscaled)
    __syncthreads();
    expm(n, Bm, Rm, T, W);
    if (blockIdx.x == 0)
        for (int e = threadIdx.x; e < nn; e += blockDim.x) state[nn + e] = Rm[e];
    build_blade_tables(L, rank, blades);
    double *C64 = state + 2 * nn;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < L.total; e += gridDim.x * blockDim.x) {
        int k = 0;
        while (e >= L.coff[k + 1]) ++k;
        const int ck = L.ck[k];
        const int ir = (e - L.coff[k]) / ck, jr = (e - L.coff[k]) % ck;
        const double v = minor_det(n, Rm, blades[L.goff[k] + ir], blades[L.goff[k] + jr], k);
        C64[e] = v;
        cs[e] = (float)v;
    }
}

// C_full[I][J] = C_k[rank I][rank J] for |I| = |J| = k, else 0 (into `M`).
__global__ void rotor_full_matrix_kernel(const float *__restrict__ cs, int n,
                                         float *__restrict__ M) {
    const Layout L = make_layout(n);
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= L.D * L.D) return;
    const uint32_t I = e / L.D, J = e % L.D;
    const int k = __popc(I);
    float v = 0.0f;
    if (k == __popc(J)) v = cs[L.coff[k] + blade_rank(I) * L.ck[k] + blade_rank(J)];
    M[e] = v;
}

// dcs[e] = G[I][J] for every grade-block entry e = (k, rank I, rank J).
__global__ void rotor_gather_dc_kernel(const float *__restrict__ G, int n,
                                       float *__restrict__ dcs) {
    const Layout L = make_layout(n);
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= L.total) return;
    int k = 0;
    while (e >= L.coff[k + 1]) ++k;
    const int ck = L.ck[k];
    const uint32_t I = blade_unrank(n, k, (e - L.coff[k]) / ck);
    const uint32_t J = blade_unrank(n, k, (e - L.coff[k]) % ck);
    dcs[e] = G[(size_t)I * L.D + J];
}

// --------------------------------------------------- backward (fast, fused) --
// dx = g C^T per grade and per-CTA partial dC = x^T g (per grade) into
// partial[blockIdx.x][entry].
template <int N>
__global__ void __launch_bounds__(1 << N)
    rotor_bwd_kernel(const float *__restrict__ cs, const float *__restrict__ x,
                     const float *__restrict__ g, float *__restrict__ dx,
                     float *__restrict__ partial, int64_t batch) {
    constexpr int D = 1 << N;
    constexpr int MAXC = (N == 7) ? 35 : 70;
    constexpr int R = 16;
    const Layout L = make_layout(N);
    extern __shared__ float sm[];
    float *xs = sm;                    // [R][rowlen]
    float *gs = sm + R * L.rowlen;     // [R][rowlen]
    float *ds = gs + R * L.rowlen;     // [R][D]
    __shared__ int rank[D], blades[D];
    build_blade_tables(L, rank, blades);

    const int t = threadIdx.x;  // grade-sorted index u of this thread
    int k = 0;
    while (t >= L.goff[k + 1]) ++k;
    const int ck = L.ck[k];
    const int u = t - L.goff[k];
    const int pk = (ck + 3) & ~3;
    const int off = L.padoff[k];
    const int out_bp = blades[t];
    constexpr int NREG = (MAXC + 3) / 4 * 4;
    float crow[NREG], dacc[NREG];
#pragma unroll
    for (int s = 0; s < NREG; ++s) {
        crow[s] = (s < ck) ? cs[L.coff[k] + u * ck + s] : 0.0f;  // row u of C_k
        dacc[s] = 0.0f;
    }
    const int in_slot = L.padoff[popc(t)] + rank[t];
    const int my_slot = off + u;
    for (int e = t; e < 2 * R * L.rowlen; e += D) xs[e] = 0.0f;
    __syncthreads();

    for (int64_t row0 = (int64_t)blockIdx.x * R; row0 < batch; row0 += (int64_t)gridDim.x * R) {
#pragma unroll 4
        for (int r = 0; r < R; ++r) {
            const int64_t row = row0 + r;
            const bool ok = row < batch;
            xs[r * L.rowlen + in_slot] = ok ? x[row * D + t] : 0.0f;
            gs[r * L.rowlen + in_slot] = ok ? g[row * D + t] : 0.0f;
        }
        __syncthreads();
#pragma unroll 1
        for (int r0 = 0; r0 < R; r0 += 4) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            float gu[4];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) gu[rr] = gs[(r0 + rr) * L.rowlen + my_slot];
#pragma unroll
            for (int q = 0; q < (MAXC + 3) / 4; ++q) {
                if (4 * q < pk) {
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        const float4 gv =
                            *reinterpret_cast<const float4 *>(gs + (r0 + rr) * L.rowlen + off + 4 * q);
                        const float4 xv =
                            *reinterpret_cast<const float4 *>(xs + (r0 + rr) * L.rowlen + off + 4 * q);
                        acc[rr] = fmaf(crow[4 * q + 0], gv.x, acc[rr]);
                        acc[rr] = fmaf(crow[4 * q + 1], gv.y, acc[rr]);
                        acc[rr] = fmaf(crow[4 * q + 2], gv.z, acc[rr]);
                        acc[rr] = fmaf(crow[4 * q + 3], gv.w, acc[rr]);
                        dacc[4 * q + 0] = fmaf(xv.x, gu[rr], dacc[4 * q + 0]);
                        dacc[4 * q + 1] = fmaf(xv.y, gu[rr], dacc[4 * q + 1]);
                        dacc[4 * q + 2] = fmaf(xv.z, gu[rr], dacc[4 * q + 2]);
                        dacc[4 * q + 3] = fmaf(xv.w, gu[rr], dacc[4 * q + 3]);
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) ds[(r0 + rr) * D + out_bp] = acc[rr];
        }
        __syncthreads();
        if (dx) {
#pragma unroll 4
            for (int r = 0; r < R; ++r) {
                const int64_t row = row0 + r;
                if (row < batch) dx[row * D + t] = ds[r * D + t];
            }
        }
        __syncthreads();
    }
    // dC_k[s][u] partial of this CTA
    float *p = partial + (size_t)blockIdx.x * L.total + L.coff[k];
#pragma unroll
    for (int s = 0; s < NREG; ++s)
        if (s < ck) p[s * ck + u] = dacc[s];
}

// ------------------------------------------------------------------ generic --
// Any n in 2..12: one row per block pass; each thread computes outputs of its
// grade-sorted columns reading C from global memory (cached).
template <int TRANS>
__global__ void __launch_bounds__(256)
    rotor_apply_generic_kernel(const float *__restrict__ cs, const float *__restrict__ in,
                               float *__restrict__ out, int64_t batch, int n) {
    const Layout L = make_layout(n);
    extern __shared__ float sm[];  // sorted row [D]
    __shared__ int rank[1 << kMaxN], blades[1 << kMaxN];
    build_blade_tables(L, rank, blades);
    const int D = L.D;
    for (int64_t row = blockIdx.x; row < batch; row += gridDim.x) {
        for (int bp = threadIdx.x; bp < D; bp += blockDim.x)
            sm[L.goff[popc(bp)] + rank[bp]] = in[row * D + bp];
        __syncthreads();
        for (int t = threadIdx.x; t < D; t += blockDim.x) {
            int k = 0;
            while (t >= L.goff[k + 1]) ++k;
            const int ck = L.ck[k], col = t - L.goff[k];
            const float *Ck = cs + L.coff[k];
            float acc = 0.0f;
            for (int s = 0; s < ck; ++s)
                acc = fmaf(TRANS ? Ck[col * ck + s] : Ck[s * ck + col], sm[L.goff[k] + s], acc);
            out[row * D + blades[t]] = acc;
        }
        __syncthreads();
    }
}

// dC contributions with float atomics (generic sizes only).
__global__ void __launch_bounds__(256)
    rotor_dc_generic_kernel(const float *__restrict__ x, const float *__restrict__ g,
                            float *__restrict__ dcs, int64_t batch, int n) {
    const Layout L = make_layout(n);
    extern __shared__ float sm[];  // xs [D], gs [D] sorted
    __shared__ int rank[1 << kMaxN], blades[1 << kMaxN];
    build_blade_tables(L, rank, blades);
    const int D = L.D;
    float *xs = sm, *gs = sm + D;
    for (int64_t row = blockIdx.x; row < batch; row += gridDim.x) {
        for (int bp = threadIdx.x; bp < D; bp += blockDim.x) {
            const int sidx = L.goff[popc(bp)] + rank[bp];
            xs[sidx] = x[row * D + bp];
            gs[sidx] = g[row * D + bp];
        }
        __syncthreads();
        for (int e = threadIdx.x; e < L.total; e += blockDim.x) {
            int k = 0;
            while (e >= L.coff[k + 1]) ++k;
            const int ck = L.ck[k];
            const int ir = (e - L.coff[k]) / ck, jr = (e - L.coff[k]) % ck;
            atomicAdd(&dcs[e], xs[L.goff[k] + ir] * gs[L.goff[k] + jr]);
        }
        __syncthreads();
    }
}

// dcs[e] = sum_p partial[p][e], fixed order.
__global__ void rotor_reduce_kernel(const float *__restrict__ partial, int parts, int total,
                                    float *__restrict__ dcs) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    float s = 0.0f;
    for (int p = 0; p < parts; ++p) s += partial[(size_t)p * total + e];
    dcs[e] = s;
}

// dcs -> dbeta (one CTA of 1024 threads, fp64).
// dRm[p][q] = sum over grades k >= 1 and blades I containing p, J containing q
// (|I| = |J| = k) of (-1)^(a+b) dC_k[I][J] det Rm[I \ p, J \ q], a and b the
// positions of p in I and of q in J: the cofactor expansion of d det / d Rm.
// One warp per entry (p, q): lane t takes the subsets I' of the other n - 1
// generators numbered t, t + 32, ... and pairs each with every J' of the same
// size; the grade k - 1 minor det Rm[I', J'] is C_{k-1} from the forward pass.
// The adjoint Frechet derivative is linear in dRm, so dRm enters the block
// exponential divided by a power of two near its largest entry (exact), which
// keeps the number of squarings set by B alone, and the result is scaled back.
constexpr int kSubsetsPerPopc = 128;  // >= C(9, k), the subsets of n - 1 <= 9 generators

__global__ void __launch_bounds__(1024)
    rotor_compile_bwd_kernel(const double *__restrict__ state, const float *__restrict__ dcs,
                             int n, float *__restrict__ dbeta, bool stage) {
    const Layout L = make_layout(n);
    const int nn = n * n, m = 2 * n;
    __shared__ double dRm[kMaxN * kMaxN];
    __shared__ double Z[4 * kMaxN * kMaxN], E[4 * kMaxN * kMaxN], T[4 * kMaxN * kMaxN],
        W[4 * kMaxN * kMaxN];
    __shared__ int rank[1 << kMaxN];
    __shared__ double dscale;
    const double *Bm = state;
    const double *C64 = state + 2 * nn;
    // n <= 8: the minors and dC staged in shared memory (dynamic, 12 B per entry)
    extern __shared__ __align__(16) unsigned char stage_raw[];
    if (stage) {
        double *c64s = reinterpret_cast<double *>(stage_raw);
        float *dcss = reinterpret_cast<float *>(c64s + L.total);
        for (int e = threadIdx.x; e < L.total; e += blockDim.x) {
            c64s[e] = C64[e];
            dcss[e] = dcs[e];
        }
        C64 = c64s;
        dcs = dcss;
    }
    for (int bp = threadIdx.x; bp < L.D; bp += blockDim.x) rank[bp] = blade_rank(bp);
    // the subsets of the other n - 1 generators grouped by size, in a fixed order
    __shared__ unsigned short subsets[kMaxN * kSubsetsPerPopc];
    __shared__ int nsubsets[kMaxN];
    if (threadIdx.x == 0) {
        for (int k = 0; k < kMaxN; ++k) nsubsets[k] = 0;
        for (uint32_t j = 0; j < (1u << (n - 1)); ++j) {
            const int k = __popc(j);
            subsets[k * kSubsetsPerPopc + nsubsets[k]++] = (unsigned short)j;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const uint32_t sub = 1u << (n - 1);
    for (int e = warp; e < nn; e += nwarps) {
        const int p = e / n, q = e % n;
        const uint32_t lowp = (1u << p) - 1, lowq = (1u << q) - 1;
        double acc = 0.0, acc2 = 0.0;
        for (uint32_t i = lane; i < sub; i += 32) {
            const uint32_t Ip = (i & lowp) | ((i & ~lowp) << 1);  // I' (skips generator p)
            const int k1 = __popc(i), k = k1 + 1;
            const int ck = L.ck[k], ck1 = L.ck[k1];
            const int a = __popc(Ip & lowp);
            const uint32_t I = Ip | (1u << p);
            const int rowI = L.coff[k] + rank[I] * ck, rowIp = L.coff[k1] + rank[Ip] * ck1;
            const unsigned short *js = subsets + k1 * kSubsetsPerPopc;
            const int nj = nsubsets[k1];
            auto term = [&](uint32_t j) {
                const uint32_t Jp = (j & lowq) | ((j & ~lowq) << 1);
                const uint32_t J = Jp | (1u << q);
                const double t = (double)dcs[rowI + rank[J]] * C64[rowIp + rank[Jp]];
                return ((a + __popc(Jp & lowq)) & 1) ? -t : t;
            };
            // only the subsets J' of the same size; two independent chains of
            // dependent shared-memory loads per step
            int u = 0;
            for (; u + 1 < nj; u += 2) {
                acc += term(js[u]);
                acc2 += term(js[u + 1]);
            }
            if (u < nj) acc += term(js[u]);
        }
        acc += acc2;
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) dRm[e] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double mx = 0.0;
        for (int e = 0; e < nn; ++e) mx = fmax(mx, fabs(dRm[e]));
        dscale = mx > 0.0 ? ldexp(1.0, ilogb(mx) + 1) : 1.0;
    }
    __syncthreads();
    // Z = [[B^T, dRm], [0, B^T]]
    for (int e = threadIdx.x; e < m * m; e += blockDim.x) {
        const int i = e / m, j = e % m;
        double v = 0.0;
        if (i < n && j < n) v = Bm[j * n + i];
        else if (i >= n && j >= n) v = Bm[(j - n) * n + (i - n)];
        else if (i < n && j >= n) v = dRm[i * n + (j - n)] / dscale;
        Z[e] = v;
    }
    __syncthreads();
    expm(m, Z, E, T, W);
    if (threadIdx.x == 0) {
        int idx = 0;
        for (int p = 0; p < n - 1; ++p)
            for (int q = p + 1; q < n; ++q, ++idx) {
                const double dpq = E[p * m + n + q], dqp = E[q * m + n + p];
                dbeta[idx] = (float)(2.0 * (dpq - dqp) * dscale);
            }
    }
}

int fast_grid(int n, int64_t batch, int rows_per_tile, const void *kern, size_t smem,
              int threads) {
    DeviceInfo di;
    if (device_info(&di)) return -1;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess)
        return -1;
    per_sm = std::max(per_sm, 1);
    const int64_t tiles = (batch + rows_per_tile - 1) / rows_per_tile;
    return (int)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)per_sm * di.sm_count));
}

int check_rotor_n(int n) {
    if (n < 2 || n > kMaxN) {
        set_error("rotor: n = %d outside 2..%d", n, kMaxN);
        return CB_ERR_UNSUPPORTED;
    }
    return CB_OK;
}

template <int N>
size_t bwd_smem() {
    const Layout L = make_layout(N);
    return (size_t)16 * (2 * L.rowlen + L.D) * sizeof(float);
}

// Sets the kernel's shared-memory attribute, then sizes its persistent grid.
template <int N>
int bwd_grid(int64_t batch) {
    if (cudaFuncSetAttribute(rotor_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bwd_smem<N>()) != cudaSuccess)
        return -1;
    return fast_grid(N, batch, 16, (const void *)rotor_bwd_kernel<N>, bwd_smem<N>(), 1 << N);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_rotor_sizes(int n, int64_t *cs_floats, int64_t *state_doubles) {
    int st = check_rotor_n(n);
    if (st) return st;
    const Layout L = make_layout(n);
    if (cs_floats) *cs_floats = L.cs_floats;
    if (state_doubles) *state_doubles = 2 * n * n + L.total;
    return CB_OK;
}

extern "C" int cb_rotor_compile(const float *beta, int n, float *cs, double *state, void *stream) {
    int st = check_rotor_n(n);
    if (st) return st;
    if (!beta || !cs || !state) {
        set_error("rotor_compile: null pointer");
        return CB_ERR_INVALID;
    }
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int cgrid = std::min((make_layout(n).total + 255) / 256, 2 * di.sm_count);
    rotor_compile_kernel<<<cgrid, 256, 0, s>>>(beta, n, cs, state);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch rotor_compile_kernel");
    const Layout L = make_layout(n);
    if (L.tensor) {  // C_full built in the C_full-hi quarter, then split in place
        const int DD = L.D * L.D;
        float *mats = cs + L.mats_off;
        rotor_full_matrix_kernel<<<(DD + 255) / 256, 256, 0, s>>>(cs, n, mats + 2 * DD);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "launch rotor_full_matrix_kernel");
        return split_mats(mats + 2 * DD, mats, L.D, s);
    }
    return CB_OK;
}

static int rotor_apply_impl(const float *cs, const float *in, float *out, int64_t batch, int n,
                            int trans, cudaStream_t s) {
    int st = check_rotor_n(n);
    if (st) return st;
    if (batch < 0 || (batch > 0 && (!cs || !in || !out)) || (batch > 0 && in == out)) {
        set_error("rotor_apply: invalid arguments");
        return CB_ERR_INVALID;
    }
    if (batch == 0) return CB_OK;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const Layout L = make_layout(n);
    if (L.tensor) {
        const int64_t DD = (int64_t)L.D * L.D;
        const float *mats = cs + L.mats_off;
        return trans ? gemm3x_kmajor(L.D, in, mats + 2 * DD, mats + 3 * DD, out, batch, s)
                     : gemm3x_kmajor(L.D, in, mats, mats + DD, out, batch, s);
    }
    const size_t smem = (size_t)(1 << n) * sizeof(float);
    const int grid = (int)std::min<int64_t>(batch, (int64_t)di.sm_count * 8);
    if (trans)
        rotor_apply_generic_kernel<1><<<grid, 256, smem, s>>>(cs, in, out, batch, n);
    else
        rotor_apply_generic_kernel<0><<<grid, 256, smem, s>>>(cs, in, out, batch, n);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_apply_generic_kernel");
}

extern "C" int cb_rotor_apply(const float *cs, const float *x, float *y, int64_t batch, int n,
                              int transpose, void *stream) {
    return rotor_apply_impl(cs, x, y, batch, n, transpose, static_cast<cudaStream_t>(stream));
}

extern "C" int cb_rotor_workspace_bytes(int n, int64_t batch, int64_t *bytes) {
    int st = check_rotor_n(n);
    if (st) return st;
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const Layout L = make_layout(n);
    int64_t floats = 0;
    if (L.tensor) {
        const int parts = gemm3x_mn_parts(batch);
        if (parts <= 0) return cuda_fail(cudaGetLastError(), "rotor workspace sizing");
        floats = (int64_t)(parts + 1) * L.D * L.D;  // split-K partials + G
    }
    *bytes = floats * (int64_t)sizeof(float);
    return CB_OK;
}

extern "C" int cb_rotor_apply_bwd(const float *cs, const float *x, const float *g, float *dx,
                                  float *dcs, int64_t batch, int n, void *workspace,
                                  int64_t workspace_bytes, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = check_rotor_n(n);
    if (st) return st;
    if (batch < 0 || !cs || !dcs || (batch > 0 && (!x || !g))) {
        set_error("rotor_apply_bwd: invalid arguments");
        return CB_ERR_INVALID;
    }
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const Layout L = make_layout(n);
    if (batch == 0) {
        cudaError_t e = cudaMemsetAsync(dcs, 0, (size_t)L.cs_floats * sizeof(float), s);
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs)");
    }
    if (L.tensor) {
        const int64_t DD = (int64_t)L.D * L.D;
        const float *mats = cs + L.mats_off;
        const int parts = gemm3x_mn_parts(batch);
        const int64_t need = (int64_t)(parts + 1) * DD * (int64_t)sizeof(float);
        if (parts <= 0 || !workspace || workspace_bytes < need) {
            set_error("rotor_apply_bwd: workspace of %lld bytes needed, %lld given",
                      (long long)need, (long long)workspace_bytes);
            return CB_ERR_INVALID;
        }
        if (dx && (st = gemm3x_kmajor(L.D, g, mats + 2 * DD, mats + 3 * DD, dx, batch, s)))
            return st;
        float *partial = static_cast<float *>(workspace);
        float *G = partial + (size_t)parts * DD;
        if ((st = gemm3x_mn(L.D, x, g, partial, batch, parts, s))) return st;
        if ((st = reduce_partials(partial, parts, L.D, G, s))) return st;
        rotor_gather_dc_kernel<<<(L.total + 255) / 256, 256, 0, s>>>(G, n, dcs);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "launch rotor_gather_dc_kernel");
        e = cudaMemsetAsync(dcs + L.total, 0, (size_t)(L.cs_floats - L.total) * sizeof(float), s);
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs tail)");
    }
    // generic sizes: dx by the transposed apply, dC by atomics
    if (dx && (st = rotor_apply_impl(cs, g, dx, batch, n, 1, s))) return st;
    cudaError_t e = cudaMemsetAsync(dcs, 0, (size_t)L.total * sizeof(float), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(dcs)");
    const int grid = (int)std::min<int64_t>(batch, (int64_t)di.sm_count * 8);
    rotor_dc_generic_kernel<<<grid, 256, 2 * (size_t)(1 << n) * sizeof(float), s>>>(x, g, dcs,
                                                                                     batch, n);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_dc_generic_kernel");
}

extern "C" int cb_rotor_compile_bwd(const double *state, const float *dcs, int n, float *dbeta,
                                    void *stream) {
    int st = check_rotor_n(n);
    if (st) return st;
    if (!state || !dcs || !dbeta) {
        set_error("rotor_compile_bwd: null pointer");
        return CB_ERR_INVALID;
    }
    DeviceInfo di;
    if ((st = device_info(&di))) return st;
    const Layout L = make_layout(n);
    const size_t stage_bytes = (size_t)L.total * (sizeof(double) + sizeof(float));
    const bool stage = stage_bytes <= (size_t)200 * 1024;
    if (stage) {
        cudaError_t e0 = cudaFuncSetAttribute(rotor_compile_bwd_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)stage_bytes);
        if (e0 != cudaSuccess) return cuda_fail(e0, "cudaFuncSetAttribute(rotor_compile_bwd)");
    }
    rotor_compile_bwd_kernel<<<1, 1024, stage ? stage_bytes : 0, static_cast<cudaStream_t>(stream)>>>(
        state, dcs, n, dbeta, stage);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_compile_bwd_kernel");
}

// --------------------------------------------- backward without allocation --
// cb_rotor_apply_bwd needs a workspace for the per-CTA partial sums of dC,
// which the caller allocates. Some callers cannot: a host program that binds
// only this C ABI from another language and has no device allocator of its
// own, or a framework whose device memory is all owned by its own pool and
// that forbids side allocations inside a training step. For them,
// cb_rotor_apply_bwd_noalloc keeps the partials in this fixed array instead:
// 2^21 floats (8 MiB), which every GPU that loads the library holds until
// the process exits. It covers n = 7 and 8, the sizes whose backward uses
// partial sums; the grid is capped so the partials fit.
namespace {

constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 21;
static __device__ __align__(256) float g_rotor_bwd_scratch[kNoAllocScratchFloats];

constexpr int kMaxScratchDevices = 64;
static float *g_scratch_addr[kMaxScratchDevices];
static std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device. In host code
// the array's name is only a host-side stand-in, so the address is looked up
// with that device current and cached once the lookup succeeds; a failed
// lookup (for example one attempted during stream capture) is reported and
// tried again on the next call.
int noalloc_scratch(float **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxScratchDevices) {
        set_error("device ordinal %d out of range", dev);
        return CB_ERR_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_rotor_bwd_scratch);
        if (e != cudaSuccess || !p)
            return cuda_fail(e, "cudaGetSymbolAddress(rotor backward scratch)");
        g_scratch_addr[dev] = static_cast<float *>(p);
    }
    *out = g_scratch_addr[dev];
    return CB_OK;
}

template <int N>
int noalloc_bwd(const float *cs, const float *x, const float *g, float *dx, float *dcs,
                int64_t batch, cudaStream_t s) {
    const Layout L = make_layout(N);
    float *scratch = nullptr;
    int st = noalloc_scratch(&scratch);
    if (st) return st;
    int parts = bwd_grid<N>(batch);
    if (parts <= 0) return cuda_fail(cudaGetLastError(), "rotor backward occupancy");
    parts = (int)std::min<int64_t>(parts, kNoAllocScratchFloats / L.total);
    // Every CTA writes all of its partial slot, so nothing needs clearing.
    rotor_bwd_kernel<N><<<parts, 1 << N, bwd_smem<N>(), s>>>(cs, x, g, dx, scratch, batch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch rotor_bwd_kernel (no-alloc)");
    rotor_reduce_kernel<<<(L.total + 255) / 256, 256, 0, s>>>(scratch, parts, L.total, dcs);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch rotor_reduce_kernel (no-alloc)");
    // the tensor-core operands appended to cs receive no gradient
    e = cudaMemsetAsync(dcs + L.total, 0, (size_t)(L.cs_floats - L.total) * sizeof(float), s);
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs tail)");
}

}  // namespace

extern "C" int cb_rotor_apply_bwd_noalloc(const float *cs, const float *x, const float *g,
                                          float *dx, float *dcs, int64_t batch, int n,
                                          void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n != 7 && n != 8) {
        set_error("rotor_apply_bwd_noalloc: n = %d unsupported; its fixed 8 MiB scratch "
                  "covers n = 7 and 8 only (use cb_rotor_apply_bwd with a workspace)", n);
        return CB_ERR_UNSUPPORTED;
    }
    if (batch < 0 || !cs || !dcs || (batch > 0 && (!x || !g))) {
        set_error("rotor_apply_bwd_noalloc: invalid arguments");
        return CB_ERR_INVALID;
    }
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    if (batch == 0) {
        cudaError_t e = cudaMemsetAsync(dcs, 0, (size_t)make_layout(n).cs_floats * sizeof(float), s);
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs)");
    }
    return n == 7 ? noalloc_bwd<7>(cs, x, g, dx, dcs, batch, s)
                  : noalloc_bwd<8>(cs, x, g, dx, dcs, batch, s);
}
