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
//   compile:  one CTA in fp64 -- Rm by scaling and squaring of a Taylor series
//             (||B / 2^s||_1 <= 1/8, 20 terms), then every equal-grade minor
//             C_k[I][J] = det(Rm[I, J]) by Gaussian elimination with partial
//             pivoting. Per grade k the C(n,k) x C(n,k) matrix is stored
//             row-major, grades concatenated (C(2n, n) entries in total).
//   apply:    y_k = x_k C_k per grade (and g_k C_k^T for the x gradient).
//             A thread owns one column of its grade's matrix, held in
//             registers; rows are staged in shared memory in grade-sorted,
//             4-padded order so each float4 load feeds four FFMAs.
//   backward: one pass over (x, g) gives dx = g C^T and per-CTA partial sums
//             of dC_k = x_k^T g_k into a caller-provided workspace; a second
//             kernel sums the partials in a fixed order. The chain to the
//             bivector runs in one CTA in fp64:
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

// Per-n layout of the compiled rotor.
struct Layout {
    int n, D;
    int ck[kMaxN + 1];       // C(n, k)
    int goff[kMaxN + 2];     // first grade-sorted index of grade k
    int coff[kMaxN + 2];     // first matrix entry of grade k (sum of C(n,j)^2)
    int padoff[kMaxN + 2];   // first slot of grade k in a 4-padded sorted row
    int total, rowlen;
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
    return L;
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
    for (int e = threadIdx.x; e < nn; e += blockDim.x) state[e] = Bm[e];  // B (unscaled)
    __syncthreads();
    expm(n, Bm, Rm, T, W);
    for (int e = threadIdx.x; e < nn; e += blockDim.x) state[nn + e] = Rm[e];
    build_blade_tables(L, rank, blades);
    double *C64 = state + 2 * nn;
    for (int e = threadIdx.x; e < L.total; e += blockDim.x) {
        int k = 0;
        while (e >= L.coff[k + 1]) ++k;
        const int ck = L.ck[k];
        const int ir = (e - L.coff[k]) / ck, jr = (e - L.coff[k]) % ck;
        const double v = minor_det(n, Rm, blades[L.goff[k] + ir], blades[L.goff[k] + jr], k);
        C64[e] = v;
        cs[e] = (float)v;
    }
}

// ------------------------------------------------------------ apply (fast) --
// TRANS = 0: out_k = in_k C_k (y from x); TRANS = 1: out_k = in_k C_k^T.
template <int N, int TRANS>
__global__ void __launch_bounds__(1 << N)
    rotor_apply_kernel(const float *__restrict__ cs, const float *__restrict__ in,
                       float *__restrict__ out, int64_t batch) {
    constexpr int D = 1 << N;
    constexpr int MAXC = (N == 7) ? 35 : 70;
    constexpr int R = 32;  // rows per tile
    const Layout L = make_layout(N);
    extern __shared__ float sm[];
    float *xs = sm;                       // [R][rowlen], grade-sorted, 4-padded
    float *ys = sm + R * L.rowlen;        // [R][D], bit-pattern order
    __shared__ int rank[D], blades[D];
    build_blade_tables(L, rank, blades);

    const int t = threadIdx.x;  // grade-sorted index of this thread's column
    int k = 0;
    while (t >= L.goff[k + 1]) ++k;
    const int ck = L.ck[k];
    const int col = t - L.goff[k];
    const int pk = (ck + 3) & ~3;
    const int xoff = L.padoff[k];
    const int out_bp = blades[t];
    constexpr int NREG = (MAXC + 3) / 4 * 4;
    float creg[NREG];
#pragma unroll
    for (int s = 0; s < NREG; ++s) {
        float v = 0.0f;
        if (s < ck) v = TRANS ? cs[L.coff[k] + col * ck + s] : cs[L.coff[k] + s * ck + col];
        creg[s] = v;
    }
    // sorted slot of input blade t (bit-pattern index t)
    const int in_slot = L.padoff[popc(t)] + rank[t];
    for (int e = t; e < R * L.rowlen; e += D) xs[e] = 0.0f;  // zero the pad slots
    __syncthreads();

    for (int64_t row0 = (int64_t)blockIdx.x * R; row0 < batch; row0 += (int64_t)gridDim.x * R) {
#pragma unroll 4
        for (int r = 0; r < R; ++r) {
            const int64_t row = row0 + r;
            xs[r * L.rowlen + in_slot] = (row < batch) ? in[row * D + t] : 0.0f;
        }
        __syncthreads();
#pragma unroll 1
        for (int r0 = 0; r0 < R; r0 += 4) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q = 0; q < (MAXC + 3) / 4; ++q) {
                if (4 * q < pk) {
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        const float4 xv =
                            *reinterpret_cast<const float4 *>(xs + (r0 + rr) * L.rowlen + xoff + 4 * q);
                        acc[rr] = fmaf(creg[4 * q + 0], xv.x, acc[rr]);
                        acc[rr] = fmaf(creg[4 * q + 1], xv.y, acc[rr]);
                        acc[rr] = fmaf(creg[4 * q + 2], xv.z, acc[rr]);
                        acc[rr] = fmaf(creg[4 * q + 3], xv.w, acc[rr]);
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) ys[(r0 + rr) * D + out_bp] = acc[rr];
        }
        __syncthreads();
#pragma unroll 4
        for (int r = 0; r < R; ++r) {
            const int64_t row = row0 + r;
            if (row < batch) out[row * D + t] = ys[r * D + t];
        }
        __syncthreads();
    }
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

// dcs -> dbeta (one CTA, fp64).
__global__ void __launch_bounds__(256)
    rotor_compile_bwd_kernel(const double *__restrict__ state, const float *__restrict__ dcs,
                             int n, float *__restrict__ dbeta) {
    const Layout L = make_layout(n);
    const int nn = n * n, m = 2 * n;
    __shared__ double dRm[kMaxN * kMaxN];
    __shared__ double Z[4 * kMaxN * kMaxN], E[4 * kMaxN * kMaxN], T[4 * kMaxN * kMaxN],
        W[4 * kMaxN * kMaxN];
    __shared__ int rank[1 << kMaxN], blades[1 << kMaxN];
    build_blade_tables(L, rank, blades);
    const double *Bm = state;
    const double *C64 = state + 2 * nn;
    for (int e = threadIdx.x; e < nn; e += blockDim.x) dRm[e] = 0.0;
    __syncthreads();
    for (int e = threadIdx.x; e < L.total; e += blockDim.x) {
        int k = 0;
        while (e >= L.coff[k + 1]) ++k;
        if (k == 0) continue;
        const double v = (double)dcs[e];
        if (v == 0.0) continue;
        const int ck = L.ck[k], ck1 = L.ck[k - 1];
        const uint32_t I = blades[L.goff[k] + (e - L.coff[k]) / ck];
        const uint32_t J = blades[L.goff[k] + (e - L.coff[k]) % ck];
        int a = 0;
        for (int p = 0; p < n; ++p) {
            if (!((I >> p) & 1u)) continue;
            const uint32_t Ip = I & ~(1u << p);
            int b = 0;
            for (int q = 0; q < n; ++q) {
                if (!((J >> q) & 1u)) continue;
                const uint32_t Jq = J & ~(1u << q);
                const double minor =
                    (k == 1) ? 1.0 : C64[L.coff[k - 1] + rank[Ip] * ck1 + rank[Jq]];
                atomicAdd(&dRm[p * n + q], ((a + b) & 1) ? -v * minor : v * minor);
                ++b;
            }
            ++a;
        }
    }
    __syncthreads();
    // Z = [[B^T, dRm], [0, B^T]]
    for (int e = threadIdx.x; e < m * m; e += blockDim.x) {
        const int i = e / m, j = e % m;
        double v = 0.0;
        if (i < n && j < n) v = Bm[j * n + i];
        else if (i >= n && j >= n) v = Bm[(j - n) * n + (i - n)];
        else if (i < n && j >= n) v = dRm[i * n + (j - n)];
        Z[e] = v;
    }
    __syncthreads();
    expm(m, Z, E, T, W);
    if (threadIdx.x == 0) {
        int idx = 0;
        for (int p = 0; p < n - 1; ++p)
            for (int q = p + 1; q < n; ++q, ++idx) {
                const double dpq = E[p * m + n + q], dqp = E[q * m + n + p];
                dbeta[idx] = (float)(2.0 * (dpq - dqp));
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

template <int N, int TRANS>
int launch_apply_fast(const float *cs, const float *in, float *out, int64_t batch,
                      cudaStream_t stream) {
    const Layout L = make_layout(N);
    const size_t smem = (size_t)32 * (L.rowlen + L.D) * sizeof(float);
    auto kern = rotor_apply_kernel<N, TRANS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rotor_apply)");
    const int grid = fast_grid(N, batch, 32, (const void *)kern, smem, 1 << N);
    if (grid < 0) return cuda_fail(cudaGetLastError(), "rotor_apply occupancy");
    kern<<<grid, 1 << N, smem, stream>>>(cs, in, out, batch);
    e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_apply_kernel");
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
    if (cs_floats) *cs_floats = L.total;
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
    rotor_compile_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(beta, n, cs, state);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_compile_kernel");
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
    if (n == 7) return trans ? launch_apply_fast<7, 1>(cs, in, out, batch, s)
                             : launch_apply_fast<7, 0>(cs, in, out, batch, s);
    if (n == 8) return trans ? launch_apply_fast<8, 1>(cs, in, out, batch, s)
                             : launch_apply_fast<8, 0>(cs, in, out, batch, s);
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
    int parts = 0;
    if (n == 7) parts = bwd_grid<7>(std::max<int64_t>(batch, 1));
    else if (n == 8) parts = bwd_grid<8>(std::max<int64_t>(batch, 1));
    *bytes = (int64_t)std::max(parts, 0) * L.total * (int64_t)sizeof(float);
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
        cudaError_t e = cudaMemsetAsync(dcs, 0, (size_t)L.total * sizeof(float), s);
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs)");
    }
    if (n == 7 || n == 8) {
        const int parts = (n == 7) ? bwd_grid<7>(batch) : bwd_grid<8>(batch);
        const int64_t need = (int64_t)parts * L.total * (int64_t)sizeof(float);
        if (parts <= 0 || !workspace || workspace_bytes < need) {
            set_error("rotor_apply_bwd: workspace of %lld bytes needed, %lld given",
                      (long long)need, (long long)workspace_bytes);
            return CB_ERR_INVALID;
        }
        float *partial = static_cast<float *>(workspace);
        if (n == 7)
            rotor_bwd_kernel<7><<<parts, 128, bwd_smem<7>(), s>>>(cs, x, g, dx, partial, batch);
        else
            rotor_bwd_kernel<8><<<parts, 256, bwd_smem<8>(), s>>>(cs, x, g, dx, partial, batch);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "launch rotor_bwd_kernel");
        rotor_reduce_kernel<<<(L.total + 255) / 256, 256, 0, s>>>(partial, parts, L.total, dcs);
        e = cudaGetLastError();
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_reduce_kernel");
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
    rotor_compile_bwd_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(state, dcs, n, dbeta);
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
static cudaError_t g_scratch_err[kMaxScratchDevices];
static std::once_flag g_scratch_once[kMaxScratchDevices];

// Device address of the scratch array on the current device. In host code
// the array's name is only a host-side stand-in, so the address is fetched
// once per device, with that device current, and cached.
int noalloc_scratch(float **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxScratchDevices) {
        set_error("device ordinal %d out of range", dev);
        return CB_ERR_UNSUPPORTED;
    }
    std::call_once(g_scratch_once[dev], [dev] {
        void *p = nullptr;
        g_scratch_err[dev] = cudaGetSymbolAddress(&p, g_rotor_bwd_scratch);
        g_scratch_addr[dev] = (g_scratch_err[dev] == cudaSuccess) ? static_cast<float *>(p) : nullptr;
    });
    if (!g_scratch_addr[dev])
        return cuda_fail(g_scratch_err[dev], "cudaGetSymbolAddress(rotor backward scratch)");
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
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch rotor_reduce_kernel (no-alloc)");
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
        cudaError_t e = cudaMemsetAsync(dcs, 0, (size_t)make_layout(n).total * sizeof(float), s);
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "cudaMemsetAsync(dcs)");
    }
    return n == 7 ? noalloc_bwd<7>(cs, x, g, dx, dcs, batch, s)
                  : noalloc_bwd<8>(cs, x, g, dx, dcs, batch, s);
}
