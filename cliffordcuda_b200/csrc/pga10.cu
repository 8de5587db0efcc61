// pga10.cu -- the geometric product of Cl(9,0,1) (nine generators squaring to
// +1, the tenth, e9, to 0: BASELINE config 5's algebra) through Cl(8,0)
// matrix products.
//
// Two exact algebra maps reduce it to the Cl(8,0) product of gp_mat16.cu:
//   * dual numbers: with a = a0 + a1 e9 (a0, a1 in Cl(9,0); rows split as
//     [a0 | a1], 512 floats each, e9 the top index bit), e9^2 = 0 and
//     e9 x = g(x) e9 (g = grade involution) give
//         c0 = a0 b0,   c1 = a0 b1 + a1 g(b0);
//   * Cl(9,0) = Cl(8,0) + Cl(8,0): with x = u + v e8 (u, v in Cl(8,0); a
//     512-block split as [u | v]) and w = e0 e1 ... e7 (w^2 = 1, w anticommutes
//     with e0..e7 and so behaves like e8), x -> (X+, X-) = (u + v w, u - v w)
//     is an algebra isomorphism onto pairs of Cl(8,0) elements multiplied
//     componentwise. Its inverse is u = (X+ + X-)/2, v = (X+ - X-) w / 2,
//     and g(x) maps to (g(X-), g(X+)).
// So c0+- = A0+- B0+-, c1+- = A0+- B1+- + A1+- g(B0-+): six Cl(8,0) products
// (each one 16 x 16 x 16 matrix product in gp_mat16) instead of the 4^10
// blade terms of the direct sum. The backward sums follow by the chain rule
// through the same linear maps (the adjoint of x -> (X+, X-) is
// (P, Q) -> [P + Q | (P - Q) w]; g and right multiplication by w are
// orthogonal and their own adjoints), with six fused Cl(8,0) backward passes.
// The maps are one HBM pass each (pga_split_kernel, pga_merge_kernel); the
// intermediate Cl(8,0) planes live in the caller's workspace.
// Reference for the product itself: extensions/ga/geom_prod.py:216-276 (the
// blade-by-blade product and its autograd backward sums, geom_prod.py:241-250).
#include <algorithm>

#include "common.cuh"

namespace cb {
namespace {

// (v w)[K] = w(~K) v[~K], w(J) = (-1)^(sum of the positions of J's generators).
__device__ __forceinline__ float wsign(uint32_t j) { return (__popc(j & 0xAAu) & 1) ? -1.0f : 1.0f; }
__device__ __forceinline__ float gsign(uint32_t j) { return (__popc(j) & 1) ? -1.0f : 1.0f; }

// Block h (0 or 1) of rows x (batch, 1024) -> planes (batch, 256):
//   p = u + v w, m = u - v w, gp = g(p), gm = g(m)   (null outputs skipped).
// One thread per float4 of a plane row.
__global__ void __launch_bounds__(256)
    pga_split_kernel(const float *__restrict__ x, int h, float *__restrict__ p,
                     float *__restrict__ m, float *__restrict__ gp, float *__restrict__ gm,
                     int64_t batch) {
    const int64_t total = batch * 64;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
         c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = c >> 6;
        const uint32_t k0 = (uint32_t)(c & 63) << 2;
        const float *blk = x + row * 1024 + h * 512;
        const float4 u = *reinterpret_cast<const float4 *>(blk + k0);
        // v[~k] for k = k0..k0+3 are v[252 - k0 .. 255 - k0], reversed
        const float4 vr = *reinterpret_cast<const float4 *>(blk + 256 + (252 - k0));
        const float vw[4] = {wsign(255 - k0) * vr.w, wsign(254 - k0) * vr.z,
                             wsign(253 - k0) * vr.y, wsign(252 - k0) * vr.x};
        const float uu[4] = {u.x, u.y, u.z, u.w};
        float pv[4], mv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            pv[e] = uu[e] + vw[e];
            mv[e] = uu[e] - vw[e];
        }
        const int64_t o = row * 256 + k0;
        if (p) *reinterpret_cast<float4 *>(p + o) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        if (m) *reinterpret_cast<float4 *>(m + o) = make_float4(mv[0], mv[1], mv[2], mv[3]);
        if (gp || gm) {
            float s[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) s[e] = gsign(k0 + e);
            if (gp)
                *reinterpret_cast<float4 *>(gp + o) =
                    make_float4(s[0] * pv[0], s[1] * pv[1], s[2] * pv[2], s[3] * pv[3]);
            if (gm)
                *reinterpret_cast<float4 *>(gm + o) =
                    make_float4(s[0] * mv[0], s[1] * mv[1], s[2] * mv[2], s[3] * mv[3]);
        }
    }
}

struct MergeIn {
    const float *p1, *p2, *q1, *q2;  // p2, q2 may be null
    int g2;                          // apply the grade involution to p2 and q2
};

// Block h of rows out (batch, 1024) = scale * [P + Q | (P - Q) w] with
// P = p1 + g?(p2), Q = q1 + g?(q2) (planes (batch, 256)).
__global__ void __launch_bounds__(256)
    pga_merge_kernel(MergeIn in, float scale, float *__restrict__ out, int h, int64_t batch) {
    const int64_t total = batch * 64;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
         c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = c >> 6;
        const uint32_t k0 = (uint32_t)(c & 63) << 2;
        const int64_t base = row * 256;
        auto ld = [&](const float *pl, uint32_t j) {
            const float4 t = *reinterpret_cast<const float4 *>(pl + base + j);
            return t;
        };
        float P[4], Q[4], Pr[4], Qr[4];  // at k0.., and at ~k (reversed) for the v part
        {
            const float4 a = ld(in.p1, k0), b = ld(in.q1, k0);
            const float4 ar = ld(in.p1, 252 - k0), br = ld(in.q1, 252 - k0);
            P[0] = a.x; P[1] = a.y; P[2] = a.z; P[3] = a.w;
            Q[0] = b.x; Q[1] = b.y; Q[2] = b.z; Q[3] = b.w;
            Pr[0] = ar.w; Pr[1] = ar.z; Pr[2] = ar.y; Pr[3] = ar.x;
            Qr[0] = br.w; Qr[1] = br.z; Qr[2] = br.y; Qr[3] = br.x;
        }
        if (in.p2) {
            const float4 a = ld(in.p2, k0), ar = ld(in.p2, 252 - k0);
            const float av[4] = {a.x, a.y, a.z, a.w}, arv[4] = {ar.w, ar.z, ar.y, ar.x};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                P[e] += in.g2 ? gsign(k0 + e) * av[e] : av[e];
                Pr[e] += in.g2 ? gsign(255 - k0 - e) * arv[e] : arv[e];
            }
        }
        if (in.q2) {
            const float4 b = ld(in.q2, k0), br = ld(in.q2, 252 - k0);
            const float bv[4] = {b.x, b.y, b.z, b.w}, brv[4] = {br.w, br.z, br.y, br.x};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                Q[e] += in.g2 ? gsign(k0 + e) * bv[e] : bv[e];
                Qr[e] += in.g2 ? gsign(255 - k0 - e) * brv[e] : brv[e];
            }
        }
        float *blk = out + row * 1024 + h * 512;
        float uo[4], vo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            uo[e] = scale * (P[e] + Q[e]);
            vo[e] = scale * wsign(255 - k0 - e) * (Pr[e] - Qr[e]);
        }
        *reinterpret_cast<float4 *>(blk + k0) = make_float4(uo[0], uo[1], uo[2], uo[3]);
        *reinterpret_cast<float4 *>(blk + 256 + k0) = make_float4(vo[0], vo[1], vo[2], vo[3]);
    }
}

int grid_for(int64_t batch) {
    DeviceInfo di;
    if (device_info(&di)) return -1;
    const int64_t blocks = (batch * 64 + 255) / 256;
    return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)di.sm_count * 8));
}

int split(const float *x, int h, float *p, float *m, float *gp, float *gm, int64_t batch,
          cudaStream_t s) {
    const int grid = grid_for(batch);
    if (grid < 0) return CB_ERR_CUDA;
    pga_split_kernel<<<grid, 256, 0, s>>>(x, h, p, m, gp, gm, batch);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch pga_split_kernel");
}

int merge(const float *p1, const float *p2, const float *q1, const float *q2, int g2,
          float *out, int h, int64_t batch, cudaStream_t s) {
    const int grid = grid_for(batch);
    if (grid < 0) return CB_ERR_CUDA;
    pga_merge_kernel<<<grid, 256, 0, s>>>(MergeIn{p1, p2, q1, q2, g2}, 0.5f, out, h, batch);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch pga_merge_kernel");
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool use_pga10(int op, int n, uint32_t neg, uint32_t zero) {
    return op == CB_OP_GP && n == 10 && neg == 0 && zero == (1u << 9);
}

int64_t pga10_workspace_bytes(int64_t batch) { return 26 * batch * 1024; }

// c = a b in Cl(9,0,1); ws holds 16 planes of (batch, 256).
int pga10_fwd(const float *a, const float *b, float *c, int64_t batch, void *ws,
              int64_t ws_bytes, cudaStream_t s) {
    if (batch == 0) return CB_OK;
    if (!ws || ws_bytes < pga10_workspace_bytes(batch) || !al16(ws) || !al16(a) || !al16(b) ||
        !al16(c)) {
        set_error("Cl(9,0,1) product route: workspace of %lld bytes (16-byte aligned) needed",
                  (long long)pga10_workspace_bytes(batch));
        return CB_ERR_INVALID;
    }
    float *W = static_cast<float *>(ws);
    auto plane = [&](int i) { return W + (size_t)i * batch * 256; };
    float *A0p = plane(0), *A0m = plane(1), *A1p = plane(2), *A1m = plane(3);
    float *B0p = plane(4), *B0m = plane(5), *gB0p = plane(6), *gB0m = plane(7);
    float *B1p = plane(8), *B1m = plane(9);
    float *P[6];
    for (int i = 0; i < 6; ++i) P[i] = plane(10 + i);
    int st;
    if ((st = split(a, 0, A0p, A0m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(a, 1, A1p, A1m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(b, 0, B0p, B0m, gB0p, gB0m, batch, s))) return st;
    if ((st = split(b, 1, B1p, B1m, nullptr, nullptr, batch, s))) return st;
    const float *L[6] = {A0p, A0m, A0p, A1p, A0m, A1m};
    const float *R[6] = {B0p, B0m, B1p, gB0m, B1m, gB0p};
    for (int i = 0; i < 6; ++i)
        if ((st = gp_mat16(CB_MODE_FWD, L[i], R[i], P[i], batch, s))) return st;
    if ((st = merge(P[0], nullptr, P[1], nullptr, 0, c, 0, batch, s))) return st;
    return merge(P[2], P[3], P[4], P[5], 0, c, 1, batch, s);
}

// Both backward sums of c = a b in Cl(9,0,1) for upstream g; ws holds 26 planes.
int pga10_bwd(const float *a, const float *b, const float *g, float *ga, float *gb, int64_t batch,
              void *ws, int64_t ws_bytes, cudaStream_t s) {
    if (batch == 0) return CB_OK;
    if (!ws || ws_bytes < pga10_workspace_bytes(batch) || !al16(ws) || !al16(a) || !al16(b) ||
        !al16(g) || (ga && !al16(ga)) || (gb && !al16(gb))) {
        set_error("Cl(9,0,1) product route: workspace of %lld bytes (16-byte aligned) needed",
                  (long long)pga10_workspace_bytes(batch));
        return CB_ERR_INVALID;
    }
    float *W = static_cast<float *>(ws);
    auto plane = [&](int i) { return W + (size_t)i * batch * 256; };
    float *A0p = plane(0), *A0m = plane(1), *A1p = plane(2), *A1m = plane(3);
    float *B0p = plane(4), *B0m = plane(5), *gB0p = plane(6), *gB0m = plane(7);
    float *B1p = plane(8), *B1m = plane(9);
    float *G0p = plane(10), *G0m = plane(11), *G1p = plane(12), *G1m = plane(13);
    float *dA[6], *dB[6];
    for (int i = 0; i < 6; ++i) {
        dA[i] = plane(14 + i);
        dB[i] = plane(20 + i);
    }
    int st;
    if ((st = split(a, 0, A0p, A0m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(a, 1, A1p, A1m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(b, 0, B0p, B0m, gB0p, gB0m, batch, s))) return st;
    if ((st = split(b, 1, B1p, B1m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(g, 0, G0p, G0m, nullptr, nullptr, batch, s))) return st;
    if ((st = split(g, 1, G1p, G1m, nullptr, nullptr, batch, s))) return st;
    // products P0..P5 of the forward: (A0+ B0+; g0+), (A0- B0-; g0-), (A0+ B1+; g1+),
    // (A1+ g(B0-); g1+), (A0- B1-; g1-), (A1- g(B0+); g1-)
    const float *L[6] = {A0p, A0m, A0p, A1p, A0m, A1m};
    const float *R[6] = {B0p, B0m, B1p, gB0m, B1m, gB0p};
    const float *G[6] = {G0p, G0m, G1p, G1p, G1m, G1m};
    for (int i = 0; i < 6; ++i)
        if ((st = gp_mat16_bwd(L[i], R[i], G[i], dA[i], dB[i], batch, s))) return st;
    if (ga) {
        if ((st = merge(dA[0], dA[2], dA[1], dA[4], 0, ga, 0, batch, s))) return st;
        if ((st = merge(dA[3], nullptr, dA[5], nullptr, 0, ga, 1, batch, s))) return st;
    }
    if (gb) {
        // b0 reaches P3 and P5 through g(B0-) and g(B0+): their grads come back
        // through g onto the other component
        if ((st = merge(dB[0], dB[5], dB[1], dB[3], 1, gb, 0, batch, s))) return st;
        if ((st = merge(dB[2], nullptr, dB[4], nullptr, 0, gb, 1, batch, s))) return st;
    }
    return CB_OK;
}

}  // namespace cb
