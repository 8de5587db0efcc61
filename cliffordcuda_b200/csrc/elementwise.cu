// elementwise.cu -- the per-blade maps of CliffordAlgebra and their norm:
// reversion, grade involution, Clifford conjugation, grade projection, the
// dual (x I^-1) and norm_sq, each one pass over HBM.
//
// Every map multiplies coefficient i of a row by a factor that depends only
// on the blade index (and, for the dual, reads the complementary blade): the
// factor is computed from popcounts in registers, so there is no table to
// load. Rows are (batch, 2^n) fp32; the kernels stream float4 chunks of the
// flattened array (coalesced 16-byte accesses, grid-stride, grid a multiple
// of the SM count) and fall back to scalar accesses for 2^n < 4 or
// misaligned pointers.
//
// Reference definitions (src/cliffordcuda/algebra.py):
//   reverse              (-1)^(k(k-1)/2), k = grade          algebra.py:195-206
//   dual                 out[m] = s(a) x[a], a = ~m           algebra.py:208-266
//   grade_involution     (-1)^k                               algebra.py:278-286
//   clifford_conjugation (-1)^(k(k+1)/2)                      algebra.py:288-296
//   grade_projection     [k == grade]                         algebra.py:298-307
//   norm_sq              sum_b x_b^2 prod_{t in b} metric[t]  algebra.py:309-336
#include <algorithm>

#include "common.cuh"

namespace cb {
namespace {

// Factor of output blade m for map `kind` (the dual's input blade is ~m).
__device__ __forceinline__ float map_factor(int kind, uint32_t m, uint32_t full, uint32_t neg,
                                            int grade, float dual_scale) {
    const int k = __popc(m);
    switch (kind) {
    case CB_MAP_REVERSE: return ((k * (k - 1) / 2) & 1) ? -1.0f : 1.0f;
    case CB_MAP_INVOLUTE: return (k & 1) ? -1.0f : 1.0f;
    case CB_MAP_CONJUGATE: return ((k * (k + 1) / 2) & 1) ? -1.0f : 1.0f;
    case CB_MAP_GRADE: return k == grade ? 1.0f : 0.0f;
    default: {
        // e_a I^-1 = s(a) e_m with a = ~m: (1 / I^2) times the sign of moving
        // e_a past the whole pseudoscalar, (-1)^(sum of the positions of a's
        // generators), times the metric over a. For CB_MAP_DUAL_T (the
        // transpose, x -> the map whose matrix is the dual's transposed) the
        // factor of output m is the dual's factor of input m.
        const uint32_t a = (kind == CB_MAP_DUAL) ? (full ^ m) : m;
        const int pos_parity = __popc(a & 0xAAAAAAAAu) & 1;  // odd positions count once
        const int neg_parity = __popc(a & neg) & 1;
        return (pos_parity ^ neg_parity) ? -dual_scale : dual_scale;
    }
    }
}

__global__ void __launch_bounds__(256)
    blade_map_kernel(int kind, const float *__restrict__ x, float *__restrict__ out,
                     int64_t total, int n, uint32_t neg, int grade, float dual_scale, bool vec) {
    const uint32_t full = (1u << n) - 1;
    const bool dual = (kind == CB_MAP_DUAL || kind == CB_MAP_DUAL_T);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (vec) {  // 2^n >= 4, 16-byte aligned: float4 chunks, four blades each
        const int64_t chunks = total >> 2;
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        float4 *o4 = reinterpret_cast<float4 *>(out);
        for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks; c += stride) {
            const uint32_t m0 = (uint32_t)((c << 2) & full);
            float4 v;
            if (dual) {  // chunk of blades m0..m0+3 reads ~m0-3..~m0, reversed
                const int64_t row = (c << 2) >> n;
                const float4 r = x4[((row << n) + (full ^ (m0 + 3))) >> 2];
                v = make_float4(r.w, r.z, r.y, r.x);
            } else {
                v = x4[c];
            }
            v.x *= map_factor(kind, m0, full, neg, grade, dual_scale);
            v.y *= map_factor(kind, m0 + 1, full, neg, grade, dual_scale);
            v.z *= map_factor(kind, m0 + 2, full, neg, grade, dual_scale);
            v.w *= map_factor(kind, m0 + 3, full, neg, grade, dual_scale);
            o4[c] = v;
        }
        return;
    }
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const uint32_t m = (uint32_t)(e & full);
        const int64_t src = dual ? ((e & ~(int64_t)full) | (full ^ m)) : e;
        out[e] = x[src] * map_factor(kind, m, full, neg, grade, dual_scale);
    }
}

__device__ __forceinline__ float norm_weight(uint32_t b, uint32_t neg, uint32_t zero) {
    if (b & zero) return 0.0f;
    return (__popc(b & neg) & 1) ? -1.0f : 1.0f;
}

// norm_sq: one row per group of `lanes` consecutive lanes (lanes = min(32,
// 2^n / 4) float4 chunks in flight per row), each lane summing its chunks,
// then a shuffle tree over the group. 2^n >= 4 and 16-byte aligned rows.
__global__ void __launch_bounds__(256)
    norm_sq_kernel(const float *__restrict__ x, float *__restrict__ out, int64_t batch, int n,
                   uint32_t neg, uint32_t zero) {
    const int D = 1 << n;
    const int cpr = D >> 2;                   // float4 chunks per row
    const int lanes = cpr < 32 ? cpr : 32;    // lanes per row
    const int rows_per_warp = 32 / lanes;
    const int lane = threadIdx.x & 31;
    const int sub = lane / lanes, sl = lane % lanes;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (int64_t r0 = warp * rows_per_warp; r0 < batch; r0 += nwarps * rows_per_warp) {
        const int64_t row = r0 + sub;
        float s = 0.0f;
        if (row < batch) {
            for (int c = sl; c < cpr; c += lanes) {
                const float4 v = x4[row * cpr + c];
                const uint32_t b = (uint32_t)c << 2;
                s = fmaf(v.x * v.x, norm_weight(b, neg, zero), s);
                s = fmaf(v.y * v.y, norm_weight(b + 1, neg, zero), s);
                s = fmaf(v.z * v.z, norm_weight(b + 2, neg, zero), s);
                s = fmaf(v.w * v.w, norm_weight(b + 3, neg, zero), s);
            }
        }
        for (int off = lanes >> 1; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (row < batch && sl == 0) out[row] = s;
    }
}

// Scalar path of norm_sq for 2^n < 4 or unaligned rows: one row per thread.
__global__ void __launch_bounds__(256)
    norm_sq_scalar_kernel(const float *__restrict__ x, float *__restrict__ out, int64_t batch,
                          int n, uint32_t neg, uint32_t zero) {
    const int D = 1 << n;
    for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < batch;
         row += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int b = 0; b < D; ++b) {
            const float v = x[row * D + b];
            s = fmaf(v * v, norm_weight(b, neg, zero), s);
        }
        out[row] = s;
    }
}

// dx[row, b] = 2 w_b x[row, b] g[row]: the gradient of norm_sq.
__global__ void __launch_bounds__(256)
    norm_sq_bwd_kernel(const float *__restrict__ x, const float *__restrict__ g,
                       float *__restrict__ dx, int64_t total, int n, uint32_t neg, uint32_t zero) {
    const uint32_t full = (1u << n) - 1;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t b = (uint32_t)(e & full);
        dx[e] = 2.0f * norm_weight(b, neg, zero) * x[e] * g[e >> n];
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int n, int64_t batch, uint32_t neg, uint32_t zero, const void *x,
                 const void *out) {
    if (n < 1 || n > 24) {
        set_error("n = %d outside 1..24", n);
        return CB_ERR_UNSUPPORTED;
    }
    if (batch < 0) {
        set_error("negative batch");
        return CB_ERR_INVALID;
    }
    const uint32_t nmask = (uint32_t)((1ull << n) - 1);
    if ((neg & ~nmask) || (zero & ~nmask) || (neg & zero)) {
        set_error("metric masks invalid for n = %d (neg 0x%x, zero 0x%x)", n, neg, zero);
        return CB_ERR_INVALID;
    }
    if (batch > 0 && (!x || !out)) {
        set_error("null pointer");
        return CB_ERR_INVALID;
    }
    return CB_OK;
}

int grid_for(int64_t work) {
    DeviceInfo di;
    if (device_info(&di)) return -1;
    const int64_t blocks = (work + 255) / 256;
    return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)di.sm_count * 8));
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_blade_map(int kind, const float *x, float *out, int64_t batch, int n,
                            uint32_t neg_mask, uint32_t zero_mask, int grade, void *stream) {
    int st = check_common(n, batch, neg_mask, zero_mask, x, out);
    if (st) return st;
    if (kind < CB_MAP_REVERSE || kind > CB_MAP_DUAL_T) {
        set_error("map kind %d out of range", kind);
        return CB_ERR_INVALID;
    }
    const bool dual = (kind == CB_MAP_DUAL || kind == CB_MAP_DUAL_T);
    if (dual && zero_mask) {
        set_error("dual undefined for degenerate metrics");
        return CB_ERR_INVALID;
    }
    if (kind == CB_MAP_GRADE && (grade < 0 || grade > n)) {
        set_error("grade %d outside 0..%d", grade, n);
        return CB_ERR_INVALID;
    }
    if (dual && batch > 0 && x == out) {
        set_error("dual: out must not alias x");
        return CB_ERR_INVALID;
    }
    if (batch == 0) return CB_OK;
    // 1 / I^2 = I^2 = (-1)^(n(n-1)/2) (-1)^(#negative generators) for a
    // non-degenerate metric.
    const int isq_parity = ((n * (n - 1) / 2) + __builtin_popcount(neg_mask)) & 1;
    const float dual_scale = isq_parity ? -1.0f : 1.0f;
    const int64_t total = batch << n;
    const bool vec = n >= 2 && aligned16(x) && aligned16(out);
    const int grid = grid_for(vec ? total / 4 : total);
    if (grid < 0) return CB_ERR_CUDA;
    blade_map_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        kind, x, out, total, n, neg_mask, grade, dual_scale, vec);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch blade_map_kernel");
}

extern "C" int cb_norm_sq(const float *x, float *out, int64_t batch, int n, uint32_t neg_mask,
                          uint32_t zero_mask, void *stream) {
    int st = check_common(n, batch, neg_mask, zero_mask, x, out);
    if (st || batch == 0) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n >= 2 && aligned16(x)) {
        const int lanes = std::min(32, (1 << n) / 4);
        const int64_t warps = (batch + (32 / lanes) - 1) / (32 / lanes);
        const int grid = grid_for(warps * 32);
        if (grid < 0) return CB_ERR_CUDA;
        norm_sq_kernel<<<grid, 256, 0, s>>>(x, out, batch, n, neg_mask, zero_mask);
    } else {
        const int grid = grid_for(batch);
        if (grid < 0) return CB_ERR_CUDA;
        norm_sq_scalar_kernel<<<grid, 256, 0, s>>>(x, out, batch, n, neg_mask, zero_mask);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch norm_sq_kernel");
}

extern "C" int cb_norm_sq_bwd(const float *x, const float *g, float *dx, int64_t batch, int n,
                              uint32_t neg_mask, uint32_t zero_mask, void *stream) {
    int st = check_common(n, batch, neg_mask, zero_mask, x, dx);
    if (st || batch == 0) return st;
    if (!g) {
        set_error("null pointer");
        return CB_ERR_INVALID;
    }
    const int64_t total = batch << n;
    const int grid = grid_for(total);
    if (grid < 0) return CB_ERR_CUDA;
    norm_sq_bwd_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, g, dx, total, n,
                                                                           neg_mask, zero_mask);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch norm_sq_bwd_kernel");
}
