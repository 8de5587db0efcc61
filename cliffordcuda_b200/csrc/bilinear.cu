// bilinear.cu -- entry points of the batch-by-batch products: argument
// checks, tiled/generic dispatch, and the generic kernel. The tiled kernel
// and its design notes are in bilinear_tiled.cuh.
#include <algorithm>
#include <cstdio>

#include "common.cuh"

namespace cb {

template <int MODE>
int bilinear_tiled(int op, const float *x, const float *y, float *out, int64_t batch, int n,
                   uint32_t neg, uint32_t zero, cudaStream_t stream);
template <int MODE>
int bilinear_tiled_cl61(const float *x, const float *y, float *out, int64_t batch,
                        cudaStream_t stream);
template <int MODE>
int bilinear_wide(int op, const float *x, const float *y, float *out, int64_t batch, int n,
                  uint32_t neg, uint32_t zero, cudaStream_t stream);

namespace {

constexpr int kThreads = 256;

// One block stages rows of x and y in shared memory and evaluates every term
// with the sign computed from popcounts. Used for metrics whose low five
// generators do not all square to +1, for n < 5, for pointers that are not
// 16-byte aligned, and for the regressive product (n <= 12; larger rows take
// bilinear_generic_global_kernel), evaluated as
// dual o wedge o dual (reference _shared/_einsum_refs.py:86-124) with the
// dual's signed reversal applied while staging and storing:
//   fwd:    X' = D a, Y' = D b,   out = D t
//   grad_*: X' = D x, Y' = D^T g, out = D^T t
// where (D v)[i] = f(i) v[~i], (D^T v)[i] = f(~i) v[~i], f(i) = s(~i, full) / I^2.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    bilinear_generic_kernel(int op, const float *__restrict__ x, const float *__restrict__ y,
                            float *__restrict__ out, int64_t batch, int n, uint32_t neg,
                            uint32_t zero) {
    extern __shared__ float gsm[];
    const int D = 1 << n;
    const uint32_t full = D - 1;
    const int rpb = D >= kThreads ? 1 : kThreads / D;  // rows per block pass
    const int tpr = kThreads / rpb;                    // threads per row
    float *xs = gsm;
    float *ys = gsm + rpb * D;
    const bool reg = (op == CB_OP_REG);
    const int base_op = reg ? CB_OP_WEDGE : op;
    const float inv_isq = reg ? (float)blade_sign(full, full, neg, zero) : 1.0f;  // 1/I^2 = I^2
    auto dual_sign = [&](uint32_t i) -> float {
        return (float)blade_sign(full ^ i, full, neg, zero) * inv_isq;
    };
    const int r = threadIdx.x / tpr;
    for (int64_t row0 = (int64_t)blockIdx.x * rpb; row0 < batch;
         row0 += (int64_t)gridDim.x * rpb) {
        for (int e = threadIdx.x; e < rpb * D; e += kThreads) {
            const int rr = e / D;
            const uint32_t i = e % D;
            const int64_t row = row0 + rr;
            float xv = 0.f, yv = 0.f;
            if (row < batch) {
                if (!reg) {
                    xv = x[row * D + i];
                    yv = y[row * D + i];
                } else {
                    xv = dual_sign(i) * x[row * D + (i ^ full)];
                    yv = (MODE == CB_MODE_FWD ? dual_sign(i) : dual_sign(i ^ full)) *
                         y[row * D + (i ^ full)];
                }
            }
            xs[e] = xv;
            ys[e] = yv;
        }
        __syncthreads();
        const int64_t row = row0 + r;
        const float *xr = xs + r * D;
        const float *yr = ys + r * D;
        for (uint32_t k = threadIdx.x % tpr; k < (uint32_t)D; k += tpr) {
            float acc = 0.f;
            for (uint32_t i = 0; i < (uint32_t)D; ++i) {
                const uint32_t j = i ^ k;
                const uint32_t P = (MODE == CB_MODE_GRAD_A) ? k : i;
                const uint32_t Q = (MODE == CB_MODE_FWD) ? j : (MODE == CB_MODE_GRAD_A ? i : k);
                if (!op_mask(base_op, P, Q)) continue;
                const int s = blade_sign(P, Q, neg, zero);
                if (s > 0) acc = fmaf(xr[i], yr[j], acc);
                if (s < 0) acc = fmaf(-xr[i], yr[j], acc);
            }
            if (row < batch) {
                if (!reg)
                    out[row * D + k] = acc;
                else if (MODE == CB_MODE_FWD)
                    out[row * D + (k ^ full)] = dual_sign(k ^ full) * acc;
                else
                    out[row * D + (k ^ full)] = dual_sign(k) * acc;
            }
        }
        __syncthreads();
    }
}

// As bilinear_generic_kernel for rows too large to stage (2^n > 4096): one
// thread per output coefficient, operands read through the caches (the
// lanes of a warp share x[i] and read 32 neighbouring y[i ^ k]).
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    bilinear_generic_global_kernel(int op, const float *__restrict__ x,
                                   const float *__restrict__ y, float *__restrict__ out,
                                   int64_t batch, int n, uint32_t neg, uint32_t zero) {
    const uint32_t D = 1u << n, full = D - 1;
    const bool reg = (op == CB_OP_REG);
    const int base_op = reg ? CB_OP_WEDGE : op;
    const float inv_isq = reg ? (float)blade_sign(full, full, neg, zero) : 1.0f;
    auto dual_sign = [&](uint32_t i) -> float {
        return (float)blade_sign(full ^ i, full, neg, zero) * inv_isq;
    };
    const int64_t total = batch << n;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = e >> n;
        const uint32_t k = (uint32_t)(e & full);
        const float *xr = x + row * D;
        const float *yr = y + row * D;
        float acc = 0.0f;
        for (uint32_t i = 0; i < D; ++i) {
            const uint32_t j = i ^ k;
            const uint32_t P = (MODE == CB_MODE_GRAD_A) ? k : i;
            const uint32_t Q = (MODE == CB_MODE_FWD) ? j : (MODE == CB_MODE_GRAD_A ? i : k);
            if (!op_mask(base_op, P, Q)) continue;
            const int s = blade_sign(P, Q, neg, zero);
            if (s == 0) continue;
            float xv, yv;
            if (!reg) {
                xv = xr[i];
                yv = yr[j];
            } else {
                xv = dual_sign(i) * xr[i ^ full];
                yv = (MODE == CB_MODE_FWD ? dual_sign(j) : dual_sign(j ^ full)) * yr[j ^ full];
            }
            acc = fmaf(s > 0 ? xv : -xv, yv, acc);
        }
        if (!reg)
            out[row * D + k] = acc;
        else if (MODE == CB_MODE_FWD)
            out[row * D + (k ^ full)] = dual_sign(k ^ full) * acc;
        else
            out[row * D + (k ^ full)] = dual_sign(k) * acc;
    }
}

template <int MODE>
int launch_generic(int op, const float *x, const float *y, float *out, int64_t batch, int n,
                   uint32_t neg, uint32_t zero, cudaStream_t stream) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    const int D = 1 << n;
    if (n > 12) {
        const int64_t total = batch << n;
        const int grid =
            (int)std::min<int64_t>((total + kThreads - 1) / kThreads, (int64_t)di.sm_count * 8);
        bilinear_generic_global_kernel<MODE>
            <<<grid, kThreads, 0, stream>>>(op, x, y, out, batch, n, neg, zero);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CB_OK : cuda_fail(e, "launch bilinear_generic_global_kernel");
    }
    const int rpb = D >= kThreads ? 1 : kThreads / D;
    const size_t smem = (size_t)2 * rpb * D * sizeof(float);
    auto kern = bilinear_generic_kernel<MODE>;
    if (smem > 48 * 1024) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bilinear_generic)");
    }
    const int64_t groups = (batch + rpb - 1) / rpb;
    const int grid = (int)std::min<int64_t>(groups, (int64_t)di.sm_count * 8);
    kern<<<grid, kThreads, smem, stream>>>(op, x, y, out, batch, n, neg, zero);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch bilinear_generic_kernel");
    return CB_OK;
}

bool use_tiled(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
               const void *o, int64_t batch) {
    if (n < 5 || n > 10) return false;
    if (zero & 31u) return false;  // no null generator among the low five
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!al(x) || !al(y) || !al(o)) return false;
    if ((uint64_t)batch * (1u << n) / 32 >= (1ull << 31)) return false;
    return true;
}

// The Cl(6,1) geometric product through two Cl(6,0) sums (bilinear_tiled.cuh,
// OPK_GP61): metric [1]*6 + [-1], the tiled kernel's alignment and size rules.
bool use_cl61(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
              const void *o, int64_t batch) {
    return op == CB_OP_GP && n == 7 && neg == (1u << 6) && zero == 0 &&
           use_tiled(op, n, neg, zero, x, y, o, batch);
}

// The large-n kernel (bilinear_wide.cuh): same sign requirements as the
// tiled one, 11 <= n <= 16.
bool use_wide(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
              const void *o, int64_t batch) {
    if (op == CB_OP_REG) return false;
    if (n < 11 || n > 16) return false;
    if ((neg | zero) & 31u) return false;
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!al(x) || !al(y) || !al(o)) return false;
    if ((uint64_t)batch * (1u << n) / 32 >= (1ull << 31)) return false;
    return true;
}

int check_args(int op, int mode, const void *x, const void *y, const void *out, int64_t batch,
               int n, uint32_t neg, uint32_t zero) {
    if (op < CB_OP_GP || op > CB_OP_REG) {
        set_error("op %d out of range", op);
        return CB_ERR_INVALID;
    }
    if (mode < CB_MODE_FWD || mode > CB_MODE_GRAD_B) {
        set_error("mode %d out of range", mode);
        return CB_ERR_INVALID;
    }
    if (n < 1 || n > 16) {
        set_error("n = %d outside 1..16", n);
        return CB_ERR_UNSUPPORTED;
    }
    if (batch < 0) {
        set_error("negative batch");
        return CB_ERR_INVALID;
    }
    const uint32_t nmask = (1u << n) - 1;
    if ((neg & ~nmask) || (zero & ~nmask) || (neg & zero)) {
        set_error("metric masks invalid for n = %d (neg 0x%x, zero 0x%x)", n, neg, zero);
        return CB_ERR_INVALID;
    }
    if (op == CB_OP_REG && zero) {
        set_error("regressive product undefined for degenerate metrics");
        return CB_ERR_INVALID;
    }
    if (batch > 0 && (!x || !y || !out)) {
        set_error("null pointer");
        return CB_ERR_INVALID;
    }
    if (batch > 0 && (out == x || out == y)) {
        set_error("out must not alias an input");
        return CB_ERR_INVALID;
    }
    return CB_OK;
}

}  // namespace

int bilinear(int op, int mode, const float *x, const float *y, float *out, int64_t batch, int n,
             uint32_t neg, uint32_t zero, cudaStream_t stream, bool direct) {
    int st = check_args(op, mode, x, y, out, batch, n, neg, zero);
    if (st || batch == 0) return st;
    if (!direct && use_mat16(op, n, neg, zero, x, y, out))
        return gp_mat16(mode, x, y, out, batch, stream);
    if (!direct && use_pga10(op, n, neg, zero, x, y, out))
        return pga10(mode, x, y, out, batch, stream);
    if (!direct && use_cl61(op, n, neg, zero, x, y, out, batch)) {
        switch (mode) {
        case CB_MODE_FWD: return bilinear_tiled_cl61<CB_MODE_FWD>(x, y, out, batch, stream);
        case CB_MODE_GRAD_A: return bilinear_tiled_cl61<CB_MODE_GRAD_A>(x, y, out, batch, stream);
        default: return bilinear_tiled_cl61<CB_MODE_GRAD_B>(x, y, out, batch, stream);
        }
    }
    if (use_tiled(op, n, neg, zero, x, y, out, batch)) {
        switch (mode) {
        case CB_MODE_FWD:
            return bilinear_tiled<CB_MODE_FWD>(op, x, y, out, batch, n, neg, zero, stream);
        case CB_MODE_GRAD_A:
            return bilinear_tiled<CB_MODE_GRAD_A>(op, x, y, out, batch, n, neg, zero, stream);
        default:
            return bilinear_tiled<CB_MODE_GRAD_B>(op, x, y, out, batch, n, neg, zero, stream);
        }
    }
    if (use_wide(op, n, neg, zero, x, y, out, batch)) {
        switch (mode) {
        case CB_MODE_FWD:
            return bilinear_wide<CB_MODE_FWD>(op, x, y, out, batch, n, neg, zero, stream);
        case CB_MODE_GRAD_A:
            return bilinear_wide<CB_MODE_GRAD_A>(op, x, y, out, batch, n, neg, zero, stream);
        default:
            return bilinear_wide<CB_MODE_GRAD_B>(op, x, y, out, batch, n, neg, zero, stream);
        }
    }
    switch (mode) {
    case CB_MODE_FWD:
        return launch_generic<CB_MODE_FWD>(op, x, y, out, batch, n, neg, zero, stream);
    case CB_MODE_GRAD_A:
        return launch_generic<CB_MODE_GRAD_A>(op, x, y, out, batch, n, neg, zero, stream);
    default:
        return launch_generic<CB_MODE_GRAD_B>(op, x, y, out, batch, n, neg, zero, stream);
    }
}

}  // namespace cb

extern "C" int cb_bilinear(int op, int mode, const float *x, const float *y, float *out,
                           int64_t batch, int n, uint32_t neg_mask, uint32_t zero_mask,
                           void *stream) {
    return cb::bilinear(op, mode, x, y, out, batch, n, neg_mask, zero_mask,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int cb_bilinear_direct(int op, int mode, const float *x, const float *y, float *out,
                                  int64_t batch, int n, uint32_t neg_mask, uint32_t zero_mask,
                                  void *stream) {
    return cb::bilinear(op, mode, x, y, out, batch, n, neg_mask, zero_mask,
                        static_cast<cudaStream_t>(stream), true);
}

extern "C" int cb_bilinear_bwd(int op, const float *a, const float *b, const float *g,
                               float *grad_a, float *grad_b, int64_t batch, int n,
                               uint32_t neg_mask, uint32_t zero_mask, void *stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = CB_OK;
    // grad_a is written before the grad_b sum reads a, so no output may alias
    // any of a, b, g or the other output, whatever kernel serves the call.
    if (batch > 0) {
        const void *outs[2] = {grad_a, grad_b};
        for (const void *o : outs)
            if (o && (o == a || o == b || o == g)) {
                cb::set_error("gradient outputs must not alias an input");
                return CB_ERR_INVALID;
            }
        if (grad_a && grad_a == grad_b) {
            cb::set_error("grad_a and grad_b must be different buffers");
            return CB_ERR_INVALID;
        }
    }
    if (grad_a && grad_b && cb::use_mat16(op, n, neg_mask, zero_mask, a, b, g) &&
        cb::use_mat16(op, n, neg_mask, zero_mask, grad_a, grad_b, g)) {
        st = cb::check_args(op, CB_MODE_GRAD_A, b, g, grad_a, batch, n, neg_mask, zero_mask);
        if (!st) st = cb::check_args(op, CB_MODE_GRAD_B, a, g, grad_b, batch, n, neg_mask, zero_mask);
        return st ? st : cb::gp_mat16_bwd(a, b, g, grad_a, grad_b, batch, s);
    }
    if (grad_a)
        st = cb::bilinear(op, CB_MODE_GRAD_A, b, g, grad_a, batch, n, neg_mask, zero_mask, s);
    if (st) return st;
    if (grad_b)
        st = cb::bilinear(op, CB_MODE_GRAD_B, a, g, grad_b, batch, n, neg_mask, zero_mask, s);
    return st;
}
