/*
 * cliffordcuda_b200.h -- C ABI of the B200 (sm_100a) multivector-product
 * library. Plain pointers, sizes and bitmasks only; no torch types.
 *
 * Conventions shared by every entry point:
 *   - multivectors are row-major (batch, 2^n) fp32 arrays in bit-pattern blade
 *     order (blade index bit t set <=> generator e_t present);
 *   - the metric of Cl(p, q, r) is passed as two bitmasks: bit t of `neg_mask`
 *     set <=> e_t^2 = -1, bit t of `zero_mask` set <=> e_t^2 = 0 (all other
 *     generators square to +1). The reference passed packed sign/validity
 *     lookup tables instead; no table is needed here;
 *   - every pointer is device memory of the current CUDA device, allocated by
 *     the caller. The library never frees caller memory;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *     stream-ordered and asynchronous; no entry point synchronises the host
 *     unless its comment says so;
 *   - return value: CB_OK (0) or an error status. cb_last_error() returns a
 *     thread-local message for the last failure on the calling thread.
 *
 * Reference paths below are relative to the CliffordCUDA project root.
 */
#ifndef CLIFFORDCUDA_B200_H
#define CLIFFORDCUDA_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define CB_OK 0
#define CB_ERR_INVALID 1     /* bad argument (shape, op, mode, metric, alignment) */
#define CB_ERR_CUDA 2        /* a CUDA runtime / driver call failed */
#define CB_ERR_UNSUPPORTED 3 /* valid request outside what this build supports */
#define CB_ERR_DEVICE 4      /* a kernel reported a device-side failure (bounded wait expired) */

/* products */
#define CB_OP_GP 0    /* geometric product                 extensions/ga/geom_prod.py:253      */
#define CB_OP_WEDGE 1 /* outer product (i & j == 0)         extensions/ga/wedge_prod/chunk.py:105 */
#define CB_OP_INNER 2 /* Hestenes inner, scalars included   extensions/ga/inner_prod/chunk.py:101 */
#define CB_OP_LC 3    /* left contraction (i subset j)      extensions/ga/left_contract.py:121  */
#define CB_OP_RC 4    /* right contraction (j subset i)     extensions/ga/right_contract.py:76  */
#define CB_OP_REG 5   /* regressive (non-degenerate only)   extensions/ga/regressive_prod.py:186 */

/* sums */
#define CB_MODE_FWD 0    /* out[k] = sum_i s(i, i^k) x[i] y[i^k]; (x, y) = (a, b) */
#define CB_MODE_GRAD_A 1 /* out[k] = sum_i s(k, i)   x[i] y[k^i]; (x, y) = (b, g) */
#define CB_MODE_GRAD_B 2 /* out[k] = sum_i s(i, k)   x[i] y[k^i]; (x, y) = (a, g) */

/*
 * One batch-by-batch bilinear sum of product `op` (s = signed product mask).
 * Replaces the pybind entry points geom_prod_fwd (kernels/ga/geom_prod.cu:553-571),
 * wedge_prod_fwd (kernels/ga/wedge_prod.cu:220-224), inner_prod_fwd
 * (kernels/ga/inner_prod.cu:298-307) and contract_fwd (kernels/ga/contract.cu:203-208),
 * each of which the reference also called with transposed LUTs for its two
 * backward sums (extensions/ga/geom_prod.py:241-250). For CB_OP_REG it
 * replaces the geom_prod_fwd + index_select pair of regressive_prod.py:143-183.
 * x, y, out: (batch, 2^n); out must not alias x or y. 1 <= n <= 12.
 */
CB_API int cb_bilinear(int op, int mode, const float *x, const float *y, float *out,
                       int64_t batch, int n, uint32_t neg_mask, uint32_t zero_mask,
                       void *stream);

/*
 * As cb_bilinear, always through the blade-by-blade sum kernels: the sum
 * out[i ^ j] += s(i, j) x_i y_j evaluated term by term on the CUDA cores.
 * cb_bilinear takes faster routes for three geometric products: Euclidean
 * Cl(8,0) through its real 16 x 16 matrix representation; Cl(9,0,1)
 * (e0..e8 square to +1, e9 to 0) as dual numbers over Cl(9,0) =
 * Cl(8,0) + Cl(8,0), six 16 x 16 products per sum; and Cl(6,1) (e6 squares
 * to -1) as two Cl(6,0) sums through its central pseudoscalar (same results
 * to fp32 rounding). This entry point keeps the term-by-term kernels
 * reachable, for comparison and for callers that want them. Same reference
 * interface as cb_bilinear (extensions/ga/geom_prod.py:216-250 and its
 * siblings).
 */
CB_API int cb_bilinear_direct(int op, int mode, const float *x, const float *y, float *out,
                              int64_t batch, int n, uint32_t neg_mask, uint32_t zero_mask,
                              void *stream);

/*
 * Both backward sums of product `op` for upstream gradient g:
 * grad_a = cb_bilinear(op, GRAD_A, b, g), grad_b = cb_bilinear(op, GRAD_B, a, g).
 * Replaces the pair of geom_prod_fwd calls in the autograd backward of
 * extensions/ga/geom_prod.py:241-250 (and its wedge/inner/contract/regressive
 * counterparts). Either output may be NULL to skip it.
 */
CB_API int cb_bilinear_bwd(int op, const float *a, const float *b, const float *g,
                           float *grad_a, float *grad_b, int64_t batch, int n,
                           uint32_t neg_mask, uint32_t zero_mask, void *stream);

/* -------------------------------------------------------- blade maps --
 * One-pass per-blade maps of CliffordAlgebra on (batch, 2^n) rows, 1 <= n <= 24.
 * The factor of each blade comes from popcounts of its index; no tables.
 * The reference computed these as torch elementwise multiplies by cached
 * sign vectors (src/cliffordcuda/algebra.py:195-336); it had no kernel. */
#define CB_MAP_REVERSE 0   /* (-1)^(k(k-1)/2), k = grade        algebra.py:195-206 */
#define CB_MAP_INVOLUTE 1  /* (-1)^k                            algebra.py:278-286 */
#define CB_MAP_CONJUGATE 2 /* (-1)^(k(k+1)/2)                   algebra.py:288-296 */
#define CB_MAP_GRADE 3     /* keep grade `grade`, zero the rest algebra.py:298-307 */
#define CB_MAP_DUAL 4      /* x I^-1: out[m] = s(~m) x[~m]      algebra.py:208-266 */
#define CB_MAP_DUAL_T 5    /* transpose of the dual: out[m] = s(m) x[~m] (its backward) */

/*
 * out = map(x). `grade` is read only by CB_MAP_GRADE. The dual maps need a
 * non-degenerate metric (zero_mask = 0) and out != x; the other maps may run
 * in place (out == x). Replaces reverse / grade_involution /
 * clifford_conjugation / grade_projection / dual of
 * src/cliffordcuda/algebra.py:195-307 and the free function reverse of
 * extensions/ga/inverse.py:64-67.
 */
CB_API int cb_blade_map(int kind, const float *x, float *out, int64_t batch, int n,
                        uint32_t neg_mask, uint32_t zero_mask, int grade, void *stream);

/*
 * out[row] = sum_b x[row, b]^2 w_b, w_b = prod over the generators t of b of
 * metric[t] (+1, -1 or 0): the squared norm <x x~>_0 of every row, fp32.
 * Replaces CliffordAlgebra.norm_sq (src/cliffordcuda/algebra.py:309-336).
 */
CB_API int cb_norm_sq(const float *x, float *out, int64_t batch, int n, uint32_t neg_mask,
                      uint32_t zero_mask, void *stream);

/* Gradient of cb_norm_sq for upstream g (batch floats): dx = 2 w x g[row]. */
CB_API int cb_norm_sq_bwd(const float *x, const float *g, float *dx, int64_t batch, int n,
                          uint32_t neg_mask, uint32_t zero_mask, void *stream);

/* ---------------------------------------------------------------- layers --
 * Shared-weight product layers y = op(x, w), w (1, 2^n) shared by the batch
 * (reference layers.py:30-76). Because op is bilinear, y = x M(w); the
 * backward is dx = dy M^T and dw = fold(x^T dy). These run as 3xTF32 tcgen05
 * GEMMs for n = 7 and 8 (other n return CB_ERR_UNSUPPORTED).
 * `mats` (caller-owned, 4 * 4^n floats) holds M and M^T split into tf32 hi/lo.
 * The reference materialised w.expand_as(x) (layers.py:46) and ran the
 * batch-by-batch kernel, then summed the per-row weight gradients.
 */

/* Bytes of workspace cb_layer_prepare / cb_layer_backward need. */
CB_API int cb_layer_workspace_bytes(int n, int64_t batch, int64_t *bytes);

/* w -> mats for product `op` (any CB_OP_*) under the metric masks. */
CB_API int cb_layer_prepare(int op, const float *w, int n, uint32_t neg_mask, uint32_t zero_mask,
                            float *mats, void *workspace, int64_t workspace_bytes, void *stream);

/* y = x M(w), x and y (batch, 2^n). */
CB_API int cb_layer_forward(const float *mats, const float *x, float *y, int64_t batch, int n,
                            void *stream);

/* dx = dy M^T (skipped if dx is NULL); dw (2^n floats) = weight gradient
 * summed over the batch (skipped if dw is NULL). */
CB_API int cb_layer_backward(int op, const float *mats, const float *x, const float *dy, float *dx,
                             float *dw, int64_t batch, int n, uint32_t neg_mask,
                             uint32_t zero_mask, void *workspace, int64_t workspace_bytes,
                             void *stream);

/*
 * GeometricProductLayer of Cl(8,0) (Euclidean metric, n = 8) through the real
 * 16 x 16 matrix representation of the algebra: y = x w is rho(y) = rho(x) W
 * with W = rho(w), one 16 x 16 product per row with a fixed matrix, instead
 * of the 256 x 256 contraction; dx = rho^-1(rho(dy) W^T) and
 * dw = rho^-1(sum over rows of rho(x)^T rho(dy)). Same results as the
 * cb_layer_* route for this layer (to fp32 rounding). Replaces, for this
 * layer, the same reference path as cb_layer_* (layers.py:43-47).
 *   prepare:  w (256 floats) -> mats (the cb_layer_* buffer; 576 floats used)
 *   forward:  y = x w, rows 16-byte aligned
 *   backward: dx (skipped if NULL) and dw (skipped if NULL); workspace as
 *             sized by cb_layer_workspace_bytes(8, batch, ...)
 */
CB_API int cb_layer_gp8_prepare(const float *w, float *mats, void *stream);
CB_API int cb_layer_gp8_forward(const float *mats, const float *x, float *y, int64_t batch,
                                void *stream);
CB_API int cb_layer_gp8_backward(const float *mats, const float *x, const float *dy, float *dx,
                                 float *dw, int64_t batch, void *workspace,
                                 int64_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- rotors --
 * A compiled rotor is two caller-owned device buffers:
 *   cs    (fp32, cs_floats entries): per grade k = 0..n the C(n,k) x C(n,k)
 *         matrix C_k[I][J] = det(Rm[I, J]), row-major, grades concatenated,
 *         blades of a grade in increasing bit-pattern order;
 *   state (fp64, state_doubles entries): B = 2 (M - M^T), Rm = expm(B), and
 *         C_k in double precision, kept for the backward pass.
 * apply maps y_k = x_k C_k, i.e. y = R~ x R with the Euclidean product (the
 * metric is not used, as in the reference). 2 <= n <= 10.
 */

/* Sizes of the cs and state buffers for n generators. */
CB_API int cb_rotor_sizes(int n, int64_t *cs_floats, int64_t *state_doubles);

/*
 * beta (1, n(n-1)/2) lex-pair bivector -> cs, state. fp64.
 * Replaces eigh_exp_fwd (kernels/rotor/eigh_exp.cu:270-322) followed by
 * givens_factor_fwd_v2 (kernels/rotor/givens_factor.cu:7-59, :233-238).
 */
CB_API int cb_rotor_compile(const float *beta, int n, float *cs, double *state, void *stream);

/*
 * y = x C (transpose = 0) or y = x C^T (transpose = 1), per grade, over
 * (batch, 2^n) rows. Replaces givens_mb_perm_packed_fwd
 * (kernels/rotor/givens_apply_mb_perm_packed.cu:8-70, :295-300).
 */
CB_API int cb_rotor_apply(const float *cs, const float *x, float *y, int64_t batch, int n,
                          int transpose, void *stream);

/* Bytes of workspace cb_rotor_apply_bwd needs for this n and batch. */
CB_API int cb_rotor_workspace_bytes(int n, int64_t batch, int64_t *bytes);

/*
 * Backward of apply for upstream gradient g: dx = g C^T (skipped if dx is
 * NULL) and dcs = sum over the batch of x_k^T g_k (cs_floats entries).
 * `workspace` holds per-CTA partial sums (size from cb_rotor_workspace_bytes).
 * Replaces givens_mb_perm_packed_bwd (givens_apply_mb_perm_packed.cu:73-179,
 * which returned only the Givens-angle gradient and no dx).
 */
CB_API int cb_rotor_apply_bwd(const float *cs, const float *x, const float *g, float *dx,
                              float *dcs, int64_t batch, int n, void *workspace,
                              int64_t workspace_bytes, void *stream);

/*
 * cb_rotor_apply_bwd without a caller workspace; no counterpart in the
 * reference. For callers that cannot allocate device memory (a host program
 * binding only this C ABI with no device allocator of its own, or a framework
 * that owns all device memory in its own pool and forbids side allocations
 * inside a step). The per-CTA partial sums live in a fixed 8 MiB array inside
 * the library, held by every GPU that loads it until the process exits; it
 * covers n = 7 and 8 (other n return CB_ERR_UNSUPPORTED). Allocates nothing.
 * The first call on a device looks up that array's device address; make that
 * first call before any stream capture. All calls share the array, so calls
 * whose work overlaps on the GPU (other streams, other threads) race.
 */
CB_API int cb_rotor_apply_bwd_noalloc(const float *cs, const float *x, const float *g,
                                      float *dx, float *dcs, int64_t batch, int n,
                                      void *stream);

/*
 * dcs -> dbeta (n(n-1)/2 floats) through the minors and the matrix exponential.
 * One CTA, fp64. Replaces givens_factor_bwd_v2 (givens_factor.cu:61-174) and
 * eigh_exp_bwd (eigh_exp.cu:79-268, 325-361).
 */
CB_API int cb_rotor_compile_bwd(const double *state, const float *dcs, int n, float *dbeta,
                                void *stream);

/* Message of the last failure on this thread ("" if none). */
CB_API const char *cb_last_error(void);

/*
 * Synchronises `stream`, then returns CB_ERR_DEVICE (and clears the flag) if a
 * kernel of this library recorded a device-side failure since the last call,
 * else CB_OK. The reference had no counterpart (it raised from
 * C10_CUDA_KERNEL_LAUNCH_CHECK only, e.g. kernels/ga/geom_prod.cu:189).
 */
CB_API int cb_device_status(void *stream);

/*
 * Self-test of the failure path: launches one thread that waits, bounded by
 * `limit_us` microseconds, on a barrier nothing completes. The wait gives up, records a
 * device-side failure, and the next cb_device_status returns CB_ERR_DEVICE; the
 * context stays usable. No counterpart in the reference (it had no bounded
 * waits).
 */
CB_API int cb_selftest_bounded_wait(uint32_t limit_us, void *stream);

/* Library ABI version (major * 100 + minor). */
CB_API int cb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CLIFFORDCUDA_B200_H */
