/*
 * ga_oracle.c -- CPU restatement of the reference's multivector-product
 * algorithm. TEST INFRASTRUCTURE ONLY: this file is the checker that the CUDA
 * path is compared against (tests/, the smoke check and the CPU-baseline leg
 * of bench.py). Nothing in the shipped library links or calls it.
 *
 * Every function restates a piece of the reference (paths relative to the
 * reference project root):
 *
 *   orc_sign           src/cliffordcuda/extensions/ga/geom_prod.py:44-74
 *                      (_build_sign_value_table: reorder parity over bit pairs
 *                      a > b, times the product of metric entries over i & j)
 *   orc_mask           _shared/_einsum_refs.py:58-83 (per-product masks)
 *   orc_product        _shared/_einsum_refs.py:26-55 (outer product, times the
 *                      signed mask, scatter-added to k = i ^ j) and, for the
 *                      backward sums, the chain rule written out at
 *                      src/cliffordcuda/extensions/ga/geom_prod.py:153-175
 *   orc_regressive_*   _shared/_einsum_refs.py:86-124 (dual o wedge o dual)
 *   orc_rotor_matrix   src/cliffordcuda/kernels/rotor/eigh_exp.cu:270-322
 *                      (Rm = expm(2 (M - M^T)), M[i][j] = beta_ij for i < j,
 *                      lex pair order, algebra.py:127); restated here with a
 *                      scaling-and-squaring Taylor series in double.
 *   orc_rotor_apply    src/cliffordcuda/kernels/rotor/givens_apply_mb_perm_packed.cu:8-70
 *                      with the Givens chain of givens_factor.cu:7-59; the
 *                      chain composes to the outermorphism of Rm^T, which is
 *                      what this function evaluates (blade minors).
 *
 * All arithmetic is double precision. Rows are independent and are split over
 * host threads by the Python wrapper (ctypes releases the GIL).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

enum { ORC_GP = 0, ORC_WEDGE = 1, ORC_INNER = 2, ORC_LC = 3, ORC_RC = 4 };
enum { ORC_FWD = 0, ORC_GRAD_A = 1, ORC_GRAD_B = 2 };

/* sigma(i, j) in {-1, 0, +1} for the metric (entries -1, 0, +1). */
int orc_sign(int n, const int *metric, uint32_t i, uint32_t j)
{
    int parity = 0;
    for (int a = 0; a < n; ++a) {
        if (!((i >> a) & 1u)) continue;
        for (int b = 0; b < a; ++b)
            parity += (int)((j >> b) & 1u);
    }
    int s = (parity & 1) ? -1 : 1;
    uint32_t common = i & j;
    for (int k = 0; k < n; ++k)
        if ((common >> k) & 1u) s *= metric[k];
    return s;
}

int orc_mask(int op, uint32_t i, uint32_t j)
{
    switch (op) {
    case ORC_GP:    return 1;
    case ORC_WEDGE: return (i & j) == 0;
    case ORC_INNER: return ((i & ~j) == 0) || ((j & ~i) == 0);
    case ORC_LC:    return (i & j) == i;
    case ORC_RC:    return (i & j) == j;
    default:        return 0;
    }
}

/* Full (D, D) signed-mask table, int8, row-major [i][j]. */
void orc_sign_table(int op, int n, const int *metric, int8_t *out)
{
    uint32_t D = 1u << n;
    for (uint32_t i = 0; i < D; ++i)
        for (uint32_t j = 0; j < D; ++j)
            out[(size_t)i * D + j] =
                (int8_t)(orc_mask(op, i, j) ? orc_sign(n, metric, i, j) : 0);
}

/*
 * mode FWD:    out[k] = sum_i T[i][i^k] * x[i] * y[i^k]      (x = a, y = b)
 * mode GRAD_A: out[k] = sum_i T[k][i]   * x[i] * y[k^i]      (x = b, y = g)
 * mode GRAD_B: out[k] = sum_i T[i][k]   * x[i] * y[k^i]      (x = a, y = g)
 * T is the signed-mask table of `op`.
 */
void orc_product(int op, int mode, int n, const int *metric, int64_t batch,
                 const double *x, const double *y, double *out)
{
    uint32_t D = 1u << n;
    int8_t *T = (int8_t *)malloc((size_t)D * D);
    orc_sign_table(op, n, metric, T);
    for (int64_t r = 0; r < batch; ++r) {
        const double *xr = x + r * D, *yr = y + r * D;
        double *o = out + r * D;
        for (uint32_t k = 0; k < D; ++k) {
            double acc = 0.0;
            for (uint32_t i = 0; i < D; ++i) {
                int s;
                if (mode == ORC_FWD)        s = T[(size_t)i * D + (i ^ k)];
                else if (mode == ORC_GRAD_A) s = T[(size_t)k * D + i];
                else                         s = T[(size_t)i * D + k];
                if (s) acc += (double)s * xr[i] * yr[i ^ k];
            }
            o[k] = acc;
        }
    }
    free(T);
}

/*
 * As orc_product for the outputs k in [k0, k1) only, with the sign evaluated
 * per term instead of from a (D, D) table, so that large n (the table is
 * 4^n bytes) and parallel splits over k stay cheap. The sign is the same
 * sigma as orc_sign: the reorder parity counts, for every generator a of i,
 * the generators of j below a (a popcount of j masked below a); the metric
 * multiplies over i & j.
 */
static int orc_sign_popc(uint32_t i, uint32_t j, uint32_t neg, uint32_t zero)
{
    uint32_t c = i & j;
    if (c & zero) return 0;
    int parity = __builtin_popcount(c & neg);
    for (uint32_t rest = i; rest; rest &= rest - 1) {
        int a = __builtin_ctz(rest);
        parity += __builtin_popcount(j & ((1u << a) - 1u));
    }
    return (parity & 1) ? -1 : 1;
}

void orc_product_range(int op, int mode, int n, const int *metric, int64_t batch,
                       const double *x, const double *y, double *out,
                       uint32_t k0, uint32_t k1)
{
    uint32_t D = 1u << n, neg = 0, zero = 0;
    for (int t = 0; t < n; ++t) {
        if (metric[t] == -1) neg |= 1u << t;
        if (metric[t] == 0) zero |= 1u << t;
    }
    for (int64_t r = 0; r < batch; ++r) {
        const double *xr = x + r * D, *yr = y + r * D;
        double *o = out + r * D;
        for (uint32_t k = k0; k < k1; ++k) {
            double acc = 0.0;
            for (uint32_t i = 0; i < D; ++i) {
                uint32_t P = (mode == ORC_GRAD_A) ? k : i;
                uint32_t Q = (mode == ORC_FWD) ? (i ^ k) : (mode == ORC_GRAD_A ? i : k);
                if (!orc_mask(op, P, Q)) continue;
                int s = orc_sign_popc(P, Q, neg, zero);
                if (s) acc += (double)s * xr[i] * yr[i ^ k];
            }
            o[k] = acc;
        }
    }
}

/* dual(x)[k] = x[~k] * sigma(~k, full) / I^2  (non-degenerate metrics only). */
void orc_dual_signs(int n, const int *metric, double *ds)
{
    uint32_t D = 1u << n, full = D - 1;
    double isq = (double)orc_sign(n, metric, full, full);
    for (uint32_t k = 0; k < D; ++k)
        ds[k] = (double)orc_sign(n, metric, full ^ k, full) / isq;
}

static void dual_rows(int n, const double *ds, int64_t batch,
                      const double *in, double *out)
{
    uint32_t D = 1u << n, full = D - 1;
    for (int64_t r = 0; r < batch; ++r)
        for (uint32_t k = 0; k < D; ++k)
            out[r * D + k] = ds[k] * in[r * D + (k ^ full)];
}

/* transpose of the dual map: (D^T y)[m] = ds[~m] * y[~m] */
static void dual_t_rows(int n, const double *ds, int64_t batch,
                        const double *in, double *out)
{
    uint32_t D = 1u << n, full = D - 1;
    for (int64_t r = 0; r < batch; ++r)
        for (uint32_t m = 0; m < D; ++m)
            out[r * D + m] = ds[m ^ full] * in[r * D + (m ^ full)];
}

/* regressive(a, b) = dual(wedge(dual a, dual b)) */
void orc_regressive_fwd(int n, const int *metric, int64_t batch,
                        const double *a, const double *b, double *out)
{
    uint32_t D = 1u << n;
    size_t sz = (size_t)batch * D;
    double *ds = malloc(D * sizeof(double));
    double *da = malloc(sz * sizeof(double)), *db = malloc(sz * sizeof(double));
    double *w = malloc(sz * sizeof(double));
    orc_dual_signs(n, metric, ds);
    dual_rows(n, ds, batch, a, da);
    dual_rows(n, ds, batch, b, db);
    orc_product(ORC_WEDGE, ORC_FWD, n, metric, batch, da, db, w);
    dual_rows(n, ds, batch, w, out);
    free(ds); free(da); free(db); free(w);
}

/* grads of regressive: ga = D^T Wga(D b, D^T g), gb = D^T Wgb(D a, D^T g) */
void orc_regressive_bwd(int n, const int *metric, int64_t batch,
                        const double *a, const double *b, const double *g,
                        double *ga, double *gb)
{
    uint32_t D = 1u << n;
    size_t sz = (size_t)batch * D;
    double *ds = malloc(D * sizeof(double));
    double *da = malloc(sz * sizeof(double)), *db = malloc(sz * sizeof(double));
    double *gt = malloc(sz * sizeof(double)), *t = malloc(sz * sizeof(double));
    orc_dual_signs(n, metric, ds);
    dual_rows(n, ds, batch, a, da);
    dual_rows(n, ds, batch, b, db);
    dual_t_rows(n, ds, batch, g, gt);
    orc_product(ORC_WEDGE, ORC_GRAD_A, n, metric, batch, db, gt, t);
    dual_t_rows(n, ds, batch, t, ga);
    orc_product(ORC_WEDGE, ORC_GRAD_B, n, metric, batch, da, gt, t);
    dual_t_rows(n, ds, batch, t, gb);
    free(ds); free(da); free(db); free(gt); free(t);
}

/* ---------------------------------------------------------------- rotor -- */

static void matmul_nn(int n, const double *A, const double *B, double *C)
{
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j) {
            double s = 0.0;
            for (int k = 0; k < n; ++k) s += A[i * n + k] * B[k * n + j];
            C[i * n + j] = s;
        }
}

/*
 * Rm = expm(Bm), Bm = 2 (M - M^T), M[p][q] = beta[idx(p, q)] for p < q in lex
 * order. Scaling and squaring: Bm / 2^s with ||Bm / 2^s||_1 <= 1/8, a 20-term
 * Taylor series (truncation far below double rounding at that norm), then s
 * squarings.
 */
void orc_rotor_matrix(int n, const double *beta, double *Rm)
{
    int nn = n * n;
    double *Bm = calloc(nn, sizeof(double));
    double *T = malloc(nn * sizeof(double)), *S = malloc(nn * sizeof(double));
    double *W = malloc(nn * sizeof(double));
    int idx = 0;
    for (int p = 0; p < n - 1; ++p)
        for (int q = p + 1; q < n; ++q, ++idx) {
            Bm[p * n + q] = 2.0 * beta[idx];
            Bm[q * n + p] = -2.0 * beta[idx];
        }
    double norm = 0.0;
    for (int j = 0; j < n; ++j) {
        double c = 0.0;
        for (int i = 0; i < n; ++i) c += fabs(Bm[i * n + j]);
        if (c > norm) norm = c;
    }
    int s = 0;
    while (norm > 0.125) { norm *= 0.5; ++s; }
    double scale = ldexp(1.0, -s);
    for (int i = 0; i < nn; ++i) Bm[i] *= scale;
    for (int i = 0; i < nn; ++i) { S[i] = 0.0; T[i] = 0.0; }
    for (int i = 0; i < n; ++i) { S[i * n + i] = 1.0; T[i * n + i] = 1.0; }
    for (int m = 1; m <= 20; ++m) {
        matmul_nn(n, T, Bm, W);
        for (int i = 0; i < nn; ++i) { T[i] = W[i] / (double)m; S[i] += T[i]; }
    }
    for (int k = 0; k < s; ++k) {
        matmul_nn(n, S, S, W);
        memcpy(S, W, nn * sizeof(double));
    }
    memcpy(Rm, S, nn * sizeof(double));
    free(Bm); free(T); free(S); free(W);
}

/* determinant of a k x k matrix (k <= 16), Gaussian elimination with
 * partial pivoting. */
static double det_small(int k, double *A)
{
    double det = 1.0;
    for (int c = 0; c < k; ++c) {
        int piv = c;
        for (int r = c + 1; r < k; ++r)
            if (fabs(A[r * k + c]) > fabs(A[piv * k + c])) piv = r;
        if (A[piv * k + c] == 0.0) return 0.0;
        if (piv != c) {
            for (int t = 0; t < k; ++t) {
                double tmp = A[c * k + t]; A[c * k + t] = A[piv * k + t]; A[piv * k + t] = tmp;
            }
            det = -det;
        }
        det *= A[c * k + c];
        for (int r = c + 1; r < k; ++r) {
            double f = A[r * k + c] / A[c * k + c];
            for (int t = c; t < k; ++t) A[r * k + t] -= f * A[c * k + t];
        }
    }
    return det;
}

/*
 * C[I][J] = det(Rm[I, J]) for blades of equal grade (rows I and columns J in
 * increasing generator order), 0 otherwise; y[J] = sum_I C[I][J] x[I] is the
 * outermorphism of Rm^T, i.e. y = R~ x R with the Euclidean product.
 */
void orc_rotor_blade_matrix(int n, const double *Rm, double *C)
{
    uint32_t D = 1u << n;
    double A[256];
    int ri[16], ci[16];
    for (uint32_t I = 0; I < D; ++I)
        for (uint32_t J = 0; J < D; ++J) {
            int gi = __builtin_popcount(I), gj = __builtin_popcount(J);
            double v = 0.0;
            if (gi == gj) {
                if (gi == 0) v = 1.0;
                else {
                    int a = 0, b = 0;
                    for (int t = 0; t < n; ++t) {
                        if ((I >> t) & 1u) ri[a++] = t;
                        if ((J >> t) & 1u) ci[b++] = t;
                    }
                    for (int r = 0; r < gi; ++r)
                        for (int c = 0; c < gi; ++c)
                            A[r * gi + c] = Rm[ri[r] * n + ci[c]];
                    v = det_small(gi, A);
                }
            }
            C[(size_t)I * D + J] = v;
        }
}

void orc_rotor_apply_matrix(int n, const double *C, int64_t batch,
                            const double *x, double *y)
{
    uint32_t D = 1u << n;
    for (int64_t r = 0; r < batch; ++r)
        for (uint32_t J = 0; J < D; ++J) {
            double s = 0.0;
            for (uint32_t I = 0; I < D; ++I) {
                double c = C[(size_t)I * D + J];
                if (c != 0.0) s += c * x[r * D + I];
            }
            y[r * D + J] = s;
        }
}
