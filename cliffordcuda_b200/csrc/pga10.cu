// pga10.cu -- the geometric product of Cl(9,0,1) (nine generators squaring to
// +1, the tenth, e9, to 0: the projective algebra of the Cl(9,0,1) benchmark
// configuration) through Cl(8,0) matrix products.
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
// So a sum is three Cl(9,0) sums of blocks, each two Cl(8,0) 16 x 16 x 16
// matrix products (pga10_kernel in gp_mat16.cu: the split into components in
// its gather, the merge in its epilogue), instead of the 4^10 blade terms of
// the direct sum; one launch runs the three of a sum. The backward sums follow
// by the chain rule through the same linear maps (the adjoint of x -> (X+, X-) is
// (P, Q) -> [P + Q | (P - Q) w]; g and right multiplication by w are
// orthogonal and their own adjoints):
//   grad_a0 = gA(b0; g0) + gA(b1; g1), grad_a1 = gA(g(b0); g1),
//   grad_b0 = gB(a0; g0) + g(gB(a1; g1)), grad_b1 = gB(a0; g1).
// Reference for the product itself: extensions/ga/geom_prod.py:216-276 (the
// blade-by-blade product and its autograd backward sums, geom_prod.py:241-250).
#include "common.cuh"

namespace cb {

bool use_pga10(int op, int n, uint32_t neg, uint32_t zero, const void *x, const void *y,
               const void *o) {
    auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return op == CB_OP_GP && n == 10 && neg == 0 && zero == (1u << 9) && al(x) && al(y) && al(o);
}

// One sum of the Cl(9,0,1) product; mode and (x, y) as in cb_bilinear: one
// launch of pga10_kernel (gp_mat16.cu), whose three stages compute the three
// block sums (the two that share an output block summed in the matrix domain;
// grad_b0's second term as g(gB(a1; g1)) = gB(g(a1); g(g1)), g being an
// orthogonal automorphism).
int pga10(int mode, const float *x, const float *y, float *out, int64_t batch, cudaStream_t s) {
    return pga10_sum(mode, x, y, out, batch, s);
}

}  // namespace cb
