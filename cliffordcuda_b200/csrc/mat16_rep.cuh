// mat16_rep.cuh -- the real 16 x 16 matrix representation of Cl(8,0) used by
// gp_mat16.cu: generator choice, register-slot and sign tables, all constexpr.
//
// Generators: tensor products of four real 2 x 2 Pauli factors I, X, Z, W = XZ
// (row index r = r1 r2 r3 r4, factor 1 most significant): G_0 = I(x)I(x)I(x)X,
// G_1 = I(x)I(x)I(x)Z, G_{2+i} = P_i (x) W with P_0..P_5 six mutually
// anticommuting 3-factor strings of square -1 (kP). Every G_i is symmetric,
// squares to 1, and the G_i anticommute.
#pragma once

namespace cb {
namespace mat16 {

// Real Pauli factor codes: I = 0, X = 1, Z = 2, W = 3 (bit 0: off-diagonal,
// bit 1: the Z part); the code of a product is the XOR of the codes.
__host__ __device__ constexpr inline int pauli_sign(int a, int b) {
    // a * b = pauli_sign(a, b) * (a ^ b)
    return (a == 2 && (b == 1 || b == 3)) || (a == 3 && (b == 1 || b == 3)) ? -1 : 1;
}

// P_0 .. P_5: codes of factors 1, 2, 3.
__host__ __device__ constexpr inline int kP(int i, int f) {
    constexpr int t[6][3] = {{0, 0, 3}, {0, 3, 1}, {1, 3, 2}, {2, 3, 2}, {3, 0, 2}, {3, 1, 1}};
    return t[i][f];
}

__host__ __device__ constexpr inline int popc8(int v) {
    int c = 0;
    for (int b = 0; b < 8; ++b) c += (v >> b) & 1;
    return c;
}

// Blade bits 2..7 (k, generators G_2..G_7): the register slot of the
// factor-1..3 string of E_I (codes of factors 1, 2, 3 at bits 4-5, 2-3, 0-1)
// and the sign of the ordered product P_i1 P_i2 ... relative to that string.
__host__ __device__ constexpr inline int slot_of(int k) {
    int c[3] = {0, 0, 0};
    for (int i = 0; i < 6; ++i)
        if ((k >> i) & 1)
            for (int f = 0; f < 3; ++f) c[f] ^= kP(i, f);
    return c[0] << 4 | c[1] << 2 | c[2];
}
__host__ __device__ constexpr inline int sig1_of(int k) {
    int c[3] = {0, 0, 0}, s = 1;
    for (int i = 0; i < 6; ++i)
        if ((k >> i) & 1)
            for (int f = 0; f < 3; ++f) {
                s *= pauli_sign(c[f], kP(i, f));
                c[f] ^= kP(i, f);
            }
    return s;
}

// Last factor of E_I: X^I0 Z^I1 W^m (m = popcount of blade bits 2..7) equals
// sign * (code q) with q = (I0 ^ m&1) | (I1 ^ m&1) << 1; the sign for lane q.
__host__ __device__ constexpr inline int last_sign(int q, int m) {
    const int pi = m & 1, i0 = (q & 1) ^ pi, i1 = ((q >> 1) & 1) ^ pi;
    int c = 0, s = 1;
    if (i0) { s *= pauli_sign(c, 1); c ^= 1; }
    if (i1) { s *= pauli_sign(c, 2); c ^= 2; }
    for (int t = 0; t < m; ++t) { s *= pauli_sign(c, 3); c ^= 3; }
    return s;
}

// Quadrant entry (i, j) (row 2i + r4, column 2j + c4) -> register slot:
// per factor f the code d | r << 1 with r = row bit, d = row bit ^ column bit.
__host__ __device__ constexpr inline int slot_ij(int i, int j) {
    const int d = i ^ j;
    int s = 0;
    for (int f = 0; f < 3; ++f) {
        const int r = (i >> (2 - f)) & 1, df = (d >> (2 - f)) & 1;
        s |= (df | r << 1) << (4 - 2 * f);
    }
    return s;
}

// Per product a 1168-byte region (292 floats, 16 bytes past a multiple of
// 128): it holds the padded input row (lane gathers then hit 32 distinct
// banks), then the matrix as four 8 x 8 blocks 288 bytes apart (a quarter
// warp's 128-bit stores and the product's 128-bit reads then hit distinct
// banks), then the output row.
}  // namespace mat16
}  // namespace cb
