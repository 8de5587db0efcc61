// bilinear_tiled.cuh -- the tiled batch-by-batch bilinear kernel (fp32 FFMA
// on the CUDA cores), instantiated per sum in bilinear_tiled_{fwd,ga,gb}.cu.
//
// Every product of the reference (geometric, wedge, inner, left/right
// contraction) and both of its backward sums have the form
//
//     out[k] = sum_i  s(P, Q) * x[i] * y[i ^ k]
//
// with (P, Q) = (i, i^k) for the forward sum, (k, i) for grad_a and (i, k)
// for grad_b, and s = (blade sign of e_P e_Q) x (product predicate on P, Q)
// (reference: extensions/ga/geom_prod.py:216-250 -- the forward LUT and the
// two transposed backward LUTs -- and the masks of _shared/_einsum_refs.py).
//
// Blade indices split into a high part (bits 5..n-1) and a low part (bits
// 0..4). The sign factorises as
//     s(P, Q) = s_H(P_h, Q_h) * s_L(P_l, Q_l) * (-1)^(popc(P_h) * popc(Q_l))
// (every high generator of P passes every low generator of Q; none of the
// reverse pairs reorder), and every product predicate except the inner
// product's factorises the same way. The kernel therefore works on 32 x 32
// register blocks: a thread owns the 32 outputs of one high block k_h of one
// row and sweeps the high blocks i_h, each step doing up to 1024 FFMAs of
//     acc[k_l] += c(i_l, k_l) * x[i_h, i_l] * y'[i_h ^ k_h, i_l ^ k_l]
// whose coefficients c in {-1, 0, +1} are compile-time constants (one body per
// count of low generators squaring to -1, which a runtime relabelling moves
// to the top of the low block; null low generators take the generic kernel).
// The runtime high-part sign and predicate are folded into y' (32
// FMULs per step, read from a per-CTA table), and so is the y side of the
// (-1)^(popc * popc) cross term, which depends only on the parity of y's low
// index once the step is fixed. What remains of the cross term is a sign on
// the odd-parity x values (grad_b, 16 FMULs per step) or on the outputs
// (grad_a). One compile-time body per product and sum keeps the loop small
// enough for the instruction cache.
//
// Data movement: persistent CTAs of four warps; a tile is 4096 floats of x and
// of y (4096 / 2^n rows), brought in by 2-D TMA loads with 128-byte swizzle
// into a two-stage mbarrier pipeline. A row's threads share a warp, so each
// warp reads and writes only its own rows: after its sweep it writes its
// results into the consumed x tile (swizzled) and counts itself done on the
// stage; the last warp to finish issues the TMA store of the tile and the
// next load into the stage. No warp waits on another except through the
// pipeline (no CTA-wide barrier in the loop, no polling producer warp); the
// inner product's diagonal correction is a warp-shuffle reduction. A 32-float
// block is one 128-byte line, and the swizzle makes the XOR-indexed line reads
// of y (eight lanes of a quarter-warp on eight different lines) conflict-free.
//
// The inner product's predicate (P subset Q or Q subset P) does not factor;
// it is evaluated as left + right contraction minus the doubly counted
// P == Q terms. The sparse products (wedge, contractions, regressive) can run
// under a balanced step schedule (StepSched), and the Cl(6,1) geometric
// product runs as two Cl(6,0) sums per row (OPK_GP61); both are described
// where they are defined below.
#pragma once
#include <algorithm>
#include <map>
#include <mutex>
#include <cstdio>
#include <type_traits>
#include <utility>

#include "common.cuh"

namespace cb {
namespace tiled {

constexpr int kThreads = 128;                 // four warps
constexpr int kLow = 5;                       // low generators per block
constexpr int kBlk = 1 << kLow;               // 32 blades per block
constexpr int kTileFloats = kThreads * kBlk;  // 4096 floats per operand tile
constexpr int kTileLines = kTileFloats / 32;  // 128 lines of 128 bytes
constexpr int kTileBytes = kTileFloats * 4;
constexpr int kStages = 2;                    // tiles in flight per CTA

enum { OPK_GP = 0, OPK_WEDGE = 1, OPK_LC = 2, OPK_RC = 3, OPK_INNER = 4, OPK_REG = 5, OPK_GP61 = 6 };

__host__ __device__ constexpr int popcl(int v) {
    int c = 0;
    for (int a = 0; a < kLow; ++a) c += (v >> a) & 1;
    return c;
}

__host__ __device__ constexpr int reorderl(int p, int q) {
    int c = 0;
    for (int a = 0; a < kLow; ++a)
        if ((p >> a) & 1)
            for (int b = 0; b < a; ++b) c += (q >> b) & 1;
    return c & 1;
}

// Low generators that square to -1: NEGL of them, relabelled (see
// LowRelabel) to the top NEGL bits of the low block, so that the low block's
// metric is a compile-time pattern.
__host__ __device__ constexpr int low_neg_mask(int negl) {
    return ((1 << negl) - 1) << (kLow - negl);
}

// Coefficient of x[i_l] * y[i_l ^ k_l] in output k_l for the low block:
// reordering sign times the low metric over P_l & Q_l times the predicate.
template <int MODE, int OPK, int NEGL = 0>
__host__ __device__ constexpr int low_coef(int il, int kl) {
    const int jl = il ^ kl;
    const int P = (MODE == CB_MODE_GRAD_A) ? kl : il;
    const int Q = (MODE == CB_MODE_FWD) ? jl : (MODE == CB_MODE_GRAD_A ? il : kl);
    const bool m = (OPK == OPK_GP)      ? true
                   : (OPK == OPK_WEDGE) ? ((P & Q) == 0)
                   : (OPK == OPK_LC)    ? ((P & ~Q & (kBlk - 1)) == 0)
                                        : ((Q & ~P & (kBlk - 1)) == 0);
    if (!m) return 0;
    return (reorderl(P, Q) ^ (popcl(P & Q & low_neg_mask(NEGL)) & 1)) ? -1 : 1;
}

// Coefficient table of one body variant, evaluated by the compiler's
// constant evaluator; the FMA expansion below emits only the non-zero terms.
struct CoefTable {
    signed char c[kBlk * kBlk];
};

template <int MODE, int OPK, int NEGL>
__host__ __device__ constexpr CoefTable make_coefs() {
    CoefTable t{};
    for (int i = 0; i < kBlk * kBlk; ++i)
        t.c[i] = (signed char)low_coef<MODE, OPK, NEGL>(i / kBlk, i % kBlk);
    return t;
}

template <int MODE, int OPK, int NEGL>
struct Coefs {
    static constexpr CoefTable table = make_coefs<MODE, OPK, NEGL>();
};

template <int MODE, int OPK, int NEGL, int I>
__device__ __forceinline__ void fma_term(float (&acc)[kBlk], const float (&xv)[kBlk],
                                         const float (&yv)[kBlk]) {
    constexpr int il = I / kBlk, kl = I % kBlk;
    constexpr int c = Coefs<MODE, OPK, NEGL>::table.c[I];
    if constexpr (c > 0) acc[kl] = fmaf(xv[il], yv[il ^ kl], acc[kl]);
    else if constexpr (c < 0) acc[kl] = fmaf(-xv[il], yv[il ^ kl], acc[kl]);
}

template <int MODE, int OPK, int NEGL, int... I>
__device__ __forceinline__ void block_fma_seq(float (&acc)[kBlk], const float (&xv)[kBlk],
                                              const float (&yv)[kBlk],
                                              std::integer_sequence<int, I...>) {
    (fma_term<MODE, OPK, NEGL, I>(acc, xv, yv), ...);
}

// acc[k_l] += c(i_l, k_l) x[i_l] y[i_l ^ k_l] over the block, i_l outer.
template <int MODE, int OPK, int NEGL = 0>
__device__ __forceinline__ void block_fma(float (&acc)[kBlk], const float (&xv)[kBlk],
                                          const float (&yv)[kBlk]) {
    block_fma_seq<MODE, OPK, NEGL>(acc, xv, yv, std::make_integer_sequence<int, kBlk * kBlk>{});
}

// Relabelling of the five low generators that moves the ones squaring to -1
// to the top bits of the low block (positives keep their order below them).
// Within each 128-byte line the coefficient of blade i_l moves to to_new[i_l]
// and changes sign when the reordering of its generators is odd (bit i_l of
// eps); results move back through to_old. Identity when inactive.
struct LowRelabel {
    unsigned char to_new[kBlk];
    unsigned char to_old[kBlk];
    uint32_t eps;
    int active;
};

inline LowRelabel make_relabel(uint32_t negL) {
    LowRelabel r{};
    int pos[kLow];
    int next = 0;
    for (int b = 0; b < kLow; ++b)
        if (!((negL >> b) & 1)) pos[b] = next++;
    for (int b = 0; b < kLow; ++b)
        if ((negL >> b) & 1) pos[b] = next++;
    r.active = 0;
    for (int b = 0; b < kLow; ++b) r.active |= pos[b] != b;
    r.eps = 0;
    for (int il = 0; il < kBlk; ++il) {
        int nw = 0, inv = 0;
        for (int a = 0; a < kLow; ++a) {
            if (!((il >> a) & 1)) continue;
            nw |= 1 << pos[a];
            for (int b = a + 1; b < kLow; ++b)
                if (((il >> b) & 1) && pos[a] > pos[b]) ++inv;
        }
        r.to_new[il] = (unsigned char)nw;
        r.to_old[nw] = (unsigned char)il;
        if (inv & 1) r.eps |= 1u << il;
    }
    return r;
}


// Swizzled shared tile: float f of the tile lives in 128-byte line f >> 5, in
// 16-byte chunk ((f >> 2) & 7) ^ (line & 7) -- the TMA 128B swizzle pattern.
// A block is one whole line.
__device__ __forceinline__ void load_block(const float *tile, int line, float (&v)[kBlk]) {
    const float *lp = tile + line * 32;
    const int sw = line & 7;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const float4 q = *reinterpret_cast<const float4 *>(lp + ((t ^ sw) << 2));
        v[4 * t + 0] = q.x;
        v[4 * t + 1] = q.y;
        v[4 * t + 2] = q.z;
        v[4 * t + 3] = q.w;
    }
}

__device__ __forceinline__ void store_block(float *tile, int line, const float (&v)[kBlk]) {
    float *lp = tile + line * 32;
    const int sw = line & 7;
#pragma unroll
    for (int t = 0; t < 8; ++t)
        *reinterpret_cast<float4 *>(lp + ((t ^ sw) << 2)) =
            make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
}

__device__ __forceinline__ int swz_index(int f) {
    const int line = f >> 5;
    return line * 32 + ((((f >> 2) & 7) ^ (line & 7)) << 2) + (f & 3);
}

// Offset of float e of line `line` within a swizzled tile.
__device__ __forceinline__ int swz_off(int line, int e) {
    return line * 32 + ((((e >> 2) & 7) ^ (line & 7)) << 2) + (e & 3);
}

// In place on line `line` of a swizzled tile: x'[to_new[i]] = eps(i) x[i].
__device__ __forceinline__ void relabel_line(float *tile, int line, const LowRelabel &rl) {
    float v[kBlk];
#pragma unroll
    for (int e = 0; e < kBlk; ++e) v[e] = tile[swz_off(line, e)];
#pragma unroll
    for (int e = 0; e < kBlk; ++e)
        tile[swz_off(line, rl.to_new[e])] = ((rl.eps >> e) & 1) ? -v[e] : v[e];
}

// Store this thread's 32 sums (relabelled order) into line `line` in the
// caller's order: out[i] = eps(i) acc[to_new[i]], i.e. acc[r] goes to to_old[r].
__device__ __forceinline__ void store_block_relabel(float *tile, int line, const float (&acc)[kBlk],
                                                    const LowRelabel &rl) {
#pragma unroll
    for (int r = 0; r < kBlk; ++r) {
        const int o = rl.to_old[r];
        tile[swz_off(line, o)] = ((rl.eps >> o) & 1) ? -acc[r] : acc[r];
    }
}

// The regressive product is dual o wedge o dual (the dual x I^-1 is a signed
// reversal of a row). Its dual steps move line L of a row to line NH-1-L,
// float e to 31 - e, with the factor I^2 (-1)^popc(P & dmask) of P = the source
// blade index (comp = false) or its complement (comp = true), where
// dmask = odd positions xor the negative generators: e_P I = that factor
// times e_~P up to the I^2 of I^-1.
__device__ __forceinline__ void dual_move(const float (&v)[kBlk], float *tile, int dst_line,
                                          uint32_t src_base, uint32_t full, uint32_t dmask,
                                          float isq, bool comp) {
#pragma unroll
    for (int e = 0; e < kBlk; ++e) {
        const uint32_t P = comp ? (full ^ (src_base + e)) : (src_base + e);
        const float f = (__popc(P & dmask) & 1) ? -isq : isq;
        tile[swz_off(dst_line, kBlk - 1 - e)] = f * v[e];
    }
}

__device__ __forceinline__ void apply_sign(float (&yv)[kBlk], float2 sg) {
#pragma unroll
    for (int e = 0; e < kBlk; ++e) yv[e] *= (popcl(e) & 1) ? sg.y : sg.x;
}

// High-part factor of the step (i_h, k_h) for one predicate: the blade sign
// of the high parts times the high-part predicate (.x, for even-parity y
// elements); .y adds the y side of the cross term for odd-parity y elements:
// (-1)^popc(i_h) for the forward sum and grad_b, (-1)^popc(k_h) for grad_a.
__host__ __device__ __forceinline__ float2 high_factor(int mode, int opk, uint32_t ih, uint32_t kh,
                                              uint32_t negH, uint32_t zeroH) {
    const uint32_t jh = ih ^ kh;
    const uint32_t P = (mode == CB_MODE_GRAD_A) ? kh : ih;
    const uint32_t Q = (mode == CB_MODE_FWD) ? jh : (mode == CB_MODE_GRAD_A ? ih : kh);
    bool m = true;
    if (opk == OPK_WEDGE) m = (P & Q) == 0;
    if (opk == OPK_LC) m = (P & ~Q) == 0;
    if (opk == OPK_RC) m = (Q & ~P) == 0;
    const float s = m ? (float)blade_sign(P, Q, negH, zeroH) : 0.0f;
    const float so = parity(mode == CB_MODE_GRAD_A ? kh : ih) ? -s : s;
    return make_float2(s, so);
}

__host__ __device__ inline size_t table_entries(int n, bool inner) {
    const size_t nh = size_t(1) << (n - kLow);
    return nh * nh * (inner ? 2 : 1);
}

// Balanced step schedule of the sparse products (wedge, contractions,
// regressive). Output block k_h has cnt(k_h) steps with a non-zero high-part
// factor, and these counts differ widely (for the left contraction's forward
// sum, 2^(#high generators not in k_h)): a lane that owns block k_h alone
// runs cnt(k_h) steps while its warp waits for the largest count. The
// schedule moves the tail of each heavy block's step list to lanes whose own
// list is short. Such a lane runs its borrowed segment first, parks that sum
// in a second accumulator, then runs its own steps; after the sweep the
// parked sums pass through the row's (then dead) y lines to the owning lane,
// which adds them in ascending donor order, so results stay deterministic.
// A lane borrows at most one segment. Steps per lane: ih[t * NH + lane],
// t < ntot[lane], the first nsec[lane] of them for block sec_kh[lane].
constexpr int kMaxNH = 32;
struct StepSched {
    unsigned char ih[kMaxNH * kMaxNH];
    unsigned char nsec[kMaxNH], ntot[kMaxNH], sec_kh[kMaxNH], pad_[kMaxNH];
    uint32_t donors[kMaxNH];  // lanes whose borrowed segment is for this block
    int T;                    // steps of the longest lane; 0: dense sweep
    int pad2_[3];
};

// Shared-memory bank conflicts of a round: the eight lanes of a quarter-warp
// read eight lines at once, and lines whose indices agree in the low three
// bits (the swizzle phase) but differ collide unless they are the same line.
inline int round_conflicts(const int *lines, int nl) {
    int cost = 0;
    for (int q0 = 0; q0 < nl; q0 += 8) {
        for (int ph = 0; ph < 8; ++ph) {
            int distinct[8], nd = 0;
            for (int l = q0; l < q0 + 8 && l < nl; ++l) {
                if (lines[l] < 0 || (lines[l] & 7) != ph) continue;
                bool seen = false;
                for (int d = 0; d < nd; ++d) seen |= distinct[d] == lines[l];
                if (!seen) distinct[nd++] = lines[l];
            }
            if (nd > 1) cost += nd - 1;
        }
    }
    return cost;
}

// Reorders each lane's steps within its borrowed and its own segment (the
// sums do not depend on the order beyond rounding) so that the lanes of a
// round read x lines (i_h) and y lines (i_h ^ k_h) with few bank conflicts:
// greedy, round by round.
inline void order_steps(StepSched &t, int NH) {
    unsigned char out[kMaxNH * kMaxNH];
    bool used[kMaxNH][kMaxNH] = {};
    for (int r = 0; r < t.T; ++r) {
        int xl[kMaxNH], yl[kMaxNH];
        for (int L = 0; L < NH; ++L) xl[L] = yl[L] = -1;
        for (int L = 0; L < NH; ++L) {
            if (r >= t.ntot[L]) continue;
            const bool sec = r < t.nsec[L];
            const int lo = sec ? 0 : t.nsec[L], hi = sec ? t.nsec[L] : t.ntot[L];
            const int k = sec ? t.sec_kh[L] : L;
            int best = -1, best_cost = 1 << 30;
            for (int c = lo; c < hi; ++c) {
                if (used[L][c]) continue;
                const int ih = t.ih[c * NH + L];
                xl[L] = ih;
                yl[L] = ih ^ k;
                const int cost = round_conflicts(xl, L + 1) + round_conflicts(yl, L + 1);
                if (cost < best_cost) {
                    best_cost = cost;
                    best = c;
                }
            }
            used[L][best] = true;
            const int ih = t.ih[best * NH + L];
            xl[L] = ih;
            yl[L] = ih ^ k;
            out[r * NH + L] = (unsigned char)ih;
        }
    }
    for (int L = 0; L < NH; ++L)
        for (int r = 0; r < t.ntot[L]; ++r) t.ih[r * NH + L] = out[r * NH + L];
    // then swaps of two steps of one lane's segment while they lower the
    // conflicts of the two rounds involved
    auto cost_of = [&](int r) {
        int xl[kMaxNH], yl[kMaxNH];
        for (int L = 0; L < NH; ++L) {
            xl[L] = yl[L] = -1;
            if (r < t.ntot[L]) {
                xl[L] = t.ih[r * NH + L];
                yl[L] = xl[L] ^ (r < t.nsec[L] ? t.sec_kh[L] : L);
            }
        }
        return round_conflicts(xl, NH) + round_conflicts(yl, NH);
    };
    for (int pass = 0; pass < 8; ++pass) {
        bool improved = false;
        for (int L = 0; L < NH; ++L)
            for (int r1 = 0; r1 < t.ntot[L]; ++r1)
                for (int r2 = r1 + 1; r2 < t.ntot[L]; ++r2) {
                    if ((r1 < t.nsec[L]) != (r2 < t.nsec[L])) continue;
                    const int before = cost_of(r1) + cost_of(r2);
                    std::swap(t.ih[r1 * NH + L], t.ih[r2 * NH + L]);
                    if (cost_of(r1) + cost_of(r2) < before) {
                        improved = true;
                    } else {
                        std::swap(t.ih[r1 * NH + L], t.ih[r2 * NH + L]);
                    }
                }
        if (!improved) break;
    }
}

// Builds the schedule for one sum; inactive (T = 0) unless it cuts the
// longest lane's steps by 1.5x or more: the scheduled sweep reads x lines that
// differ across lanes (no broadcast) and parks a second sum, which costs more
// than it saves where the sum is bound by HBM (the sparse products at n <= 7).
inline StepSched make_sched(int mode, int opk, int n, uint32_t neg, uint32_t zero) {
    StepSched s{};
    if (opk == OPK_GP || opk == OPK_INNER) return s;
    const int opb = opk == OPK_REG ? OPK_WEDGE : opk;
    const int lgNH = n - kLow, NH = 1 << lgNH;
    const uint32_t negH = neg >> kLow, zeroH = zero >> kLow;
    unsigned char list[kMaxNH][kMaxNH];
    int cnt[kMaxNH] = {}, total = 0, maxc = 0;
    for (int k = 0; k < NH; ++k) {
        for (int ih = 0; ih < NH; ++ih)
            if (high_factor(mode, opb, ih, k, negH, zeroH).x != 0.0f) list[k][cnt[k]++] = ih;
        total += cnt[k];
        maxc = std::max(maxc, cnt[k]);
    }
    for (int T = (total + NH - 1) / NH; 3 * T <= 2 * maxc; ++T) {
        int keep[kMaxNH], cap[kMaxNH], order[kMaxNH];
        for (int k = 0; k < NH; ++k) {
            keep[k] = std::min(cnt[k], T);
            cap[k] = std::max(0, T - cnt[k]);
            order[k] = k;
        }
        // heavy blocks by excess and donors by spare capacity, largest first
        std::sort(order, order + NH, [&](int a, int b) {
            return cnt[a] != cnt[b] ? cnt[a] > cnt[b] : a < b;
        });
        StepSched t{};
        int next_donor = NH - 1;  // order[] from the end: the lightest lanes
        bool ok = true;
        for (int h = 0; h < NH && ok; ++h) {
            const int k = order[h];
            int pos = keep[k];
            while (pos < cnt[k]) {
                while (next_donor >= 0 && cap[order[next_donor]] == 0) --next_donor;
                if (next_donor < 0) {
                    ok = false;
                    break;
                }
                const int d = order[next_donor--];
                const int seg = std::min(cap[d], cnt[k] - pos);
                t.sec_kh[d] = (unsigned char)k;
                t.nsec[d] = (unsigned char)seg;
                for (int q = 0; q < seg; ++q) t.ih[q * NH + d] = list[k][pos + q];
                t.donors[k] |= 1u << d;
                pos += seg;
            }
        }
        if (!ok) continue;
        for (int k = 0; k < NH; ++k) {
            for (int q = 0; q < keep[k]; ++q) t.ih[(t.nsec[k] + q) * NH + k] = list[k][q];
            t.ntot[k] = (unsigned char)(t.nsec[k] + keep[k]);
        }
        t.T = T;
        order_steps(t, NH);
        return t;
    }
    return s;
}

// The schedule for one sum, built once per (sum, product, n, metric).
inline StepSched cached_sched(int mode, int opk, int n, uint32_t neg, uint32_t zero) {
    static std::mutex mu;
    static std::map<uint64_t, StepSched> cache;
    const uint64_t key = ((uint64_t)neg << 32) ^ ((uint64_t)zero << 12) ^ (uint64_t)(mode << 8) ^
                         (uint64_t)(opk << 4) ^ (uint64_t)n;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    const StepSched s = make_sched(mode, opk, n, neg, zero);
    cache.emplace(key, s);
    return s;
}

// Balanced schedule of the inner product (left + right contraction): its two
// bodies run in separate phases, LC rounds then RC rounds, so in every round
// the whole warp runs one body (the row-major sweep runs both bodies on every
// step, since the lane of line 0 needs both). Each phase is balanced as
// StepSched does; a lane borrows at most one segment over both phases. A
// segment borrowed in the LC phase runs first and is parked in the second
// accumulator; one borrowed in the RC phase runs in the first accumulator
// while the lane's own partial sum waits in the second. Steps of lane L in
// phase p: ih[p][t * NH + L], t < n[p][L], the first nsec[L] of them (if
// sec_ph[L] == p) for line sec_kh[L].
struct InnerSched {
    unsigned char ih[2][kMaxNH * kMaxNH];
    unsigned char n[2][kMaxNH];
    unsigned char nsec[kMaxNH], sec_kh[kMaxNH], sec_ph[kMaxNH], pad_[kMaxNH];
    uint32_t donors[kMaxNH];
    int T[2];  // rounds per phase; T[0] = 0: the row-major sweep
    int pad2_[2];
};

inline InnerSched make_inner_sched(int mode, int n, uint32_t neg, uint32_t zero) {
    InnerSched none{};
    const int lgNH = n - kLow, NH = 1 << lgNH;
    const uint32_t negH = neg >> kLow, zeroH = zero >> kLow;
    unsigned char list[2][kMaxNH][kMaxNH];
    int cnt[2][kMaxNH] = {}, tot[2] = {0, 0}, maxc[2] = {0, 0};
    for (int ph = 0; ph < 2; ++ph)
        for (int k = 0; k < NH; ++k) {
            for (int ih = 0; ih < NH; ++ih)
                if (high_factor(mode, ph == 0 ? OPK_LC : OPK_RC, ih, k, negH, zeroH).x != 0.0f)
                    list[ph][k][cnt[ph][k]++] = (unsigned char)ih;
            tot[ph] += cnt[ph][k];
            maxc[ph] = std::max(maxc[ph], cnt[ph][k]);
        }
    const int base[2] = {(tot[0] + NH - 1) / NH, (tot[1] + NH - 1) / NH};
    // The row-major sweep runs NH steps of both bodies and loads each step's
    // lines once for both; one body per round costs its own loads and signs,
    // so the schedule pays only well below that: at most 45 % of the body runs
    // (measured fwd + both grads: n = 9, 0.60 -> 0.44 ms; n = 10, 1.22 -> 0.67
    // ms, 0.52 ms with a null generator; n = 7 (75 %) slower, 0.34 -> 0.42 ms).
    for (int extra = 0; 20 * (base[0] + base[1] + extra) <= 9 * 2 * NH; ++extra) {
        for (int e0 = 0; e0 <= extra; ++e0) {
            const int T[2] = {std::min(base[0] + e0, maxc[0]), std::min(base[1] + extra - e0, maxc[1])};
            InnerSched t{};
            bool borrowed[kMaxNH] = {};
            bool ok = true;
            for (int ph = 0; ph < 2 && ok; ++ph) {
                int order[kMaxNH];
                for (int k = 0; k < NH; ++k) order[k] = k;
                std::sort(order, order + NH, [&](int a, int b) {
                    return cnt[ph][a] != cnt[ph][b] ? cnt[ph][a] > cnt[ph][b] : a < b;
                });
                int keep[kMaxNH];
                for (int k = 0; k < NH; ++k) keep[k] = std::min(cnt[ph][k], T[ph]);
                for (int h = 0; h < NH && ok; ++h) {
                    const int k = order[h];
                    int pos = keep[k];
                    while (pos < cnt[ph][k]) {
                        int d = -1;  // the lightest lane still free to borrow
                        for (int c = NH - 1; c >= 0; --c) {
                            const int cand = order[c];
                            if (!borrowed[cand] && cnt[ph][cand] < T[ph]) {
                                d = cand;
                                break;
                            }
                        }
                        if (d < 0) {
                            ok = false;
                            break;
                        }
                        const int seg = std::min(T[ph] - cnt[ph][d], cnt[ph][k] - pos);
                        borrowed[d] = true;
                        t.sec_kh[d] = (unsigned char)k;
                        t.sec_ph[d] = (unsigned char)ph;
                        t.nsec[d] = (unsigned char)seg;
                        for (int q = 0; q < seg; ++q) t.ih[ph][q * NH + d] = list[ph][k][pos + q];
                        t.donors[k] |= 1u << d;
                        pos += seg;
                    }
                }
                if (!ok) break;
                for (int k = 0; k < NH; ++k) {
                    const int off = (borrowed[k] && t.sec_ph[k] == ph) ? t.nsec[k] : 0;
                    for (int q = 0; q < keep[k]; ++q) t.ih[ph][(off + q) * NH + k] = list[ph][k][q];
                    t.n[ph][k] = (unsigned char)(off + keep[k]);
                }
            }
            if (!ok) continue;
            t.T[0] = std::max(T[0], 1);
            t.T[1] = std::max(T[1], 1);
            return t;
        }
    }
    return none;
}

inline InnerSched cached_inner_sched(int mode, int n, uint32_t neg, uint32_t zero) {
    static std::mutex mu;
    static std::map<uint64_t, InnerSched> cache;
    const uint64_t key = ((uint64_t)neg << 32) ^ ((uint64_t)zero << 12) ^ (uint64_t)(mode << 8) ^
                         (uint64_t)n;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    const InnerSched s = make_inner_sched(mode, n, neg, zero);
    cache.emplace(key, s);
    return s;
}

// The dense sweep's kernels take this in place of a StepSched (no parameter
// space or shared memory spent on a schedule they do not use).
struct NoSched {
    int T;
};

__host__ __device__ inline size_t smem_bytes(int n, bool inner, size_t sched_bytes = 0) {
    return 1024 /* alignment slack */ + 2 * kStages * size_t(kTileBytes) +
           table_entries(n, inner) * sizeof(float2) + 64 + sched_bytes;
}

template <int MODE, int OPK, int NEGL>
__device__ __forceinline__ void sweep(float (&acc)[kBlk], const float *xt, const float *yt,
                                      const float2 *tab, const float2 *tab2, int rowl, int kh,
                                      int lgNH, bool skip_zero) {
    const int NH = 1 << lgNH;
#pragma unroll 1
    for (int ih = 0; ih < NH; ++ih) {
        const int jh = ih ^ kh;
        const float2 sg = tab[(ih << lgNH) | kh];
        const float2 sg2 = OPK == OPK_INNER ? tab2[(ih << lgNH) | kh] : make_float2(0.0f, 0.0f);
        // A step whose high-part factor is zero for the whole warp (a null
        // generator in both high parts, or the product's predicate) adds
        // nothing: skip its loads and FMAs. Enabled where such steps occur
        // (skip_zero, warp-uniform): a warp then spans at most half the
        // high-block outputs of a row, or a null generator sits in the high bits.
        if (skip_zero &&
            __all_sync(0xffffffffu, sg.x == 0.0f && sg.y == 0.0f && sg2.x == 0.0f && sg2.y == 0.0f))
            continue;
        float xv[kBlk], yv[kBlk];
        load_block(xt, rowl + ih, xv);
        load_block(yt, rowl + jh, yv);
        if (MODE == CB_MODE_GRAD_B) {  // x side of the cross term
            const float sx = parity(ih) ? -1.0f : 1.0f;
#pragma unroll
            for (int e = 0; e < kBlk; ++e)
                if (popcl(e) & 1) xv[e] *= sx;
        }
        if (OPK == OPK_INNER) {
            float y2[kBlk];
#pragma unroll
            for (int e = 0; e < kBlk; ++e) y2[e] = yv[e];
            apply_sign(yv, sg);
            apply_sign(y2, sg2);
            block_fma<MODE, OPK_LC, NEGL>(acc, xv, yv);
            block_fma<MODE, OPK_RC, NEGL>(acc, xv, y2);
        } else {
            apply_sign(yv, sg);
            block_fma<MODE, OPK, NEGL>(acc, xv, yv);
        }
    }
}

// The sweep under a StepSched (single-product bodies only): this lane's
// borrowed steps into acc, parked in acc2, then its own steps into acc.
template <int MODE, int OPK, int NEGL>
__device__ __forceinline__ void sweep_sched(float (&acc)[kBlk], float (&acc2)[kBlk],
                                            const float *xt, const float *yt, const float2 *tab,
                                            int rowl, int kh, int lgNH, const unsigned char *steps,
                                            int nsec, int ntot, int skh) {
    const int NH = 1 << lgNH;
#pragma unroll 1
    for (int t = 0; t < ntot; ++t) {
        if (t == nsec && nsec > 0) {
#pragma unroll
            for (int e = 0; e < kBlk; ++e) {
                acc2[e] = acc[e];
                acc[e] = 0.0f;
            }
        }
        const int k = t < nsec ? skh : kh;
        const int ih = steps[t * NH + kh];
        const float2 sg = tab[(ih << lgNH) | k];
        float xv[kBlk], yv[kBlk];
        load_block(xt, rowl + ih, xv);
        load_block(yt, rowl + (ih ^ k), yv);
        if (MODE == CB_MODE_GRAD_B) {
            const float sx = parity(ih) ? -1.0f : 1.0f;
#pragma unroll
            for (int e = 0; e < kBlk; ++e)
                if (popcl(e) & 1) xv[e] *= sx;
        }
        apply_sign(yv, sg);
        block_fma<MODE, OPK, NEGL>(acc, xv, yv);
    }
    if (nsec > 0 && ntot == nsec) {
#pragma unroll
        for (int e = 0; e < kBlk; ++e) {
            acc2[e] = acc[e];
            acc[e] = 0.0f;
        }
    }
}

// The inner product's sweep under an InnerSched (see there).
template <int MODE, int NEGL>
__device__ __forceinline__ void sweep_inner_sched(float (&acc)[kBlk], float (&acc2)[kBlk],
                                                  const float *xt, const float *yt,
                                                  const float2 *tab, const float2 *tab2, int rowl,
                                                  int kh, int lgNH, const InnerSched *sch) {
    const int NH = 1 << lgNH;
    const int nsec = sch->nsec[kh], skh = sch->sec_kh[kh], sph = sch->sec_ph[kh];
#pragma unroll 1
    for (int ph = 0; ph < 2; ++ph) {
        const int T = sch->T[ph], nown = sch->n[ph][kh];
        const bool borrow = nsec > 0 && sph == ph;
        const float2 *tb = ph == 0 ? tab : tab2;
        if (borrow && ph == 1) {  // the own partial sum waits in acc2 (zero until now)
#pragma unroll
            for (int e = 0; e < kBlk; ++e) {
                const float t = acc[e];
                acc[e] = acc2[e];
                acc2[e] = t;
            }
        }
#pragma unroll 1
        for (int t = 0; t <= T; ++t) {
            if (borrow && t == nsec) {  // the borrowed segment is done: swap it out
#pragma unroll
                for (int e = 0; e < kBlk; ++e) {
                    const float v = acc[e];
                    acc[e] = acc2[e];
                    acc2[e] = v;
                }
            }
            if (t >= nown) continue;
            const int k = (borrow && t < nsec) ? skh : kh;
            const int ih = sch->ih[ph][t * NH + kh];
            const float2 sg = tb[(ih << lgNH) | k];
            float xv[kBlk], yv[kBlk];
            load_block(xt, rowl + ih, xv);
            load_block(yt, rowl + (ih ^ k), yv);
            if (MODE == CB_MODE_GRAD_B) {  // x side of the cross term
                const float sx = parity(ih) ? -1.0f : 1.0f;
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    if (popcl(e) & 1) xv[e] *= sx;
            }
            apply_sign(yv, sg);
            if (ph == 0)
                block_fma<MODE, OPK_LC, NEGL>(acc, xv, yv);
            else
                block_fma<MODE, OPK_RC, NEGL>(acc, xv, yv);
        }
    }
}

// Sign s_L(e, e) (-1)^(popc(k_h) popc(e)) of the diagonal term e of line k_h
// (the inner product's correction).
template <int NEGL>
__device__ __forceinline__ int diag_sign(int e, int kh) {
    return (reorderl(e, e) ^ (popcl(e & low_neg_mask(NEGL)) & 1) ^ ((popcl(e) & 1) & parity(kh)))
               ? -1 : 1;
}

// Cl(6,1) geometric product through Cl(6,0) + Cl(6,0) (OPK_GP61). With
// omega = e0 ... e6 (central, omega^2 = +1) every x is u + v omega (u, v
// even), and x -> (u + v, u - v) is an algebra isomorphism onto pairs of
// elements of the even subalgebra, which is Cl(6,0) through f_i = e_i e_6.
// Per Cl(6,0) blade k: f_k = a(k) e_E (E = k, plus e_6 when k is odd) and
// e_O omega = s(O) e_(O^127), so with O = E ^ 127 and b = a s(O):
//     P[k] = a x[E] + b x[O],  Q[k] = a x[E] - b x[O],
// and back x[E] = a (P + Q)/2, x[O] = b (P - Q)/2. The map satisfies
// phi^T phi = 2 I, so each of the three sums is phi^-1 of the Cl(6,0) sum of
// the same mode over the pairs: the tile's 128-float rows turn in place into
// pairs of 64-float rows, the n = 6 sweep runs, and the results turn back.
// Bit k of amask / bmask: a(k) / b(k) = -1. The four lanes of a Cl(6,1) row
// (one warp) take blades 16 l .. 16 l + 15 each.
// In float4 chunks: with x0 / x1 the row's blades without / with e_6 and
// chunk m = blades 4m..4m+3 (64-blade halves), E(k) = k (even parity) or
// 64 + k (odd) and O(k) = E ^ 127 is blade 63 - k of the other half, so chunk
// m of P and Q needs chunk m of x0, x1 and chunk 15 - m of both, reversed.
__device__ __forceinline__ float4 ld4(const float *tile, int f) {
    return *reinterpret_cast<const float4 *>(tile + swz_index(f));
}
__device__ __forceinline__ void st4(float *tile, int f, float4 v) {
    *reinterpret_cast<float4 *>(tile + swz_index(f)) = v;
}
__device__ __forceinline__ float f4(const float4 &v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
__device__ __forceinline__ float sgn_bit(uint64_t mask, int k, float v) {
    return ((mask >> k) & 1) ? -v : v;
}

// Lane l of a row handles chunks m = 4l + c (c = 0..3), in the order
// c ^ (2 (R & 1)) so that rows R and R + 1 of a quarter-warp touch disjoint
// 16-byte bank groups. Its sign bits (bit i for blade k = 16 l + i): al = a(k),
// bk = b(k), bl = b(63 - k).
__device__ __forceinline__ void phi61_lane(int tid, uint64_t amask, uint64_t bmask, int &base,
                                           int &l, int &cx, uint32_t &al, uint32_t &bk,
                                           uint32_t &bl) {
    const int R = tid >> 2;
    l = tid & 3;
    base = 128 * R;
    cx = 2 * (R & 1);
    al = (uint32_t)(amask >> (16 * l)) & 0xFFFFu;
    bk = (uint32_t)(bmask >> (16 * l)) & 0xFFFFu;
    const uint32_t w = (uint32_t)(bmask >> (48 - 16 * l)) & 0xFFFFu;
    bl = __brev(w) >> 16;
}

// x rows -> [P | Q] in place, for the x and the y tile (one code copy).
__device__ __forceinline__ void phi61_in(float *xt, float *yt, int tid, uint64_t amask,
                                         uint64_t bmask) {
    int base, l, cx;
    uint32_t al, bk, bl;
    phi61_lane(tid, amask, bmask, base, l, cx, al, bk, bl);
#pragma unroll 1
    for (int t = 0; t < 2; ++t) {
        float *tile = t == 0 ? xt : yt;
        float4 P[4], Q[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int cc = c ^ cx, m = 4 * l + cc, mr = 15 - m;
            const float4 x0 = ld4(tile, base + 4 * m), x1 = ld4(tile, base + 64 + 4 * m);
            const float4 r0 = ld4(tile, base + 4 * mr), r1 = ld4(tile, base + 64 + 4 * mr);
            const int pm = parity((uint32_t)m);
            float p[4], q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = 4 * cc + j;                        // k = 16 l + i
                const bool odd = pm ^ ((j ^ (j >> 1)) & 1);      // parity of k
                const float xe = odd ? f4(x1, j) : f4(x0, j);    // x[E(k)]
                const float xo = odd ? f4(r0, 3 - j) : f4(r1, 3 - j);  // x[O(k)]
                const float te = ((al >> i) & 1) ? -xe : xe;
                const float to = ((bk >> i) & 1) ? -xo : xo;
                p[j] = te + to;
                q[j] = te - to;
            }
            P[c] = make_float4(p[0], p[1], p[2], p[3]);
            Q[c] = make_float4(q[0], q[1], q[2], q[3]);
        }
        __syncwarp();  // the row's four lanes have read it
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int m = 4 * l + (c ^ cx);
            st4(tile, base + 4 * m, P[c]);
            st4(tile, base + 64 + 4 * m, Q[c]);
        }
    }
    __syncwarp();
}

// Back, in place: x0[p] = a(p) U[p] (p even parity) or b(63-p) V[63-p] (odd),
// and x1[p] the other way round, U = (P + Q)/2, V = (P - Q)/2.
__device__ __forceinline__ void phi61_out(float *tile, int tid, uint64_t amask, uint64_t bmask) {
    int base, l, cx;
    uint32_t al, bk, bl;
    phi61_lane(tid, amask, bmask, base, l, cx, al, bk, bl);
    float4 X0[4], X1[4];
    __syncwarp();  // the row's lanes have stored both halves
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int cc = c ^ cx, m = 4 * l + cc, mr = 15 - m;
        const float4 P = ld4(tile, base + 4 * m), Q = ld4(tile, base + 64 + 4 * m);
        const float4 Pr = ld4(tile, base + 4 * mr), Qr = ld4(tile, base + 64 + 4 * mr);
        const int pm = parity((uint32_t)m);
        float u0[4], u1[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = 4 * cc + j;                       // p = 16 l + i
            const bool odd = pm ^ ((j ^ (j >> 1)) & 1);     // parity of p (= of 63 - p)
            const float U = 0.5f * (f4(P, j) + f4(Q, j));
            const float V = 0.5f * (f4(Pr, 3 - j) - f4(Qr, 3 - j));  // at blade 63 - p
            const float eu = ((al >> i) & 1) ? -U : U;
            const float ov = ((bl >> i) & 1) ? -V : V;  // b(63 - p)
            u0[j] = odd ? ov : eu;
            u1[j] = odd ? eu : ov;
        }
        X0[c] = make_float4(u0[0], u0[1], u0[2], u0[3]);
        X1[c] = make_float4(u1[0], u1[1], u1[2], u1[3]);
    }
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int m = 4 * l + (c ^ cx);
        st4(tile, base + 4 * m, X0[c]);
        st4(tile, base + 64 + 4 * m, X1[c]);
    }
}

// a / b masks of the Cl(6,1) route (metric: e6 squares to -1, e0..e5 to +1).
inline void phi61_masks(uint64_t *amask, uint64_t *bmask) {
    const uint32_t neg = 1u << 6;
    *amask = *bmask = 0;
    for (int k = 0; k < 64; ++k) {
        uint32_t blade = 0;
        int sign = 1;
        for (int i = 0; i < 6; ++i) {
            if (!((k >> i) & 1)) continue;
            const uint32_t gs[2] = {1u << i, 1u << 6};
            for (uint32_t g : gs) {
                sign *= blade_sign(blade, g, neg, 0);
                blade ^= g;
            }
        }
        const int sb = sign * blade_sign(blade ^ 127u, 127u, neg, 0);
        if (sign < 0) *amask |= 1ull << k;
        if (sb < 0) *bmask |= 1ull << k;
    }
}

template <int MODE, int OPK, int NEGL, bool SCHED>
__global__ void __launch_bounds__(kThreads, 3)
    bilinear_tiled_kernel(const __grid_constant__ CUtensorMap mx,
                          const __grid_constant__ CUtensorMap my,
                          const __grid_constant__ CUtensorMap mo, int n, uint32_t neg,
                          uint32_t zero, int num_tiles, int *err, bool skip_zero,
                          const LowRelabel rl,
                          const __grid_constant__ std::conditional_t<
                              SCHED, std::conditional_t<OPK == OPK_INNER, InnerSched, StepSched>,
                              NoSched> sched,
                          uint64_t phi_a, uint64_t phi_b) {
    extern __shared__ unsigned char smem_raw[];
    // 1 KB-aligned start, derived by pointer arithmetic on the shared array so
    // the compiler keeps the shared address space (32-bit LDS/STS addressing).
    unsigned char *const base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    float *xs = reinterpret_cast<float *>(base);  // [kStages][kTileFloats], x in, then out
    float *ys = xs + kStages * kTileFloats;       // [kStages][kTileFloats]
    const int lgNH = n - kLow;
    const int NH = 1 << lgNH;
    constexpr bool inner = (OPK == OPK_INNER);
    constexpr bool reg = (OPK == OPK_REG);
    constexpr bool phi = (OPK == OPK_GP61);
    constexpr int OPB = reg ? OPK_WEDGE : (phi ? OPK_GP : OPK);  // the sweep's product
    float2 *tab = reinterpret_cast<float2 *>(ys + kStages * kTileFloats);
    float2 *tab2 = tab + NH * NH;
    uint64_t *bars = reinterpret_cast<uint64_t *>(tab + table_entries(n, inner));
    uint64_t *full = bars;
    int *done_count = reinterpret_cast<int *>(bars + kStages);  // [kStages]
    constexpr bool scheduled = SCHED && !inner && OPK != OPK_GP;  // sched.T > 0
    constexpr bool isched = SCHED && inner;                       // sched.T[0] > 0
    using SchedT = std::conditional_t<isched, InnerSched, StepSched>;
    SchedT *sch = reinterpret_cast<SchedT *>(bars + 8);  // 64 bytes past the barriers

    const int tid = threadIdx.x;
    const int D = 1 << n;
    const uint32_t negH = neg >> kLow, zeroH = zero >> kLow;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            done_count[s] = 0;
        }
        fence_barrier_init();
        prefetch_tensormap(&mx);
        prefetch_tensormap(&my);
        prefetch_tensormap(&mo);
    }
    if constexpr (scheduled || isched) {  // lanes index the schedule by lane: shared memory
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&sched);
        uint32_t *dst = reinterpret_cast<uint32_t *>(sch);
        for (int w = tid; w < (int)(sizeof(SchedT) / 4); w += kThreads) dst[w] = src[w];
    }
    // per-CTA table of high-part factors, [i_h][k_h]
    for (int e = tid; e < NH * NH; e += kThreads) {
        const uint32_t ih = e >> lgNH, k = e & (NH - 1);
        if (inner) {
            tab[e] = high_factor(MODE, OPK_LC, ih, k, negH, zeroH);
            tab2[e] = high_factor(MODE, OPK_RC, ih, k, negH, zeroH);
        } else {
            tab[e] = high_factor(MODE, OPB, ih, k, negH, zeroH);
        }
    }
    __syncthreads();

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            const int tile = blockIdx.x + s * gridDim.x;
            if (tile < num_tiles) {
                mbar_arrive_expect_tx(&full[s], 2 * kTileBytes);
                tma_load_2d(xs + s * kTileFloats, &mx, 0, tile * kTileLines, &full[s]);
                tma_load_2d(ys + s * kTileFloats, &my, 0, tile * kTileLines, &full[s]);
            }
        }
    }

    const int r = tid >> lgNH;
    const int lane = tid & 31;
    const int kh = tid & (NH - 1);
    const int rowl = (r * D) >> 5;  // first line of this thread's row
    for (int it = 0;; ++it) {
        const int tile = blockIdx.x + it * gridDim.x;
        if (tile >= num_tiles) break;
        const int s = it % kStages;
        // warp-uniform: the sweep below uses full-warp votes and shuffles
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (it / kStages) & 1, err, 0x101)))
            break;
        float *xt = xs + s * kTileFloats;
        float *yt = ys + s * kTileFloats;
        if (rl.active) {  // the row's lines move to the relabelled low order
            relabel_line(xt, rowl + kh, rl);
            relabel_line(yt, rowl + kh, rl);
            __syncwarp();  // a row's lines are read by the row's threads, one warp
        }
        if constexpr (phi) {  // Cl(6,1) rows -> pairs of Cl(6,0) rows
            phi61_in(xt, yt, tid, phi_a, phi_b);
        }
        const uint32_t allb = (uint32_t)D - 1;  // the pseudoscalar's blade
        const uint32_t dmask = (0xAAAAAAAAu ^ neg) & allb;
        const float isq = reg ? (float)blade_sign(allb, allb, neg, zero) : 1.0f;  // I^2 = 1/I^2
        if (reg) {  // x' = D x; y' = D b (forward) or D^T g (backward sums)
            float xv[kBlk], yv[kBlk];
            load_block(xt, rowl + kh, xv);
            load_block(yt, rowl + kh, yv);
            __syncwarp();
            dual_move(xv, xt, rowl + NH - 1 - kh, (uint32_t)kh * kBlk, allb, dmask, isq, false);
            dual_move(yv, yt, rowl + NH - 1 - kh, (uint32_t)kh * kBlk, allb, dmask, isq,
                      MODE != CB_MODE_FWD);
            __syncwarp();
        }

        float acc[kBlk];
#pragma unroll
        for (int e = 0; e < kBlk; ++e) acc[e] = 0.0f;
        if constexpr (scheduled) {
            {
                float acc2[kBlk];
                const int nsec = sch->nsec[kh];
                sweep_sched<MODE, OPB, NEGL>(acc, acc2, xt, yt, tab, rowl, kh, lgNH, sch->ih, nsec,
                                             sch->ntot[kh], sch->sec_kh[kh]);
                // every lane of the row is past its sweep: the row's y lines are
                // free to carry the borrowed sums to their blocks' lanes
                __syncwarp();
                if (nsec > 0) store_block(yt, rowl + kh, acc2);
                __syncwarp();
                for (uint32_t dm = sch->donors[kh]; dm; dm &= dm - 1) {
                    float part[kBlk];
                    load_block(yt, rowl + __ffs(dm) - 1, part);
#pragma unroll
                    for (int e = 0; e < kBlk; ++e) acc[e] += part[e];
                }
            }
        } else if constexpr (isched) {
            float acc2[kBlk];
#pragma unroll
            for (int e = 0; e < kBlk; ++e) acc2[e] = 0.0f;
            sweep_inner_sched<MODE, NEGL>(acc, acc2, xt, yt, tab, tab2, rowl, kh, lgNH, sch);
            // the diagonal correction's inputs, before the y lines carry the
            // borrowed sums (the correction applies after the grad_a flip)
            float dpart = 0.0f, y0 = 0.0f;
            const int shh = blade_sign(kh, kh, negH, zeroH);
            if (MODE == CB_MODE_FWD) {  // out[0] -= sum_i s(i, i) x_i y_i
                float xv[kBlk], yv[kBlk];
                load_block(xt, rowl + kh, xv);
                load_block(yt, rowl + kh, yv);
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    dpart = fmaf((float)(shh * diag_sign<NEGL>(e, kh)) * xv[e], yv[e], dpart);
                for (int m = 1; m < NH; m <<= 1) dpart += __shfl_xor_sync(0xffffffffu, dpart, m);
            } else {
                y0 = yt[swz_index(rowl << 5)];
            }
            __syncwarp();
            if (sch->nsec[kh] > 0) store_block(yt, rowl + kh, acc2);
            __syncwarp();
            for (uint32_t dm = sch->donors[kh]; dm; dm &= dm - 1) {
                float part[kBlk];
                load_block(yt, rowl + __ffs(dm) - 1, part);
#pragma unroll
                for (int e = 0; e < kBlk; ++e) acc[e] += part[e];
            }
            if (MODE == CB_MODE_GRAD_A && parity(kh)) {
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    if (popcl(e) & 1) acc[e] = -acc[e];
            }
            if (MODE == CB_MODE_FWD) {
                if (kh == 0) acc[0] -= dpart;
            } else {  // out[k] -= s(k, k) x_k y_0
                float xv[kBlk];
                load_block(xt, rowl + kh, xv);
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    acc[e] = fmaf(-(float)(shh * diag_sign<NEGL>(e, kh)) * xv[e], y0, acc[e]);
            }
        } else {
            sweep<MODE, OPB, NEGL>(acc, xt, yt, tab, tab2, rowl, kh, lgNH, skip_zero);
        }

        if (!isched && MODE == CB_MODE_GRAD_A && parity(kh)) {
#pragma unroll
            for (int e = 0; e < kBlk; ++e)
                if (popcl(e) & 1) acc[e] = -acc[e];
        }
        // inner: remove the P == Q terms counted by both contractions.
        // s(k, k) = s_H(k_h, k_h) s_L(k_l, k_l) (-1)^(popc(k_h) popc(k_l)).
        if (inner && !isched) {
            float xv[kBlk];
            load_block(xt, rowl + kh, xv);
            const int shh = blade_sign(kh, kh, negH, zeroH);
            if (MODE == CB_MODE_FWD) {  // out[0] -= sum_i s(i, i) x_i y_i
                float yv[kBlk];
                load_block(yt, rowl + kh, yv);
                float dpart = 0.0f;
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    dpart = fmaf((float)(shh * diag_sign<NEGL>(e, kh)) * xv[e], yv[e], dpart);
                // the row's NH threads are consecutive lanes of one warp
                for (int m = 1; m < NH; m <<= 1) dpart += __shfl_xor_sync(0xffffffffu, dpart, m);
                if (kh == 0) acc[0] -= dpart;
            } else {  // out[k] -= s(k, k) x_k y_0
                const float y0 = yt[swz_index(rowl << 5)];
#pragma unroll
                for (int e = 0; e < kBlk; ++e)
                    acc[e] = fmaf(-(float)(shh * diag_sign<NEGL>(e, kh)) * xv[e], y0, acc[e]);
            }
        }
        // This warp's rows are read only by this warp: once its lanes are done
        // reading, the results can replace the x values of those rows.
        __syncwarp();
        if (reg)  // out = D t (forward) or D^T t (backward sums)
            dual_move(acc, xt, rowl + NH - 1 - kh, (uint32_t)kh * kBlk, allb, dmask, isq,
                      MODE != CB_MODE_FWD);
        else if (rl.active)
            store_block_relabel(xt, rowl + kh, acc, rl);
        else
            store_block(xt, rowl + kh, acc);
        if constexpr (phi) phi61_out(xt, tid, phi_a, phi_b);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&done_count[s], 1) == kThreads / 32 - 1) {  // last warp
                __threadfence_block();
                done_count[s] = 0;
                tma_store_2d(&mo, xt, 0, tile * kTileLines);
                bulk_commit();
                const int next = tile + kStages * gridDim.x;
                if (next < num_tiles) {
                    bulk_wait_read_all();  // the store has read stage s's x tile
                    mbar_arrive_expect_tx(&full[s], 2 * kTileBytes);
                    tma_load_2d(xt, &mx, 0, next * kTileLines, &full[s]);
                    tma_load_2d(ys + s * kTileFloats, &my, 0, next * kTileLines, &full[s]);
                }
            }
        }
        __syncwarp();
    }
    // Stores issued by this thread must finish before the CTA exits.
    if (lane == 0) bulk_wait_all();
}

template <int MODE, int OPK, int NEGL>
int launch_tiled_k(const float *x, const float *y, float *out, int64_t batch, int n, uint32_t neg,
                   uint32_t zero, const LowRelabel &rl, cudaStream_t stream, uint64_t phi_a = 0,
                   uint64_t phi_b = 0) {
    DeviceInfo di;
    int st = device_info(&di);
    if (st) return st;
    int *err = nullptr;
    if ((st = device_error_word(&err))) return st;
    const int D = 1 << n;
    const uint64_t lines = (uint64_t)batch * D / 32;
    CUtensorMap mx, my, mo;
    if ((st = make_tmap_lines(&mx, x, lines, kTileLines))) return st;
    if ((st = make_tmap_lines(&my, y, lines, kTileLines))) return st;
    if ((st = make_tmap_lines(&mo, out, lines, kTileLines))) return st;
    const int rows_per_tile = kTileFloats / D;
    const int64_t tiles = (batch + rows_per_tile - 1) / rows_per_tile;
    if (tiles > ((int64_t)1 << 30)) {
        set_error("batch too large for one call");
        return CB_ERR_UNSUPPORTED;
    }
    const bool skip_zero = n >= 9 || (zero >> kLow) != 0;
    auto run = [&](auto kern, size_t smem, const auto &sched_arg) -> int {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bilinear_tiled)");
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (per_sm < 1) {
            set_error("bilinear tiled kernel does not fit an SM (smem %zu)", smem);
            return CB_ERR_UNSUPPORTED;
        }
        const int grid = (int)std::min<int64_t>(tiles, (int64_t)per_sm * di.sm_count);
        kern<<<grid, kThreads, smem, stream>>>(mx, my, mo, n, neg, zero, (int)tiles, err,
                                               skip_zero, rl, sched_arg, phi_a, phi_b);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(e, "launch bilinear_tiled_kernel");
        return CB_OK;
    };
    if constexpr (OPK == OPK_INNER) {
        const InnerSched isch = cached_inner_sched(MODE, n, neg, zero);
        if (isch.T[0] > 0)
            return run(bilinear_tiled_kernel<MODE, OPK, NEGL, true>,
                       smem_bytes(n, true, sizeof(InnerSched)), isch);
    }
    if constexpr (OPK != OPK_GP && OPK != OPK_INNER && OPK != OPK_GP61) {
        const StepSched sched = cached_sched(MODE, OPK, n, neg, zero);
        if (sched.T)
            return run(bilinear_tiled_kernel<MODE, OPK, NEGL, true>,
                       smem_bytes(n, false, sizeof(StepSched)), sched);
    }
    return run(bilinear_tiled_kernel<MODE, OPK, NEGL, false>, smem_bytes(n, OPK == OPK_INNER),
               NoSched{0});
}

// Low generators squaring to -1 are relabelled to the top of the low block
// and served by the body compiled for their count; the wedge product never
// meets the metric (P & Q = 0), so it keeps the Euclidean body.
template <int MODE, int OPK>
int launch_tiled(const float *x, const float *y, float *out, int64_t batch, int n, uint32_t neg,
                 uint32_t zero, cudaStream_t stream) {
    if constexpr (OPK == OPK_WEDGE) {
        const uint32_t negh = neg & ~(uint32_t)(kBlk - 1);
        return launch_tiled_k<MODE, OPK, 0>(x, y, out, batch, n, negh, zero, make_relabel(0),
                                            stream);
    } else if constexpr (OPK == OPK_REG) {  // wedge body; the dual steps read the full metric
        return launch_tiled_k<MODE, OPK, 0>(x, y, out, batch, n, neg, zero, make_relabel(0),
                                            stream);
    } else {
        const uint32_t negL = neg & (kBlk - 1);
        const int negl = __builtin_popcount(negL);
        const LowRelabel rl = make_relabel(negL);
        // the relabelled metric: low negatives on the top bits
        const uint32_t negr = (neg & ~(uint32_t)(kBlk - 1)) | (uint32_t)low_neg_mask(negl);
        switch (negl) {
        case 0: return launch_tiled_k<MODE, OPK, 0>(x, y, out, batch, n, negr, zero, rl, stream);
        case 1: return launch_tiled_k<MODE, OPK, 1>(x, y, out, batch, n, negr, zero, rl, stream);
        case 2: return launch_tiled_k<MODE, OPK, 2>(x, y, out, batch, n, negr, zero, rl, stream);
        case 3: return launch_tiled_k<MODE, OPK, 3>(x, y, out, batch, n, negr, zero, rl, stream);
        case 4: return launch_tiled_k<MODE, OPK, 4>(x, y, out, batch, n, negr, zero, rl, stream);
        default: return launch_tiled_k<MODE, OPK, 5>(x, y, out, batch, n, negr, zero, rl, stream);
        }
    }
}

}  // namespace tiled

// Explicitly instantiated per mode in bilinear_tiled_{fwd,ga,gb}.cu.
template <int MODE>
int bilinear_tiled(int op, const float *x, const float *y, float *out, int64_t batch, int n,
                   uint32_t neg, uint32_t zero, cudaStream_t stream) {
    using namespace tiled;
    switch (op) {
    case CB_OP_GP: return launch_tiled<MODE, OPK_GP>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_WEDGE: return launch_tiled<MODE, OPK_WEDGE>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_LC: return launch_tiled<MODE, OPK_LC>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_RC: return launch_tiled<MODE, OPK_RC>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_INNER: return launch_tiled<MODE, OPK_INNER>(x, y, out, batch, n, neg, zero, stream);
    case CB_OP_REG: return launch_tiled<MODE, OPK_REG>(x, y, out, batch, n, neg, zero, stream);
    }
    set_error("op %d has no tiled kernel", op);
    return CB_ERR_INVALID;
}

// The Cl(6,1) geometric product (metric [1]*6 + [-1]) through two Cl(6,0)
// sums per row (OPK_GP61); mode as in cb_bilinear.
template <int MODE>
int bilinear_tiled_cl61(const float *x, const float *y, float *out, int64_t batch,
                        cudaStream_t stream) {
    using namespace tiled;
    static uint64_t amask = 0, bmask = 0;
    static const bool once = (phi61_masks(&amask, &bmask), true);
    (void)once;
    return launch_tiled_k<MODE, OPK_GP61, 0>(x, y, out, 2 * batch, 6, 0, 0, make_relabel(0), stream,
                                             amask, bmask);
}

}  // namespace cb
