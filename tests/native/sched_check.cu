// Host-side check of the tiled kernel's step schedules (bilinear_tiled.cuh):
// for every n = 5..10, mode and a few metrics, each step with a non-zero
// high-part factor is scheduled exactly once, to the right output line, no
// lane runs more than the schedule's round count, and the donor masks match
// the borrowed segments. Prints "bad <count>", the schedules' lengths and the
// sign masks of the Cl(6,1) route.
#include <cstdio>

#include "../../cliffordcuda_b200/csrc/bilinear_tiled.cuh"

using namespace cb;
using namespace cb::tiled;

int main() {
    int bad = 0, active = 0, iactive = 0;
    for (int n = 5; n <= 10; ++n) {
        const int NH = 1 << (n - 5);
        const uint32_t zeros[3] = {0u, 1u << (n - 1), 3u << (n - 2)};
        for (uint32_t zero : zeros)
            for (int mode = 0; mode < 3; ++mode) {
                const uint32_t negH = 0, zeroH = zero >> 5;
                for (int opk : {OPK_WEDGE, OPK_LC, OPK_RC, OPK_REG}) {
                    const StepSched s = make_sched(mode, opk, n, 0, zero);
                    if (!s.T) continue;
                    ++active;
                    const int opb = opk == OPK_REG ? OPK_WEDGE : opk;
                    int seen[32][32] = {};
                    for (int L = 0; L < NH; ++L) {
                        if (s.ntot[L] > s.T) ++bad;
                        for (int t = 0; t < s.ntot[L]; ++t) {
                            const int k = t < s.nsec[L] ? s.sec_kh[L] : L;
                            if (t < s.nsec[L] && !((s.donors[k] >> L) & 1)) ++bad;
                            ++seen[s.ih[t * NH + L]][k];
                        }
                    }
                    for (int k = 0; k < NH; ++k)
                        for (int ih = 0; ih < NH; ++ih)
                            if (seen[ih][k] != (high_factor(mode, opb, ih, k, negH, zeroH).x != 0.0f))
                                ++bad;
                }
                const InnerSched q = make_inner_sched(mode, n, 1u << (n - 1), zero);
                if (!q.T[0]) continue;
                ++iactive;
                int seen[2][32][32] = {};
                for (int L = 0; L < NH; ++L)
                    for (int ph = 0; ph < 2; ++ph) {
                        if (q.n[ph][L] > q.T[ph]) ++bad;
                        const bool borrow = q.nsec[L] > 0 && q.sec_ph[L] == ph;
                        for (int t = 0; t < q.n[ph][L]; ++t) {
                            const int k = (borrow && t < q.nsec[L]) ? q.sec_kh[L] : L;
                            if (borrow && t < q.nsec[L] && !((q.donors[k] >> L) & 1)) ++bad;
                            ++seen[ph][q.ih[ph][t * NH + L]][k];
                        }
                    }
                for (int ph = 0; ph < 2; ++ph)
                    for (int k = 0; k < NH; ++k)
                        for (int ih = 0; ih < NH; ++ih)
                            if (seen[ph][ih][k] !=
                                (high_factor(mode, ph ? OPK_RC : OPK_LC, ih, k, 1u << (n - 6), zeroH)
                                     .x != 0.0f))
                                ++bad;
            }
    }
    // the config-5 left contraction: six rounds for every sum
    for (int mode = 0; mode < 3; ++mode) {
        const StepSched s = make_sched(mode, OPK_LC, 10, 0, 1u << 9);
        printf("lc10 mode %d rounds %d\n", mode, s.T);
    }
    // the Cl(6,1) route's sign masks (a(k), b(k) = -1 for bit k set)
    uint64_t am = 0, bm = 0;
    phi61_masks(&am, &bm);
    printf("phi61 %016llx %016llx\n", (unsigned long long)am, (unsigned long long)bm);
    printf("active %d inner %d\nbad %d\n", active, iactive, bad);
    return 0;
}
