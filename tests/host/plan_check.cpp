// CPU check of jx::balanced_split (jxai_b200/csrc/jx_plan.h), the host-side
// slicing of a step's flattened row space over the fused decode kernel's
// persistent CTAs.  On seeded random layouts -- few or many segments per
// CTA, empty segments, small and large per-piece penalties -- it checks that
// the boundaries start at 0, end at the total and never decrease, and that
// the bisection's two layout forms (a plain walk over the CTAs, and one that
// lays out runs of CTAs inside a segment at once) give the same boundaries.
// Prints "ok <cases>" and exits 0, or prints the first failing case.
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "jx_plan.h"

int main(int argc, char** argv) {
    const int n_cases = argc > 1 ? std::atoi(argv[1]) : 20000;
    std::mt19937_64 rng(0x6a78616900000001ull);
    int checked = 0;
    for (int it = 0; it < n_cases; ++it) {
        const int m = 1 + static_cast<int>(rng() % (it % 3 == 0 ? 8 : it % 3 == 1 ? 64 : 3000));
        const long long P = 1 + static_cast<long long>(rng() % 600);
        std::vector<long long> seg_off{0};
        const long long lenmax = 1 + static_cast<long long>(rng() % (it % 2 ? 300 : 20000));
        for (int i = 0; i < m; ++i)
            seg_off.push_back(seg_off.back() +
                              (rng() % 8 == 0 ? 0 : 1 + static_cast<long long>(rng() % lenmax)));
        const long long total = seg_off.back();
        if (total == 0) continue;
        const double penalty = rng() % 4 == 0 ? static_cast<double>(rng() % 3) + 0.001
                                              : static_cast<double>(rng() % 100000) / 37.0 + 0.001;
        const std::vector<long long> b = jx::balanced_split(seg_off, total, P, penalty);
        bool ok = b.size() == static_cast<size_t>(P) + 1 && b.front() == 0 && b.back() == total;
        for (size_t i = 1; ok && i < b.size(); ++i) ok = b[i] >= b[i - 1];
        if (ok && static_cast<size_t>(m) <= static_cast<size_t>(64 * P)) {
            ok = jx::balanced_split(seg_off, total, P, penalty, 0) == b &&
                 jx::balanced_split(seg_off, total, P, penalty, 1) == b;
        }
        if (!ok) {
            std::printf("case %d: m=%d P=%lld total=%lld penalty=%f\n", it, m, P, total, penalty);
            return 1;
        }
        ++checked;
    }
    std::printf("ok %d\n", checked);
    return 0;
}
