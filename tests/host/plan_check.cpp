// CPU check of jx::balanced_split (jxai_b200/csrc/jx_plan.h), the host-side
// slicing of a step's flattened row space over the fused decode kernel's
// persistent CTAs.  On seeded random layouts -- few or many segments per
// CTA, empty segments, small and large per-piece penalties -- it checks that
// the boundaries start at 0, end at the total and never decrease, and that
// the bisection's two layout forms (a plain walk over the CTAs, and one that
// lays out runs of CTAs inside a segment at once) give the same boundaries,
// with or without a warm-start hint.
// It also checks jx::schedule_items, the order and CTA assignment of the
// tensor-core prefill's work items: the result is a permutation, the CTA
// ranges tile it, and no CTA's cost exceeds total / P + the largest item
// (either dealing: striding largest first, or list scheduling in batches of
// streams).
// Prints "ok <cases>" and exits 0, or prints the first failing case.
#include <algorithm>
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
            // a warm-start hint (near or far from the answer) changes nothing
            long long h = 1 + static_cast<long long>(rng() % (2 * (total / P + 2)));
            long long h2 = h;
            ok = ok && jx::balanced_split(seg_off, total, P, penalty, -1, &h) == b;
            ok = ok && jx::balanced_split(seg_off, total, P, penalty, -1, &h) == b &&
                 jx::balanced_split(seg_off, total, P, penalty, -1, &h2) == b;
        }
        if (!ok) {
            std::printf("case %d: m=%d P=%lld total=%lld penalty=%f\n", it, m, P, total, penalty);
            return 1;
        }
        ++checked;
    }
    for (int it = 0; it < n_cases / 20; ++it) {
        // prompts: streams of chunks whose tile counts grow along the prompt
        const int P = 1 + static_cast<int>(rng() % 200);
        const int n_streams = 1 + static_cast<int>(rng() % 300);
        std::vector<long long> stream;
        std::vector<int> tiles;
        for (int s = 0; s < n_streams; ++s) {
            const int chunks = 1 + static_cast<int>(rng() % 70);
            const int per = 1 + static_cast<int>(rng() % 3);
            for (int c = 0; c < chunks; ++c) {
                stream.push_back(s * 7919LL);
                tiles.push_back(1 + c / per + static_cast<int>(rng() % 2));
            }
        }
        std::vector<int> first;
        const int window = it % 4 == 0 ? 0 : 1 + static_cast<int>(rng() % 40);
        const std::vector<size_t> order = jx::schedule_items(stream, tiles, P, 2, window, first);
        bool ok = order.size() == tiles.size() && first.size() == static_cast<size_t>(P) + 1 &&
                  first.front() == 0 && first.back() == static_cast<int>(order.size());
        std::vector<size_t> sorted = order;
        std::sort(sorted.begin(), sorted.end());
        for (size_t i = 0; ok && i < sorted.size(); ++i) ok = sorted[i] == i;
        long long total = 0, biggest = 0;
        for (int t : tiles) {
            total += t + 2;
            biggest = std::max<long long>(biggest, t + 2);
        }
        for (int b = 0; ok && b < P; ++b) {
            ok = first[b + 1] >= first[b];
            long long cost = 0;
            for (int i = first[b]; ok && i < first[b + 1]; ++i) cost += tiles[order[i]] + 2;
            // list scheduling: a CTA's last item starts no later than total / P;
            // largest-first striding: no CTA holds more than one item above
            // any other's share (each round deals P items in falling size)
            ok = ok && cost <= total / P + biggest + 1;
        }
        if (!ok) {
            std::printf("schedule case %d: P=%d items=%zu\n", it, P, tiles.size());
            return 1;
        }
        ++checked;
    }
    std::printf("ok %d\n", checked);
    return 0;
}
