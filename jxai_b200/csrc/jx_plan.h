// jx_plan.h -- host-side slicing of a step's flattened row space over the
// persistent CTAs of the fused decode kernel (host-only C++, no CUDA: the CPU
// tests build it with g++).
#pragma once

#include <algorithm>
#include <cstddef>
#include <functional>
#include <map>
#include <queue>
#include <type_traits>
#include <utility>
#include <vector>

namespace jx {

// Slice boundaries b[0..P] over the flattened rows (segment j starts at
// seg_off[j], seg_off.back() == total) so that every CTA's rows plus
// `penalty` rows per extra piece (each segment boundary inside its slice)
// come out equal.
//  * Few segments per CTA: the smallest whole-row per-CTA budget that covers
//    every row, by bisection (each step a walk over the CTAs and segments).
//    *hint (optional) is the budget of a previous call, updated on return:
//    a decode loop's next step moves it by about one row, so the search
//    brackets it in a few passes -- with the same result as without a hint.
//  * Many (a prefill's thousands of short segments): one pass -- with
//    F(x) = x + penalty * (segment starts <= x), CTA c takes
//    [F^-1(c*C/P), F^-1((c+1)*C/P)), C = F(total).  Here a CTA's share is
//    much larger than one penalty, so no CTA falls inside a single step of F
//    (which would leave it empty).
inline std::vector<long long> balanced_split(const std::vector<long long>& seg_off,
                                             long long total, long long P, double penalty,
                                             int form = -1, long long* hint = nullptr) {
    std::vector<long long> b(static_cast<size_t>(P) + 1, total);
    const size_t m = seg_off.size() - 1;  // segments
    b[0] = 0;
    if (m == 0 || P <= 1) return b;
    if (m > static_cast<size_t>(64 * P)) {
        std::vector<double> F(m);  // F just after segment j's start
        for (size_t j = 0; j < m; ++j)
            F[j] = static_cast<double>(seg_off[j]) + penalty * static_cast<double>(j + 1);
        const double C = static_cast<double>(total) + penalty * static_cast<double>(m);
        for (long long c = 1; c < P; ++c) {
            const double target = C * static_cast<double>(c) / static_cast<double>(P);
            const size_t j = static_cast<size_t>(
                std::upper_bound(F.begin(), F.end(), target) - F.begin());
            long long x = 0;
            if (j > 0) {
                const size_t sj = j - 1;
                x = std::min(seg_off[sj] + static_cast<long long>(target - F[sj]), seg_off[sj + 1]);
            }
            b[static_cast<size_t>(c)] = std::max(x, b[static_cast<size_t>(c - 1)]);
        }
        b[static_cast<size_t>(P)] = total;
        return b;
    }
    // One layout pass for a per-CTA budget: CTA boundaries (write) and how
    // far the P slices reach.  With kRuns, a run of fresh CTAs that each end
    // inside the current segment takes `step` rows apiece and is laid out at
    // once, so a pass costs O(segments) rather than O(P) where segments are
    // long (a pass runs a dozen times per bisection, on every call whose plan
    // changed); both forms give the same boundaries.
    auto layout = [&](double budget_rows, bool write, auto runs) -> long long {
        const long long step = static_cast<long long>(budget_rows);  // rows of a fresh CTA
        long long x = 0;
        size_t j = 0;  // seg_off[j] <= x < seg_off[j+1]
        for (long long c = 0; c < P; ++c) {
            if (write) b[static_cast<size_t>(c)] = x;
            double budget = budget_rows;
            while (x < total) {
                while (j + 1 < seg_off.size() && seg_off[j + 1] <= x) ++j;
                const long long seg_end = seg_off[j + 1];
                const long long avail = seg_end - x;
                if (static_cast<double>(avail) >= budget) {
                    if constexpr (decltype(runs)::value) {
                        if (budget == budget_rows && step > 0 &&
                            static_cast<double>(avail) >= 4.0 * budget_rows) {
                            // CTA i of the run needs avail - i*step >= budget_rows
                            long long k = static_cast<long long>(
                                              (static_cast<double>(avail) - budget_rows) /
                                              static_cast<double>(step)) + 1;
                            while (k > 1 &&
                                   static_cast<double>(avail - (k - 1) * step) < budget_rows)
                                --k;
                            while (static_cast<double>(avail - k * step) >= budget_rows) ++k;
                            k = std::min(k, P - c);
                            if (write)
                                for (long long i = 1; i < k; ++i)
                                    b[static_cast<size_t>(c + i)] = x + i * step;
                            x += k * step;
                            c += k - 1;
                            break;
                        }
                    }
                    x += static_cast<long long>(budget);
                    break;
                }
                x = seg_end;
                budget -= static_cast<double>(avail) + penalty;
                if (budget <= 0.0) break;
            }
        }
        if (write) b[static_cast<size_t>(P)] = total;
        return x;
    };
    // runs pay off when a CTA's share is well under a segment (form: -1 by
    // that rule, 0 the plain loop, 1 with runs -- the same boundaries)
    const bool long_segments = form < 0 ? P >= 4 * static_cast<long long>(m) : form == 1;
    auto pass = [&](double budget_rows, bool write) -> long long {
        return long_segments ? layout(budget_rows, write, std::true_type{})
                             : layout(budget_rows, write, std::false_type{});
    };
    // lo: below the mean share, so no layout covers the rows; hi: covers them
    auto covers = [&](long long budget) { return pass(static_cast<double>(budget), false) >= total; };
    long long lo = std::max<long long>(0, total / P - 1);
    long long hi = static_cast<long long>(static_cast<double>(total) / static_cast<double>(P) +
                                          penalty * static_cast<double>(m)) + 2;
    if (hint && *hint > lo && *hint < hi) {
        const long long h = *hint;
        if (covers(h)) {
            hi = h;
            for (long long d = 1; h - d > lo; d *= 2) {
                if (!covers(h - d)) {
                    lo = h - d;
                    break;
                }
                hi = h - d;
            }
        } else {
            lo = h;
            for (long long d = 1; h + d < hi; d *= 2) {
                if (covers(h + d)) {
                    hi = h + d;
                    break;
                }
                lo = h + d;
            }
        }
    }
    while (hi - lo > 1) {
        const long long mid = lo + (hi - lo) / 2;
        if (covers(mid)) hi = mid; else lo = mid;
    }
    if (hint) *hint = hi;
    pass(static_cast<double>(hi), true);
    return b;
}

// Order and CTA assignment of the tensor-core prefill's work items: item i
// reads the cache rows of K/V stream stream[i] (sequence, cache layer, kv
// head) in tiles[i] tiles.  Returns the items in launch order, where CTA b of
// P runs [first[b], first[b + 1]).
//  * window == 0: all items largest first, CTA b taking items b, b + P, ...
//    (balanced, but the CTAs working at one time read P different streams).
//  * window = k > 0: the streams (those with the largest item first) go in
//    batches of k; each batch's items largest first, batch after batch, so the
//    CTAs working at one time share about k streams' rows through L2.  The
//    last 3P items are ordered largest first across batches, so the CTAs end
//    together.  Items are dealt by list scheduling: each to the CTA whose
//    earlier items end first, at a cost of its tiles plus item_cost (staging
//    its queries).
inline std::vector<size_t> schedule_items(const std::vector<long long>& stream,
                                          const std::vector<int>& tiles, int P,
                                          long long item_cost, int window,
                                          std::vector<int>& first) {
    const size_t n = tiles.size();
    const size_t np = static_cast<size_t>(std::max(P, 1));
    std::vector<size_t> idx(n);
    for (size_t i = 0; i < n; ++i) idx[i] = i;
    auto larger = [&](size_t x, size_t y) { return tiles[x] > tiles[y]; };
    std::vector<std::vector<size_t>> lists(np);
    if (window <= 0) {
        std::stable_sort(idx.begin(), idx.end(), larger);
        for (size_t k = 0; k < n; ++k) lists[k % np].push_back(idx[k]);
    } else {
        std::map<long long, int> gid;
        std::vector<int> g_of(n), gmax;
        for (size_t i = 0; i < n; ++i) {
            const auto ins = gid.emplace(stream[i], static_cast<int>(gid.size()));
            const int g = ins.first->second;
            if (ins.second) gmax.push_back(0);
            gmax[static_cast<size_t>(g)] = std::max(gmax[static_cast<size_t>(g)], tiles[i]);
            g_of[i] = g;
        }
        std::vector<int> gorder(gmax.size()), batch(gmax.size());
        for (size_t g = 0; g < gorder.size(); ++g) gorder[g] = static_cast<int>(g);
        std::stable_sort(gorder.begin(), gorder.end(), [&](int x, int y) {
            return gmax[static_cast<size_t>(x)] > gmax[static_cast<size_t>(y)];
        });
        for (size_t r = 0; r < gorder.size(); ++r)
            batch[static_cast<size_t>(gorder[r])] = static_cast<int>(r / static_cast<size_t>(window));
        std::stable_sort(idx.begin(), idx.end(), [&](size_t x, size_t y) {
            const int bx = batch[static_cast<size_t>(g_of[x])], by = batch[static_cast<size_t>(g_of[y])];
            if (bx != by) return bx < by;
            return tiles[x] > tiles[y];
        });
        const size_t tail = std::min(n, 3 * np);
        std::stable_sort(idx.end() - static_cast<std::ptrdiff_t>(tail), idx.end(), larger);
        using Slot = std::pair<long long, int>;  // (time this CTA's items end, CTA)
        std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> free_at;
        for (size_t b = 0; b < np; ++b) free_at.push({0, static_cast<int>(b)});
        for (size_t i : idx) {
            const Slot sl = free_at.top();
            free_at.pop();
            lists[static_cast<size_t>(sl.second)].push_back(i);
            free_at.push({sl.first + tiles[i] + item_cost, sl.second});
        }
    }
    std::vector<size_t> order;
    order.reserve(n);
    first.assign(np + 1, 0);
    for (size_t b = 0; b < np; ++b) {
        for (size_t i : lists[b]) order.push_back(i);
        first[b + 1] = static_cast<int>(order.size());
    }
    return order;
}

}  // namespace jx
