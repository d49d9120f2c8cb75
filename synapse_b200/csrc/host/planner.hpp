// Static memory planning for the device arena (graph/planner.hpp:1-150 of the
// reference): every activation and scratch tensor of a decode step gets a
// fixed offset, computed once; tensors whose live intervals (node indices,
// closed) do not intersect share bytes. Placement is the reference's greedy
// rule -- largest first, each at the lowest aligned gap that does not overlap
// a placed tensor live at the same time -- so a session's footprint matches
// the reference's arena for the same graph, and invariants P1-P3 hold.
#pragma once

#include <algorithm>
#include <cstddef>
#include <numeric>
#include <vector>

namespace syn::plan {

struct tensor {
    size_t bytes = 0;
    size_t first = 0, last = 0;  // live over nodes [first, last]
};

struct result {
    std::vector<size_t> offset;
    size_t arena_bytes = 0;
    size_t naive_bytes = 0;
};

inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

inline bool intersects(const tensor& a, const tensor& b) { return a.first <= b.last && b.first <= a.last; }

inline result place(const std::vector<tensor>& ts, size_t alignment) {
    std::vector<size_t> order(ts.size());
    std::iota(order.begin(), order.end(), size_t{0});
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return ts[a].bytes > ts[b].bytes; });
    result r;
    r.offset.assign(ts.size(), 0);
    std::vector<size_t> placed, conflicts;
    for (size_t t : order) {
        r.naive_bytes += align_up(ts[t].bytes, alignment);
        conflicts.clear();
        for (size_t u : placed)
            if (intersects(ts[t], ts[u])) conflicts.push_back(u);
        std::sort(conflicts.begin(), conflicts.end(), [&](size_t a, size_t b) { return r.offset[a] < r.offset[b]; });
        size_t candidate = 0;
        for (size_t u : conflicts) {
            if (candidate + ts[t].bytes <= r.offset[u]) break;
            candidate = std::max(candidate, align_up(r.offset[u] + ts[u].bytes, alignment));
        }
        r.offset[t] = candidate;
        r.arena_bytes = std::max(r.arena_bytes, align_up(candidate + ts[t].bytes, alignment));
        placed.push_back(t);
    }
    return r;
}

// P1 alignment, P2 in bounds, P3 live-overlapping tensors are disjoint.
inline bool valid(const std::vector<tensor>& ts, const result& r, size_t alignment) {
    if (r.offset.size() != ts.size()) return false;
    for (size_t t = 0; t < ts.size(); ++t) {
        if (r.offset[t] % alignment || r.offset[t] + ts[t].bytes > r.arena_bytes) return false;
        for (size_t u = t + 1; u < ts.size(); ++u) {
            const bool disjoint = r.offset[t] + ts[t].bytes <= r.offset[u] || r.offset[u] + ts[u].bytes <= r.offset[t];
            if (intersects(ts[t], ts[u]) && !disjoint && ts[t].bytes && ts[u].bytes) return false;
        }
    }
    return true;
}

}  // namespace syn::plan
