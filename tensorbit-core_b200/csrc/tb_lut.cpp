// Tie tables for the top-N mask (MaskStrategy::kTopN / kIterative).
//
// The reference picks the kept elements of a group with
//   std::nth_element(buf, buf + N, buf + M, [](a, b){ return a.first > b.first; })
// on (score, index) pairs (include/tensorbit/core/coring.hpp:376-392).  When
// scores tie at the N-th place, which indices it keeps is up to the standard
// library's algorithm.  Because nth_element only ever compares scores, its
// choice is a function of the group's weak order alone.  This file enumerates
// every weak order of M elements, encodes it as the vector of greater-than
// counts gt[i] = #{j : v[j] > v[i]} (key = sum gt[i] * M^i), and records the
// mask that this very std::nth_element call returns for scores with that
// order.  The device looks a group up only when its N-th and (N+1)-th scores
// tie.  Built with the same C++ standard library as the reference's host code,
// the tables reproduce its choice exactly.
#include <algorithm>
#include <cstdint>
#include <utility>
#include <vector>

namespace tb {

namespace {

struct Builder {
    int n, m;
    std::vector<uint8_t>* table;
    int gt[16];

    uint8_t select(const int* g) const {
        std::pair<float, int> buf[16];
        for (int i = 0; i < m; ++i) buf[i] = {static_cast<float>(m - g[i]), i};
        std::nth_element(buf, buf + n, buf + m, [](auto& a, auto& b) { return a.first > b.first; });
        uint8_t byte = 0;
        for (int k = 0; k < n; ++k) byte |= static_cast<uint8_t>(1u << buf[k].second);
        return byte;
    }

    // Places the elements of `rest` (bitmask) at levels >= `above`: every
    // non-empty subset can form the next tie class.
    void place(uint32_t rest, int above) {
        if (rest == 0) {
            uint32_t key = 0, scale = 1;
            for (int i = 0; i < m; ++i) { key += static_cast<uint32_t>(gt[i]) * scale; scale *= static_cast<uint32_t>(m); }
            (*table)[key] = select(gt);
            return;
        }
        for (uint32_t sub = rest; sub; sub = (sub - 1) & rest) {
            int cnt = 0;
            for (int i = 0; i < m; ++i)
                if (sub & (1u << i)) { gt[i] = above; ++cnt; }
            place(rest & ~sub, above + cnt);
        }
    }
};

}  // namespace

// Table of m^m bytes for top-n of m (2 <= m <= 8, 1 <= n < m).
std::vector<uint8_t> build_topn_table(int n, int m) {
    uint32_t size = 1;
    for (int i = 0; i < m; ++i) size *= static_cast<uint32_t>(m);
    std::vector<uint8_t> table(size, 0);
    Builder b{n, m, &table, {}};
    b.place((1u << m) - 1u, 0);
    return table;
}

}  // namespace tb
