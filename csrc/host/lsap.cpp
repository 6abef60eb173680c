#include "lsap.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <numeric>

namespace mmltk {

namespace {
constexpr double kInf = std::numeric_limits<double>::infinity();

// One Dijkstra-like search from `start_row` over the reduced costs; returns the
// sink column (or -1 if no finite path exists).  `min_val` receives the length
// of the shortest augmenting path.
int64_t shortest_path(int64_t nr, int64_t nc, const double* c, int64_t start_row, LsapWorkspace& w, double& min_val) {
    double mv = 0.0;
    int64_t n_rem = nc;
    // columns are scanned from the highest index down (scipy's order, which
    // decides the winner among exactly equal reduced costs)
    for (int64_t k = 0; k < nc; ++k) w.remaining[k] = nc - 1 - k;
    std::fill(w.sr.begin(), w.sr.begin() + nr, 0);
    std::fill(w.sc.begin(), w.sc.begin() + nc, 0);
    std::fill(w.spc.begin(), w.spc.begin() + nc, kInf);
    int64_t i = start_row;
    int64_t sink = -1;
    while (sink < 0) {
        w.sr[i] = 1;
        int64_t best = -1;
        double lowest = kInf;
        const double ui = w.u[i];
        const double* ci = c + i * nc;
        for (int64_t k = 0; k < n_rem; ++k) {
            const int64_t j = w.remaining[k];
            const double r = mv + ci[j] - ui - w.v[j];
            if (r < w.spc[j]) {
                w.path[j] = i;
                w.spc[j] = r;
            }
            const double s = w.spc[j];
            if (s < lowest || (s == lowest && w.row4col[j] < 0)) {
                lowest = s;
                best = k;
            }
        }
        mv = lowest;
        if (!(mv < kInf)) return -1;
        const int64_t j = w.remaining[best];
        if (w.row4col[j] < 0) {
            sink = j;
        } else {
            i = w.row4col[j];
        }
        w.sc[j] = 1;
        w.remaining[best] = w.remaining[--n_rem];
    }
    min_val = mv;
    return sink;
}
}  // namespace

void lsap_sanitize(double* cost, int64_t n) {
    bool bad = false, any = false;
    double fmax = -kInf, amax = 0.0;
    for (int64_t k = 0; k < n; ++k) {
        const double x = cost[k];
        if (!std::isfinite(x)) {
            bad = true;
            continue;
        }
        any = true;
        fmax = std::max(fmax, x);
        amax = std::max(amax, std::fabs(x));
    }
    if (!bad) return;
    double rep = static_cast<double>(std::numeric_limits<float>::max());
    if (any) {
        const double cand = fmax + amax + 1.0;
        if (std::isfinite(cand)) rep = std::min(cand, rep);
    }
    for (int64_t k = 0; k < n; ++k)
        if (!std::isfinite(cost[k])) cost[k] = rep;
}

LsapStatus lsap_solve(int64_t nr, int64_t nc, const double* cost, bool maximize, int64_t* rows, int64_t* cols,
                      LsapWorkspace& w) {
    if (nr == 0 || nc == 0) return LsapStatus::kOk;
    const bool transpose = nc < nr;
    const double* c = cost;
    if (transpose || maximize) {
        w.transposed.resize(static_cast<size_t>(nr * nc));
        for (int64_t i = 0; i < nr; ++i)
            for (int64_t j = 0; j < nc; ++j) {
                const double x = maximize ? -cost[i * nc + j] : cost[i * nc + j];
                if (transpose)
                    w.transposed[j * nr + i] = x;
                else
                    w.transposed[i * nc + j] = x;
            }
        c = w.transposed.data();
        if (transpose) std::swap(nr, nc);
    }
    for (int64_t k = 0; k < nr * nc; ++k) {
        if (std::isnan(c[k]) || c[k] == -kInf) return LsapStatus::kInvalid;
    }
    w.u.assign(nr, 0.0);
    w.v.assign(nc, 0.0);
    w.spc.resize(nc);
    w.path.assign(nc, -1);
    w.col4row.assign(nr, -1);
    w.row4col.assign(nc, -1);
    w.remaining.resize(nc);
    w.sr.resize(nr);
    w.sc.resize(nc);

    for (int64_t cur = 0; cur < nr; ++cur) {
        double min_val = 0.0;
        const int64_t sink = shortest_path(nr, nc, c, cur, w, min_val);
        if (sink < 0) return LsapStatus::kInfeasible;
        // dual update
        w.u[cur] += min_val;
        for (int64_t i = 0; i < nr; ++i)
            if (w.sr[i] && i != cur) w.u[i] += min_val - w.spc[w.col4row[i]];
        for (int64_t j = 0; j < nc; ++j)
            if (w.sc[j]) w.v[j] -= min_val - w.spc[j];
        // augment along the path back to `cur`
        int64_t j = sink;
        while (true) {
            const int64_t i = w.path[j];
            w.row4col[j] = i;
            std::swap(w.col4row[i], j);
            if (i == cur) break;
        }
    }
    if (transpose) {
        // rows of the transposed problem are the original columns; report
        // pairs sorted by original row
        std::vector<int64_t> order(nr);
        std::iota(order.begin(), order.end(), 0);
        std::sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return w.col4row[a] < w.col4row[b]; });
        for (int64_t k = 0; k < nr; ++k) {
            rows[k] = w.col4row[order[k]];
            cols[k] = order[k];
        }
    } else {
        for (int64_t i = 0; i < nr; ++i) {
            rows[i] = i;
            cols[i] = w.col4row[i];
        }
    }
    return LsapStatus::kOk;
}

}  // namespace mmltk
