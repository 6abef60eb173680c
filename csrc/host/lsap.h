// Rectangular linear sum assignment (shortest augmenting path with dual
// potentials, the method of D. F. Crouse, "On implementing 2D rectangular
// assignment algorithms", IEEE TAES 52(4), 2016 -- the algorithm behind
// scipy.optimize.linear_sum_assignment and the reference's
// `src/rfdetr/utils/scipy_rectangular_lsap.cpp`).
//
// Written for this framework: the solver keeps a reusable workspace so a
// batch of thousands of small problems (layers x images x Group-DETR groups)
// allocates nothing per problem.
#pragma once

#include <cstdint>
#include <vector>

namespace mmltk {

enum class LsapStatus { kOk = 0, kInfeasible = 1, kInvalid = 2 };

struct LsapWorkspace {
    std::vector<double> u, v, spc, transposed;
    std::vector<int64_t> path, col4row, row4col, remaining;
    std::vector<char> sr, sc;
};

// cost: nr x nc, row-major.  On success writes min(nr, nc) pairs into
// rows/cols (rows ascending), like scipy.
LsapStatus lsap_solve(int64_t nr, int64_t nc, const double* cost, bool maximize, int64_t* rows, int64_t* cols,
                      LsapWorkspace& ws);

// Replace non-finite entries by (max finite + max |finite| + 1), as the
// reference matcher does before solving (`src/rfdetr/detection_ops.cpp:412-459`).
void lsap_sanitize(double* cost, int64_t n);

}  // namespace mmltk
