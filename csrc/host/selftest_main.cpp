// Host self-test of the torch-free runtime sources, built as a stand-alone executable for the
// sanitizer build (`python -m mmltk_b200.build --host-sanitize address,undefined`): AddressSanitizer
// and UndefinedBehaviorSanitizer watch every access while it runs.  Exit code 0 = all checks held.
//
// Covers: the rectangular LSAP solver against brute force on small random problems (square, tall,
// wide, with non-finite entries sanitised first), the worker pool (parallel_for, nested calls that
// must run inline, enqueue futures), the PNG codec round trip and the two resizers.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <numeric>
#include <random>
#include <vector>

#include "image_io.h"
#include "lsap.h"
#include "worker_pool.h"

namespace {

int g_failures = 0;

void check(bool ok, const char* what) {
    if (!ok) {
        std::fprintf(stderr, "selftest FAILED: %s\n", what);
        ++g_failures;
    }
}

// minimum total cost over all injective row->column (or column->row) assignments
double brute_force(int nr, int nc, const std::vector<double>& c) {
    const bool rows_small = nr <= nc;
    const int k = rows_small ? nr : nc, m = rows_small ? nc : nr;
    std::vector<int> perm(m);
    std::iota(perm.begin(), perm.end(), 0);
    double best = std::numeric_limits<double>::infinity();
    do {
        double s = 0;
        for (int i = 0; i < k; ++i) s += rows_small ? c[i * nc + perm[i]] : c[perm[i] * nc + i];
        best = std::min(best, s);
    } while (std::next_permutation(perm.begin(), perm.end()));
    return best;
}

void test_lsap() {
    std::mt19937 rng(7);
    std::uniform_real_distribution<double> U(0.0, 10.0);
    mmltk::LsapWorkspace ws;
    const int shapes[][2] = {{1, 1}, {3, 3}, {5, 5}, {2, 6}, {6, 3}, {4, 7}, {7, 4}, {6, 6}};
    for (int rep = 0; rep < 40; ++rep) {
        for (const auto& sh : shapes) {
            const int nr = sh[0], nc = sh[1];
            std::vector<double> c(static_cast<size_t>(nr) * nc);
            for (auto& v : c) v = U(rng);
            if (rep % 5 == 0) c[rng() % c.size()] = std::numeric_limits<double>::infinity();
            mmltk::lsap_sanitize(c.data(), static_cast<int64_t>(c.size()));
            for (double v : c) check(std::isfinite(v), "lsap_sanitize leaves only finite costs");
            const int k = std::min(nr, nc);
            std::vector<int64_t> rows(k), cols(k);
            const auto st = mmltk::lsap_solve(nr, nc, c.data(), false, rows.data(), cols.data(), ws);
            check(st == mmltk::LsapStatus::kOk, "lsap_solve status");
            double s = 0;
            std::vector<char> used_r(nr, 0), used_c(nc, 0);
            for (int i = 0; i < k; ++i) {
                check(rows[i] >= 0 && rows[i] < nr && cols[i] >= 0 && cols[i] < nc, "lsap index range");
                check(!used_r[rows[i]] && !used_c[cols[i]], "lsap assignment is injective");
                used_r[rows[i]] = used_c[cols[i]] = 1;
                if (i > 0) check(rows[i] > rows[i - 1], "lsap rows ascending");
                s += c[rows[i] * nc + cols[i]];
            }
            check(std::fabs(s - brute_force(nr, nc, c)) < 1e-9, "lsap optimal vs brute force");
        }
    }
}

void test_worker_pool() {
    mmltk::WorkerPool pool(4);
    std::vector<int64_t> out(10000, 0);
    pool.parallel_for(static_cast<int64_t>(out.size()), [&](int64_t i) { out[i] = i * i; });
    bool ok = true;
    for (int64_t i = 0; i < static_cast<int64_t>(out.size()); ++i) ok = ok && out[i] == i * i;
    check(ok, "parallel_for writes every index once");
    // nested parallel_for from a worker runs inline instead of deadlocking
    std::vector<int> nested(64, 0);
    pool.parallel_for(8, [&](int64_t i) { pool.parallel_for(8, [&](int64_t j) { nested[i * 8 + j] += 1; }); });
    check(std::all_of(nested.begin(), nested.end(), [](int v) { return v == 1; }), "nested parallel_for");
    std::vector<std::future<void>> fs;
    std::vector<int> hits(16, 0);
    for (int i = 0; i < 16; ++i) fs.push_back(pool.enqueue([&hits, i] { hits[i] = i + 1; }));
    for (auto& f : fs) f.get();
    bool all = true;
    for (int i = 0; i < 16; ++i) all = all && hits[i] == i + 1;
    check(all, "enqueue futures complete");
    check(mmltk::format_cpuset(mmltk::parse_cpuset("0-3,8,10-11")) == "0-3,8,10-11", "cpuset round trip");
}

void test_image_io() {
    const int W = 37, H = 23;
    std::vector<uint8_t> px(static_cast<size_t>(W) * H * 3);
    for (size_t i = 0; i < px.size(); ++i) px[i] = static_cast<uint8_t>((i * 7 + 3) & 0xff);
    const auto png = mmltk::img::encode_png(px.data(), W, H, 3);
    const auto back = mmltk::img::decode_png(png.data(), png.size());
    check(back.width == W && back.height == H && back.rgb == px, "PNG round trip");
    std::vector<float> planar(3 * 11 * 17);
    mmltk::img::resize_rgb_to_planar(back, 17, 11, planar.data());
    check(std::all_of(planar.begin(), planar.end(), [](float v) { return v >= 0.f && v <= 1.f; }), "resize range");
    std::vector<float> up(3 * 50 * 70);
    mmltk::img::resize_rgb_to_planar(back, 70, 50, up.data());
    check(std::all_of(up.begin(), up.end(), [](float v) { return v >= 0.f && v <= 1.f; }), "upscale range");
    std::vector<uint8_t> mask(static_cast<size_t>(W) * H), small(9 * 13);
    for (size_t i = 0; i < mask.size(); ++i) mask[i] = (i % 5) == 0;
    mmltk::img::resize_mask_nearest(mask.data(), W, H, small.data(), 13, 9);
    check(std::all_of(small.begin(), small.end(), [](uint8_t v) { return v <= 1; }), "mask resize values");
    bool threw = false;
    try {
        const uint8_t junk[8] = {1, 2, 3, 4, 5, 6, 7, 8};
        (void)mmltk::img::decode_png(junk, sizeof(junk));
    } catch (const std::exception&) {
        threw = true;
    }
    check(threw, "corrupt PNG is rejected with an exception");
}

}  // namespace

int main() {
    test_lsap();
    test_worker_pool();
    test_image_io();
    if (g_failures) {
        std::fprintf(stderr, "selftest: %d check(s) failed\n", g_failures);
        return 1;
    }
    std::printf("host selftest ok\n");
    return 0;
}
