// qmv_table.cpp — regenerate the quantised mat-vec numerics table from the
// restated oracle (p100_oracle.cpp).
//
// TEST INFRASTRUCTURE ONLY.  The reference commits the output of its own
// generator (tests/qmv_numerics.cpp:15-62) as a golden table.  This program
// draws the same seeded inputs — weights from the random_row generator with
// seed 60060+K+type, activations from std::normal_distribution<float> with
// seed 20261010+K+distribution, the outlier/swiglu/large variants of
// tests/qmv_numerics.cpp:28-37 — evaluates every row through the restatement
// and prints the table in the same format, so a byte comparison with the
// reference's table pins the restatement.
#include "p100_oracle.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <iomanip>
#include <iostream>
#include <random>
#include <vector>

namespace {
struct Stats {
    std::vector<double> norm, rel;
    int nonfinite = 0;
};
double mid(std::vector<double> v) {  // 256 rows: mean of the two middle values
    std::sort(v.begin(), v.end());
    return (v[127] + v[128]) * 0.5;
}
const char* type_name(int t) { return t == 0 ? "q4_0" : t == 1 ? "q8_0" : "q4_K"; }
}  // namespace

int main() {
    std::cout << "Seeds: activations=20261010 + K + distribution_index; weights=60060 + K + type_index.\n"
              << "256 rows per cell; same weight rows across distributions; outlier uses four distinct channels.\n"
              << "Weight scales uniform [0.002,0.08], packed quant/scales bytes uniform [0,255].\n"
              << "type path distribution K norm_median norm_max relative_median relative_max nonfinite\n";
    bool bad = false;
    const char* paths[4] = {"q81", "h16<8>", "h16<16>", "h16_exact"};
    const char* dists[4] = {"normal", "outlier", "swiglu", "large"};
    for (int k : {4096, 14336}) {
        for (int t = 0; t < 3; ++t) {
            void* wrng = p100o_rng_new(60060u + k + t);
            const int row_bytes = k / p100o_block_elems(t) * p100o_block_bytes(t);
            std::vector<std::vector<uint8_t>> rows(256, std::vector<uint8_t>(row_bytes));
            for (auto& row : rows) p100o_random_row(t, k, wrng, row.data());
            p100o_rng_free(wrng);
            for (int di = 0; di < 4; ++di) {
                std::mt19937 rng(20261010u + k + di);
                std::normal_distribution<float> normal(0, 1);
                std::vector<float> x(k);
                for (auto& v : x) {
                    v = normal(rng);
                    if (di == 2) v *= normal(rng) * 3.f;
                    if (di == 3) v *= 1000.f;
                }
                if (di == 1) {
                    std::vector<int> pos(k);
                    for (int i = 0; i < k; ++i) pos[i] = i;
                    std::shuffle(pos.begin(), pos.end(), rng);
                    for (int i = 0; i < 4; ++i) x[pos[i]] *= 50.f;
                }
                double xn = 0;
                for (float v : x) xn += double(v) * v;
                xn = std::sqrt(xn);
                std::vector<p100o_act> acts(k / 32);
                p100o_prepare(x.data(), k, acts.data());
                std::array<Stats, 4> cells;
                for (const auto& w : rows) {
                    p100o_eval y;
                    p100o_evaluate(t, w.data(), x.data(), k, acts.data(), &y);
                    const double got[4] = {y.q81, y.h8, y.h16, y.h16_exact};
                    for (int j = 0; j < 4; ++j) {
                        const double err = std::fabs(got[j] - y.exact), scale = y.weight_norm * xn;
                        cells[j].norm.push_back(err / scale);
                        cells[j].rel.push_back(err / std::max(std::fabs(y.exact), 1e-6 * scale));
                        if (!std::isfinite(got[j])) {
                            ++cells[j].nonfinite;
                            bad = true;
                        }
                    }
                }
                for (int j = 0; j < 4; ++j) {
                    const Stats& c = cells[j];
                    std::cout << type_name(t) << ' ' << paths[j] << ' ' << dists[di] << ' ' << k << ' '
                              << std::scientific << std::setprecision(8) << mid(c.norm) << ' '
                              << *std::max_element(c.norm.begin(), c.norm.end()) << ' ' << mid(c.rel) << ' '
                              << *std::max_element(c.rel.begin(), c.rel.end()) << ' ' << c.nonfinite << '\n';
                }
            }
        }
    }
    return bad ? 1 : 0;
}
