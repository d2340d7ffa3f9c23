// acc_emul.cpp — CPU check of the exact sequential-f32 emulation used by the kernels.
//
// Replays the tile algorithm of acc_tile (llama.rs_b200/csrc/lrs_kernels.cu) serially,
// with the kernel's own grid arithmetic (lrs_grid.h): order-free increments on one
// binade grid, and exact hardware operations only at events (ties, big elements, grid
// changes, stops).  Every result is compared bit for bit with plain sequential f32
// arithmetic, the semantics of rust-llama src/ops.rs:408-411 and src/sampler.rs:137-158.
// Build: g++ -O2 -ffp-contract=off -fno-fast-math -I<csrc> acc_emul.cpp
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "lrs_grid.h"

using namespace lrs;

static const float kInf = INFINITY;

// Serial replay of acc_tile: returns the stop position or -1; updates s.
static int acc_emul(const std::vector<float>& v, int cnt, int dir, float& s, float thr) {
    int consumed = -1;
    float cur = s;
    for (;;) {
        const int uu = unit_exp(cur);
        const uint32_t A = grid_count(cur, uu);
        const uint32_t lower = (uu == -149) ? 0u : kTwo23;
        float tq = kInf;
        if (dir > 0 && thr < kInf) tq = ldexpf(thr, -uu);
        std::vector<uint32_t> inc(cnt, 0);
        std::vector<char> ev(cnt, 0);
        uint32_t total = 0;
        bool any = false, nonzero = false;
        for (int i = consumed + 1; i < cnt; ++i) {
            Cls c = classify(lrs_f2u(v[i]), uu);
            inc[i] = c.inc;
            ev[i] = c.tie || c.big;
            any |= ev[i];
            nonzero |= v[i] != 0.0f;
            total = sat_add(total, c.inc);
        }
        if (!nonzero) {  // nothing left that can change s
            s = cur;
            return -1;
        }
        bool fast = dir > 0 ? (!any && A + total <= kTwo24 - 1u && (float)(A + total) < tq)
                            : (!any && total < A - lower);
        if (fast) {
            s = grid_value(uu, dir > 0 ? A + total : A - total);
            return -1;
        }
        uint32_t run = 0;
        int first = -1;
        uint32_t first_excl = 0;
        for (int i = consumed + 1; i < cnt; ++i) {
            const uint32_t excl = run;
            run = sat_add(run, inc[i]);
            bool e = ev[i];
            if (dir > 0)
                e = e || (A + run >= kTwo24) || ((float)(A + run) >= tq);
            else
                e = e || (run >= A - lower);
            if (e) {
                first = i;
                first_excl = excl;
                break;
            }
        }
        if (first < 0) {
            fprintf(stderr, "no event found\n");
            exit(3);
        }
        const float before = grid_value(uu, dir > 0 ? A + first_excl : A - first_excl);
        float after;
        bool stop;
        if (dir > 0) {
            after = before + v[first];
            stop = after >= thr;
        } else {
            after = before - v[first];
            stop = after <= 0.0f;
        }
        if (stop) {
            s = after;
            return first;
        }
        cur = after;
        consumed = first;
    }
}

// Reference: plain sequential f32 arithmetic.
static int seq_ref(const std::vector<float>& v, int cnt, int dir, float& s, float thr) {
    for (int i = 0; i < cnt; ++i) {
        if (dir > 0) {
            s = s + v[i];
            if (s >= thr) return i;
        } else {
            s = s - v[i];
            if (s <= 0.0f) return i;
        }
    }
    return -1;
}

static int failures = 0;

static void check_seq(const std::vector<float>& vals, int dir, float s0, float thr, const char* what, int tile) {
    float a = s0, b = s0;
    int pa = -1, pb = -1;
    for (size_t t0 = 0; t0 < vals.size(); t0 += tile) {
        const int cnt = (int)std::min<size_t>(tile, vals.size() - t0);
        std::vector<float> chunk(vals.begin() + t0, vals.begin() + t0 + cnt);
        int p = acc_emul(chunk, cnt, dir, a, thr);
        if (p >= 0) {
            pa = (int)t0 + p;
            break;
        }
    }
    pb = seq_ref(vals, (int)vals.size(), dir, b, thr);
    if (pa != pb || lrs_f2u(a) != lrs_f2u(b)) {
        if (failures < 10)
            fprintf(stderr, "%s: emul stop %d value %a | sequential stop %d value %a\n", what, pa, a, pb, b);
        ++failures;
    }
}

int main() {
    std::mt19937_64 rng(12345);
    std::uniform_real_distribution<double> U(0.0, 1.0);
    const int tiles[] = {1, 3, 64, 4096};
    for (int trial = 0; trial < 3000; ++trial) {
        const int n = 1 + (int)(rng() % 20000);
        const int kind = (int)(rng() % 8);
        std::vector<float> v(n);
        for (int i = 0; i < n; ++i) {
            double x;
            switch (kind) {
                case 0: x = std::exp(-60.0 * U(rng)); break;                        // wide range
                case 1: x = std::exp(-3.0 * U(rng)); break;                         // flat
                case 2: x = std::ldexp(std::floor(U(rng) * 64) + 0.5, -30); break;  // ties on many grids
                case 3: x = 1.0; break;                                              // equal values
                case 4: x = std::ldexp(1.0, -(int)(rng() % 150)); break;            // powers of two, subnormals
                case 5: x = U(rng) < 0.01 ? 1.0 : std::exp(-20.0 * U(rng)); break;  // spiky
                case 6: x = std::ldexp((double)(rng() % 3), -149); break;           // subnormal steps
                default: x = U(rng) * 1e-6; break;
            }
            v[i] = (float)x;
        }
        const int tile = tiles[rng() % 4];
        // sums from zero (softmax denominator), no stop
        check_seq(v, +1, 0.0f, kInf, "sum", tile);
        // descending order with a top-p style stop
        std::vector<float> d = v;
        std::sort(d.begin(), d.end(), [](float a, float b) { return a > b; });
        double tot = 0;
        for (float x : d) tot += x;
        const float thr = (float)(tot * (0.5 + 0.5 * U(rng)));
        check_seq(d, +1, 0.0f, thr, "cum", tile);
        // the draw: r0 = u * sum, subtract in sorted order until <= 0
        float s = 0;
        for (float x : d) s += x;
        const float u = (float)(rng() >> 40) / 16777216.0f;
        check_seq(d, -1, u * s, 0.0f, "walk", tile);
    }
    if (failures) {
        fprintf(stderr, "%d failures\n", failures);
        return 1;
    }
    printf("acc_emul: ok\n");
    return 0;
}
