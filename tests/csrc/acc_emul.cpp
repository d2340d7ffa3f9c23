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

// Serial replay of the two-grid tile algorithm (the kernels' tile2 / sum-pass tiles):
// classify on grids uu and uu + dir, one prefix per grid, ordered steps only where
// needs_step says so, falling back to acc_emul after a second grid change.
static int tile2_emul(const std::vector<float>& v, int cnt, int start, int dir, float& s, float thr) {
    const int uu = unit_exp(s);
    std::vector<Cls2> c(cnt);
    std::vector<uint32_t> incl0(cnt, 0), incl1(cnt, 0);
    uint32_t tot0 = 0, r0 = 0, r1 = 0;
    bool spec0 = false, nonzero = false;
    for (int i = start; i < cnt; ++i) {
        c[i] = classify2(lrs_f2u(v[i]), uu, dir);
        tot0 = sat_add(tot0, c[i].inc0);
        spec0 |= c[i].spec0;
        nonzero |= v[i] != 0.0f;
        r0 = sat_add(r0, c[i].inc0);
        r1 = sat_add(r1, c[i].inc1);
        incl0[i] = r0;
        incl1[i] = r1;
    }
    if (!nonzero) return -1;
    {
        const uint32_t A = grid_count(s, uu);
        const float tq = (dir > 0 && thr < kInf) ? ldexpf(thr, -uu) : kInf;
        const bool fast = dir > 0 ? (!spec0 && A + tot0 <= kTwo24 - 1u && (float)(A + tot0) < tq)
                                  : (!spec0 && tot0 < A - grid_lower(uu));
        if (fast) {
            s = grid_value(uu, dir > 0 ? A + tot0 : A - tot0);
            return -1;
        }
    }
    int consumed = start - 1;
    float cur = s;
    uint32_t base0 = 0, base1 = 0;
    for (;;) {
        const int ucur = unit_exp(cur);
        int ch = ucur == uu ? 0 : (ucur == channel_uu(uu, dir, 1) ? 1 : -1);
        if (ch < 0) {  // a second grid change: general algorithm for the rest
            std::vector<float> rest(v.begin() + consumed + 1, v.begin() + cnt);
            s = cur;
            const int p = acc_emul(rest, (int)rest.size(), dir, s, thr);
            return p < 0 ? -1 : consumed + 1 + p;
        }
        const uint32_t A = grid_count(cur, ucur);
        const uint32_t lower = grid_lower(ucur);
        const float tq = (dir > 0 && thr < kInf) ? ldexpf(thr, -ucur) : kInf;
        const uint32_t base = ch == 0 ? base0 : base1;
        int first = -1;
        for (int i = consumed + 1; i < cnt; ++i) {
            const uint32_t incl = ch == 0 ? incl0[i] : incl1[i];
            const bool sp = ch == 0 ? c[i].spec0 : c[i].spec1;
            if (needs_step(dir, sp, A, incl - base, lower, tq)) {
                first = i;
                break;
            }
        }
        if (first < 0) {
            const uint32_t tot = (ch == 0 ? incl0[cnt - 1] : incl1[cnt - 1]) - base;
            s = grid_value(ucur, dir > 0 ? A + tot : A - tot);
            return -1;
        }
        const uint32_t inc = ch == 0 ? c[first].inc0 : c[first].inc1;
        const uint32_t excl = (ch == 0 ? incl0[first] : incl1[first]) - inc - base;
        const float before = grid_value(ucur, dir > 0 ? A + excl : A - excl);
        const float after = dir > 0 ? before + v[first] : before - v[first];
        const bool stop = dir > 0 ? after >= thr : after <= 0.0f;
        if (stop) {
            s = after;
            return first;
        }
        cur = after;
        consumed = first;
        base0 = incl0[first];
        base1 = incl1[first];
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

static void check_seq(const std::vector<float>& vals, int dir, float s0, float thr, const char* what, int tile,
                      bool two = false) {
    float a = s0, b = s0;
    int pa = -1, pb = -1;
    for (size_t t0 = 0; t0 < vals.size(); t0 += tile) {
        const int cnt = (int)std::min<size_t>(tile, vals.size() - t0);
        std::vector<float> chunk(vals.begin() + t0, vals.begin() + t0 + cnt);
        int p = two ? tile2_emul(chunk, cnt, 0, dir, a, thr) : acc_emul(chunk, cnt, dir, a, thr);
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

// The kernels' fast path rounds a value e < B = 2^23 * U onto the grid with two float
// operations, inc = (B + e) - B, and detects ties as |e - inc| == U / 2.  It must agree
// with the integer classification on every non-big, non-tie value.
static void check_fp_increment(std::mt19937_64& rng) {
    for (int t = 0; t < 2000000; ++t) {
        const int uu = -148 + (int)(rng() % 170);
        const float bm = grid_value(uu, kTwo23);
        const float halfu = ldexpf(1.0f, uu - 1);
        // e spread over the grid's useful range [U/4, B)
        const uint32_t lo = lrs_f2u(ldexpf(1.0f, uu - 2)), hi = lrs_f2u(bm);
        const uint32_t eb = lo + (uint32_t)(rng() % (hi - lo));
        const float e = lrs_u2f(eb);
        const Cls c = classify(eb, uu);
        const float inc = (bm + e) - bm;
        const float rr = std::fabs(e - inc);
        const bool tie = rr == halfu;
        if (tie != c.tie) {
            if (failures < 10) fprintf(stderr, "fp tie mismatch e=%a uu=%d\n", e, uu);
            ++failures;
            continue;
        }
        if (!c.tie && !c.big && lrs_f2u(inc) != lrs_f2u(ldexpf((float)c.inc, uu))) {
            if (failures < 10) fprintf(stderr, "fp inc mismatch e=%a uu=%d inc=%a int=%u\n", e, uu, inc, c.inc);
            ++failures;
        }
    }
}

int main() {
    std::mt19937_64 rng(12345);
    check_fp_increment(rng);
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
        check_seq(v, +1, 0.0f, kInf, "sum2", tile, true);
        // descending order with a top-p style stop
        std::vector<float> d = v;
        std::sort(d.begin(), d.end(), [](float a, float b) { return a > b; });
        double tot = 0;
        for (float x : d) tot += x;
        const float thr = (float)(tot * (0.5 + 0.5 * U(rng)));
        check_seq(d, +1, 0.0f, thr, "cum", tile);
        check_seq(d, +1, 0.0f, thr, "cum2", tile, true);
        // the draw: r0 = u * sum, subtract in sorted order until <= 0
        float s = 0;
        for (float x : d) s += x;
        const float u = (float)(rng() >> 40) / 16777216.0f;
        check_seq(d, -1, u * s, 0.0f, "walk", tile);
        check_seq(d, -1, u * s, 0.0f, "walk2", tile, true);
    }
    if (failures) {
        fprintf(stderr, "%d failures\n", failures);
        return 1;
    }
    printf("acc_emul: ok\n");
    return 0;
}
