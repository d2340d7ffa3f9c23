// lrs_grid.h — binade-grid arithmetic shared by the kernels (nvcc) and host tests (g++).
//
// A non-negative float s is A * 2^uu; while a running sum or difference stays on one
// grid (one binade, or the subnormal range plus the first normal binade), each f32
// operation s +/- v rounds v to a multiple of 2^uu independently of s (ties aside).
#pragma once
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define LRS_HD __host__ __device__ __forceinline__
#else
#define LRS_HD inline
#endif

namespace lrs {

constexpr uint32_t kSat = 1u << 25;   // saturation of increment sums (> 2^24)
constexpr uint32_t kTwo24 = 1u << 24;
constexpr uint32_t kTwo23 = 1u << 23;

LRS_HD uint32_t lrs_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
#endif
}
LRS_HD float lrs_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    std::memcpy(&f, &u, 4);
    return f;
#endif
}

// ------------------------------------------------------------- binade grids ----
// A non-negative float s is A * 2^uu with uu = max(expfield, 1) - 150 and integer
// A < 2^24 (A >= 2^23 unless s < 2^-126).  All values with the same uu share one
// rounding grid; bits(s) = ((uu + 149) << 23) + A for every such pair, including
// A == 2^24 (the next binade's base).
LRS_HD int unit_exp(float s) {
    const int f = (int)(lrs_f2u(s) >> 23);
    return (f > 1 ? f : 1) - 150;
}
LRS_HD uint32_t grid_count(float s, int uu) {
    return lrs_f2u(s) - ((uint32_t)(uu + 149) << 23);
}
LRS_HD float grid_value(int uu, uint32_t a) {
    return lrs_u2f(((uint32_t)(uu + 149) << 23) + a);
}

// Increment of v >= 0 on the grid of unit 2^uu: inc = RN(v / 2^uu) for non-ties.
// tie: v / 2^uu has fractional part exactly 1/2 (result then depends on parity).
// big: inc >= 2^23 (v alone spans half a binade; always handled exactly).
struct Cls {  // inc <= 2^23 always
    uint32_t inc;
    bool tie;
    bool big;
};
LRS_HD Cls classify(uint32_t vb, int uu) {
    Cls c{0u, false, false};
    int ee = (int)(vb >> 23);
    uint32_t m = vb & 0x7FFFFFu;
    if (ee) m |= 0x800000u; else ee = 1;
    const int sh = uu - (ee - 150);
    if (sh <= 0) {
        if (-sh >= 8) { c.inc = kTwo23; c.big = true; return c; }
        c.inc = m << (-sh);
    } else if (sh >= 25) {
        return c;
    } else {
        const uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u);
        const uint32_t half = 1u << (sh - 1);
        c.inc = q + (rem > half ? 1u : 0u);
        c.tie = (rem == half);
    }
    // An element spanning half a binade or more is always an ordered event; its
    // increment is capped so prefix sums before the first event never saturate.
    if (c.inc >= kTwo23) {
        c.inc = kTwo23;
        c.big = true;
    }
    return c;
}

LRS_HD uint32_t sat_add(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;
    return s < kSat ? s : kSat;
}


// ------------------------------------------------------------ two-grid tiles ----
// A tile is classified on two grids at once: channel 0 is the running value's grid
// at the tile start (unit 2^uu), channel 1 the grid it moves to after one binade step
// (2^(uu+1) for sums, 2^(uu-1) for the draw's decreasing differences).  A tile whose
// running value crosses one binade is then finished from one prefix scan per channel;
// only a second crossing needs a re-classification.
LRS_HD int channel_uu(int uu, int dir, int c) {
    if (c == 0) return uu;
    const int u1 = uu + dir;
    return u1 < -149 ? -149 : u1;
}

struct Cls2 {
    uint32_t inc0, inc1;
    bool spec0, spec1;  // tie or big on that grid: always an ordered step
};
LRS_HD Cls2 classify2(uint32_t vb, int uu, int dir) {
    const Cls a = classify(vb, channel_uu(uu, dir, 0));
    const Cls b = classify(vb, channel_uu(uu, dir, 1));
    return Cls2{a.inc, b.inc, a.tie || a.big, b.tie || b.big};
}

// Lowest grid count a difference may reach on grid uu before leaving it.
LRS_HD uint32_t grid_lower(int uu) { return uu == -149 ? 0u : kTwo23; }

// Does the element at inclusive prefix `rel` (increments since the last ordered step,
// on the current grid) need an ordered step?  a: grid count of the running value at
// the last ordered step; tq: stop threshold in grid units (sums), +inf if none.
LRS_HD bool needs_step(int dir, bool spec, uint32_t a, uint32_t rel, uint32_t lower, float tq) {
    if (spec) return true;
    if (dir > 0) return a + rel >= kTwo24 || (float)(a + rel) >= tq;
    return rel >= a - lower;
}

}  // namespace lrs
