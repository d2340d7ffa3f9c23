// lrs_kernels.cu — the batched token-sampling kernel (sm_100a).
//
// Computes, for every row, exactly what rust-llama's Sampler::sample computes
// (src/sampler.rs:56-163 with ops::softmax_inplace, src/ops.rs:397-419):
//   greedy fast path (sampler.rs:62-70), windowed once-per-token repetition penalty
//   (sampler.rs:82-102), greedy after penalty (104-113), temperature (115-118),
//   softmax (ops.rs:397-419), top-k (122-132), top-p (135-146), survivor sum (148-151)
//   and the categorical draw with the row's xorshift64* state (152-162).
//
// Structure.  A persistent CTA (two per SM) has seven consumer warps and one producer
// warp.  The producer takes rows from a global counter, passes them to the consumers
// through a small row queue and streams each row through a ring of 4 KB shared-memory
// slots with bulk copies (TMA engine; a slot's `full` mbarrier completes on the bytes,
// its `empty` mbarrier is released by the warp that consumed it).  A slot holds one tile
// of 1024 floats; consumer warp w takes tiles w, w+7, w+14, ... and each lane owns a run
// of 32 consecutive elements of the tile.
//   pass 1  per tile: the max (NaN-propagating), the argmax of greedy rows, the tile's
//           online-softmax statistics (its max and the sum of exp relative to it), on
//           path K a per-warp streaming top-k filter, and the tile's candidate list: the
//           elements no more than 18.1 below a lower bound of the running max (the only
//           ones that can change the softmax sum or reach a path-N bucket).  A tile with
//           more than kDense candidates is marked dense instead.
//   prep    the row max; from the tile statistics an estimate of the running softmax
//           sum at every tile start with a proven relative error bound, hence the
//           lowest binade grid the exact running sum can be on there and a threshold
//           below which an element cannot change it.  Tiles without a live element are
//           skipped by pass 2; the producer streams only the dense tiles again.
//   pass 2  per lane, the increments of its run on the two grids the running sum can
//           be on over that run (lrs_grid.h), from the staged tile (dense) or from the
//           candidate list (sparse).  The exact running sum is then handed from tile to
//           tile (a baton in shared memory); each hand-over is one warp scan of the 32
//           lane increments, and only a run with a binade crossing, a tie, an element of
//           half a binade or a missed grid is summed element by element with hardware
//           f32 adds.
//   finish  path K (top_k <= kKMax): the filter's candidates sorted in shared memory;
//           path N: candidates bucketed by (max - x) during pass 2, gathered into global
//           scratch with approximate keys, and made exact and sorted bucket by bucket
//           only where the top-p scan and the draw need the order (sampler.rs:122-162).
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/llamars_sampler.h"
#include "lrs_device.cuh"
#include "lrs_kernels_decl.cuh"

namespace lrs {

constexpr int kTile = 1024;          // floats per ring slot = one warp tile
constexpr int kSlots = 12;           // ring depth
constexpr int kRowQ = 4;             // row queue depth
constexpr int kBlock = kThreads + 32;  // consumer warps + the producer warp
constexpr int kKMax = 128;           // path K handles 1 <= k <= kKMax (k < n)
constexpr int kWCap = 256;           // per-warp path-K candidate buffer (entries)
constexpr int kKCap = kWarps * kWCap;  // union of the warp buffers
constexpr int kKSortMax = 2048;      // path K candidates kept after the final compaction
constexpr int kNB = 580;             // path N buckets of width 1/32 in (max - x); the last is
                                     // everything below the candidate lists' range (d < -579/32)
constexpr float kBScale = 32.0f;
constexpr int kSortCap = 4096;       // largest bucket sorted in shared memory
constexpr uint32_t kGatherItemsOff = 1024;  // path-N gather: per-warp item lists, in 32-bit words after the cursors
constexpr float kTopPMargin = 0.002f;     // first-gather limit: head mass reached by (top_p + this) S
constexpr float kTailMargin = 4.8828125e-04f;  // ... or tail mass at most (1 - top_p - this) S (2^-11:
                                           // the f32 rounding of a cumulative sum of a few thousand terms)
constexpr int kSerial = 512;         // elements summed one by one at the start of a scan
constexpr int kTilesSmem = 256;      // tile records kept in shared memory (larger rows: global)
constexpr int kMaxTiles = 4096;      // tiles of the longest row (n <= 2^22)
constexpr int kGatherRuns = 48;      // path-N gather: dense runs a warp stages at a time
constexpr int kDense = 256;          // a tile with more candidates is streamed again in pass 2
constexpr int kRunS = kDense / 32;   // list entries per lane run of a sparse tile
constexpr uint32_t kDenseMark = 0xFFFFFFFFu;  // TileRec::lcnt of a dense tile
constexpr uint32_t kNoTag = 0xFFFFFFFFu;
constexpr uint32_t kApxKey = 0x80000000u;  // path-N key flag: p from CUDA's expf, not yet exact
constexpr int kUBase = 149;          // skip-threshold table index = grid exponent + kUBase
constexpr int kNU = 288;
constexpr uint32_t kSumLive = 1u << 16;   // tile record flags
constexpr uint32_t kHistLive = 1u << 17;
constexpr long long kWaitCycles = 1ll << 32;  // bound of every wait (about 2 s)
constexpr float kLog2e = 1.44269504f;

// dynamic shared memory (bytes)
constexpr size_t kRingBytes = (size_t)kSlots * kTile * 4;
constexpr size_t kRegionABytes = (size_t)kWarps * kWCap * 8;  // warp candidate buffers | path-N counts + offsets
constexpr size_t kRegionBBytes = (size_t)kSortCap * 8;  // warp radix counts | candidates + keys | bucket sort
constexpr size_t kTTabBytes = (size_t)kTilesSmem * 32;
constexpr size_t kDynSmem = kRingBytes + kRegionABytes + kRegionBBytes + kTTabBytes;
static_assert(kRegionABytes >= (size_t)kKCap * 8, "warp candidate buffers");
static_assert(kRegionABytes >= (size_t)kNB * 8, "bucket counts and offsets");
static_assert(kRegionBBytes >= (size_t)kKCap * 8 + (size_t)kKSortMax * 8, "candidates and sort keys");
static_assert(kRegionBBytes >= (size_t)kWarps * 256 * 4, "per-warp radix counts");
static_assert(kRegionBBytes >= (size_t)kNB * 4, "bucket cursors");
static_assert(kRegionBBytes >= ((size_t)kGatherItemsOff + (size_t)kWarps * 1024) * 4, "gather item lists");
static_assert((size_t)kNB <= (size_t)kGatherItemsOff, "bucket cursors before the gather item lists");
static_assert((size_t)kWarps * kGatherRuns * 32 * 4 <= kRingBytes, "gather staging areas in the ring");
static_assert((size_t)kKCap * 8 + (size_t)kWarps * 32 * kRunS * 4 <= (size_t)kRegionBBytes, "pass-2 live list values");

using SampleArgs = lrs_kernel_args_t;

// One tile of a row (32 bytes; shared memory, or per-CTA scratch for long rows).
struct __align__(16) TileRec {
    float mt;        // pass 1: max of the tile's scaled logits
    uint32_t tag;    // pass 1: the row id once mt is final (kNoTag before); (mt, tag) is one 64-bit word
    float pt;        // pass 1: sum of exp relative to mt; prep: estimate of the running sum at the tile
    uint32_t flags;  // prep: lowest grid exponent + 256 | kSumLive | kHistLive
    uint32_t next;   // prep: next sum-live tile (the baton's route)
    uint32_t loff;   // pass 1: first list entry (sparse tiles)
    uint32_t lcnt;   // pass 1: list entries, or kDenseMark
    uint32_t rank;   // prep: load number of a dense tile within pass 2
};

// ---------------------------------------------------------------- shared state ----
struct RowShared {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    uint64_t rq_full[kRowQ];
    uint64_t rq_empty[kRowQ];
    uint64_t bwait[kWarps];    // baton: one phase per hand-over to warp w (its next chain step)
    uint64_t gbar[kWarps];     // path-N gather: bulk copies into warp w's staging area
    uint32_t gph[kWarps];      // ... and the phase warp w waits for next
    uint32_t rq_row[kRowQ];
    volatile uint32_t abort;   // a wait ran out: every later wait returns at once
    volatile uint32_t bseq;    // baton: the tile whose chain step may run
    volatile float bval;       // baton: exact running sum before that tile
    uint32_t red[kWarps + 2];
    uint32_t red2[kWarps + 2];
    float fstate;
    int32_t stop;
    uint32_t cand_n;
    uint32_t cand_over;
    float theta;
    float delta_min;
    uint32_t ktheta;     // path K: largest threshold any warp has applied (order-preserving key)
    uint32_t kdelta;     // path K: smallest margin of a published threshold (float bits, >= 0)
    uint32_t hist256[256];
    float vk;
    uint32_t events;
    uint32_t ev_base0, ev_base1;
    uint32_t misc[8];
    float wmax[kWarps];
    float gvs[kWarps];
    uint32_t gis[kWarps];
    uint32_t wcnt[kWarps];
    float wdelta[kWarps];
    uint32_t wover;
    float xhist;
    float xthr[kNU];
    float ser[kSerial + 4];
    lrs_row_info info;     // the row's diagnostics, assembled by thread 0
    uint32_t dense[kMaxTiles / 32];  // pass 1: tiles streamed again in pass 2 (read by the producer)
    volatile uint32_t p1done;        // pass-1 tiles of two-pass rows finished by this CTA (monotone)
    volatile uint32_t claim_ok;      // rows taken by the consumers after which the producer may
                                     // claim the next one (monotone)
    uint32_t ndense;                 // dense tiles of the current row
    uint32_t bsorted[(kNB + 31) / 32];  // path N: buckets in exact sorted order
};

struct Geo {
    const float* row;
    uint32_t n, head, tail, nchunks, body;  // body: elements in the 16-byte aligned middle
};

__device__ __forceinline__ Geo row_geometry(const SampleArgs& a, uint32_t r) {
    Geo g;
    g.row = a.logits + (uint64_t)r * a.ld;
    g.n = a.n;
    const uintptr_t p = (uintptr_t)g.row;
    uint32_t head = (uint32_t)(((16u - (uint32_t)(p & 15u)) & 15u) >> 2);
    if (head > g.n) head = g.n;
    g.head = head;
    g.body = ((g.n - head) / 4u) * 4u;
    g.tail = g.n - head - g.body;
    g.nchunks = (g.body + kTile - 1) / kTile;
    return g;
}

__device__ __forceinline__ uint32_t chunk_count(const Geo& g, uint32_t c) {
    const uint32_t left = g.body - c * kTile;
    return left < (uint32_t)kTile ? left : (uint32_t)kTile;
}

// Streaming passes over a row: pass 2 exists for stochastic rows with n >= 2
// (sampler.rs:62 and 104: temperature <= 0 is greedy, NaN is not).
__device__ __forceinline__ uint32_t row_passes(const lrs_params& P, uint32_t n) {
    if (n == 0) return 0u;
    const bool stochastic = !(P.temperature <= 0.0f);
    return (stochastic && n >= 2) ? 2u : 1u;
}

// Rows are claimed roughly longest first, so that no CTA starts a long row near the
// end of the launch: the exact softmax sum costs more the higher the temperature
// (more elements can change it), and rows whose finish orders a large candidate set
// (top_k off or above kKMax, the path-N finish) cost more than the others.  Four
// temperature bands (from 1.25 down, 0.25 apart) times the two finishes; class 0 is
// claimed first, kRowClasses - 1 last (with greedy rows).
constexpr uint32_t kRowClasses = 8;
static_assert(kRowClasses == (uint32_t)kLrsRowCounters, "one row counter per claim class");
__device__ __forceinline__ uint32_t row_class(const lrs_params& P, uint32_t n) {
    if (row_passes(P, n) != 2u) return kRowClasses - 1;
    const uint32_t k = (P.top_k == 0 || P.top_k > n) ? n : P.top_k;
    const bool long_finish = !(k < n && k <= (uint32_t)kKMax);
    const float t = P.temperature;  // (NaN: the hottest band; such a row fails fast anyway)
    const uint32_t band = t < 0.75f ? 3u : t < 1.0f ? 2u : t < 1.25f ? 1u : 0u;
    return band * 2u + (long_finish ? 0u : 1u);
}

// Bounded wait on an mbarrier phase.  On timeout the CTA's abort flag and the sticky
// error word are set; every later wait then returns false at once, so all warps run
// their (bounded) loops to the end and leave.
__device__ __forceinline__ bool wait_bar_bounded(volatile uint32_t* abort, uint64_t* bar, uint32_t parity,
                                                 int32_t* err, long long bound) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > bound) {
            *abort = 1u;
            atomicExch(err, LRS_E_TIMEOUT);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool wait_bar(RowShared& sh, uint64_t* bar, uint32_t parity, int32_t* err) {
    return wait_bar_bounded(&sh.abort, bar, parity, err, kWaitCycles);
}

// Test of the bounded wait: one thread waits for the first phase of an mbarrier that
// nothing arrives on, with a bound of `bound` cycles; the wait runs out, sets the error
// word to LRS_E_TIMEOUT and returns (no copy is in flight, no other thread waits).
__global__ void lrs_wait_probe(int32_t* err, long long bound) {
    __shared__ uint64_t bar;
    __shared__ volatile uint32_t abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort = 0u;
        (void)wait_bar_bounded(&abort, &bar, 0u, err, bound);
    }
}

// Bounded wait until load q of the ring has landed.  A parity wait only distinguishes
// the current phase of an mbarrier from the one before it, and bulk copies may land out
// of order while warps run tiles apart; so first wait until the slot's previous use
// (load q - kSlots) was released by its consumer: then the slot's `full` barrier is in
// the phase of load q and the parity wait is exact.
__device__ __forceinline__ bool wait_full(RowShared& sh, uint32_t q, int32_t* err) {
    const uint32_t s = q % kSlots, use = q / kSlots;
    if (use > 0 && !wait_bar(sh, &sh.empty[s], (use - 1) & 1u, err)) return false;
    return wait_bar(sh, &sh.full[s], use & 1u, err);
}

// ------------------------------------------------------------- producer warp ----
// One thread: takes rows, publishes them in the row queue, and issues the bulk copies
// in the order the consumers take them (load q lands in slot q % kSlots and completes
// phase (q / kSlots) & 1 of its `full` barrier): every tile for pass 1; then, once the
// consumers have finished the row's pass 1, the dense tiles again for pass 2.
__device__ __noinline__ void producer(const SampleArgs& a, RowShared& sh, float* ring) {
    const uint64_t pol_keep = policy_evict_last(), pol_drop = policy_evict_first();
    uint32_t q = 0, rqi = 0, p1target = 0, sweep = 0;
    // next row: sweep c over the rows claims the rows of class c (each sweep has its
    // own counter, so every row is claimed exactly once)
    auto claim = [&]() -> uint32_t {
        if (a.order) {  // rows in the order of the ordering pass (or a given list of rows)
            const uint32_t i = atomicAdd(a.row_counter, 1u);
            const uint32_t lim = a.claim_count ? *(volatile const uint32_t*)a.claim_count : a.rows;
            return i < lim ? __ldcg(a.order + i) : a.rows;
        }
        for (;;) {
            const uint32_t r = atomicAdd(a.row_counter + sweep, 1u);
            if (r >= a.rows) {
                if (sweep + 1u == kRowClasses) return a.rows;
                ++sweep;
                continue;
            }
            if (row_class(a.params[r], a.n) == sweep) return r;
        }
    };
    auto issue = [&](const Geo& g, uint32_t c, uint64_t pol) -> bool {
        const uint32_t s = q % kSlots, use = q / kSlots;
        if (use > 0 && !wait_bar(sh, &sh.empty[s], (use - 1) & 1u, a.err_flag)) return false;
        const uint32_t bytes = chunk_count(g, c) * 4u;
        mbar_expect_tx(&sh.full[s], bytes);
        bulk_load(ring + (size_t)s * kTile, g.row + g.head + (size_t)c * kTile, bytes, &sh.full[s], pol);
        ++q;
        return true;
    };
    for (;;) {
        const uint32_t qs = rqi % kRowQ, use = rqi / kRowQ;
        if (use > 0 && !wait_bar(sh, &sh.rq_empty[qs], (use - 1) & 1u, a.err_flag)) break;
        const uint32_t r = sh.abort ? a.rows : claim();
        sh.rq_row[qs] = r < a.rows ? r : a.rows;
        mbar_arrive(&sh.rq_full[qs]);
        ++rqi;
        if (r >= a.rows) break;
        const Geo g = row_geometry(a, r);
        const uint32_t passes = row_passes(a.params[r], g.n);
        bool ok = true;
        for (uint32_t c = 0; c < g.nchunks && ok; ++c) ok = issue(g, c, pol_keep);
        if (!ok) break;
        if (passes == 2 && g.nchunks) {
            p1target += g.nchunks;
            const long long t0 = clock64();
            while ((int)(sh.p1done - p1target) < 0) {
                if (sh.abort) break;
                if (clock64() - t0 > kWaitCycles) {
                    sh.abort = 1u;
                    atomicExch(a.err_flag, LRS_E_TIMEOUT);
                    break;
                }
                __nanosleep(64);
            }
            if (sh.abort) break;
            __threadfence_block();
            for (uint32_t c = 0; c < g.nchunks && ok; ++c)
                if ((sh.dense[c >> 5] >> (c & 31)) & 1u) ok = issue(g, c, pol_drop);
            if (!ok) break;
        }
        if (passes == 2) {
            // A two-pass row can run long after its last load (pass 2, a long finish): the
            // next row is claimed only once the consumers say the row is nearly done, so
            // that a CTA still busy with a long row leaves the remaining rows to others.
            // (Bounded at 16 times the usual wait: a whole row's work lies in between, and
            // the consumers' own waits are bounded separately.)
            const long long t0 = clock64();
            while ((int)(sh.claim_ok - rqi) < 0) {
                if (sh.abort) break;
                if (clock64() - t0 > 16 * kWaitCycles) {
                    sh.abort = 1u;
                    atomicExch(a.err_flag, LRS_E_TIMEOUT);
                    break;
                }
                __nanosleep(256);
            }
            if (sh.abort) break;
        }
    }
    // Leave no copy in flight behind: wait (bounded, ignoring the abort flag) for the
    // last kSlots loads to land.
    for (uint32_t j = q > (uint32_t)kSlots ? q - kSlots : 0u; j < q; ++j) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&sh.full[j % kSlots], (j / kSlots) & 1u))
            if (clock64() - t0 > kWaitCycles) break;
    }
}

// --------------------------------------------------------------- block helpers ----
__device__ __forceinline__ int li_of(int i) {  // local position of per-thread slot i
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    return w * 512 + (i >> 2) * 128 + l * 4 + (i & 3);
}

// Saturating inclusive prefix (in local-position order) of per-thread incs.
// Returns per-slot inclusive sums in incl[].
__device__ __forceinline__ uint32_t block_incl_scan(const uint32_t (&inc)[kVpt], uint32_t (&incl)[kVpt],
                                                    uint32_t* sh) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    uint32_t jtot[4], jexcl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t s = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) s = sat_add(s, inc[j * 4 + e]);
        const uint32_t sc = warp_incl_scan(s);
        const uint32_t up = __shfl_up_sync(0xFFFFFFFFu, sc, 1);
        jexcl[j] = l == 0 ? 0u : up;
        jtot[j] = __shfl_sync(0xFFFFFFFFu, sc, 31);
    }
    uint32_t wt = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) wt = sat_add(wt, jtot[j]);
    csync();
    if (l == 0) sh[w] = wt;
    csync();
    uint32_t off = 0, total = 0;
    for (int i = 0; i < kWarps; ++i) {
        if (i < w) off = sat_add(off, sh[i]);
        total = sat_add(total, sh[i]);
    }
    uint32_t jb = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t run = sat_add(sat_add(off, jb), jexcl[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            run = sat_add(run, inc[j * 4 + e]);
            incl[j * 4 + e] = run;
        }
        jb = sat_add(jb, jtot[j]);
    }
    return total;
}

// Exact emulation of a run of sequential f32 operations over one tile of values in
// local-position order (sampler.rs:137-139 / 148-151 / 156-158, ops.rs:408-411).
//   dir > 0: s <- fl(s + v), stop at the first position with s >= thr (thr may be +inf);
//   dir < 0: s <- fl(s - v), stop at the first position with s <= 0.
// Values with their `exact` bit clear are approximations within 8 float steps of the
// exact value; exactify(i) returns the exact value of slot i when it matters.
// Positions >= cnt are ignored.  Returns the local stop position or -1 and leaves in
// s the value after the stop position (or after the tile).
template <typename Exactify>
__device__ __noinline__ int acc_tile(float (&v)[kVpt], uint32_t& exact, int cnt, int dir, float& s, float thr,
                        Exactify exactify, RowShared& sh, int start = 0) {
    int consumed = start - 1;
    float cur = s;
    for (int round = 0;; ++round) {
        const int uu = unit_exp(cur);
        const uint32_t A = grid_count(cur, uu);
        const uint32_t lower = (uu == -149) ? 0u : kTwo23;
        float tq = __int_as_float(0x7F800000);  // +inf: no stop
        if (dir > 0 && thr < __int_as_float(0x7F800000)) tq = ldexpf(thr, -uu);
        uint32_t inc[kVpt];
        uint32_t ev_local = 0;  // bit i: tie or big
        bool nonzero = false;   // some remaining value is > 0
        uint32_t tot = 0;
#pragma unroll 1
        for (int i = 0; i < kVpt; ++i) {
            const int li = li_of(i);
            inc[i] = 0;
            if (li < cnt && li > consumed) {
                Cls c;
                const uint32_t vb = __float_as_uint(v[i]);
                if (exact & (1u << i)) {
                    c = classify(vb, uu);
                } else {
                    const Cls lo = classify(vb > 8u ? vb - 8u : 0u, uu);
                    const Cls hi = classify(vb + 8u, uu);
                    if ((lo.inc == hi.inc && !lo.tie && !hi.tie && !lo.big && !hi.big) || (lo.big && hi.big)) {
                        c = lo;  // same increment (or big) for every value within the error bound
                    } else {
                        v[i] = exactify(i);
                        exact |= 1u << i;
                        c = classify(__float_as_uint(v[i]), uu);
                    }
                }
                inc[i] = c.inc;
                if (c.tie || c.big) ev_local |= 1u << i;
                nonzero |= v[i] != 0.0f;
                tot = sat_add(tot, c.inc);
            }
        }
        const uint32_t total = block_reduce_u32(tot, SatAdd(), sh.red);
        const uint32_t flags = block_reduce_u32((ev_local ? 1u : 0u) | (nonzero ? 2u : 0u), OrOp(), sh.red2);
        const bool any_ev = flags & 1u;
        if (!(flags & 2u)) {  // nothing left that can change s
            s = cur;
            return -1;
        }
        bool fast;
        if (dir > 0)
            fast = !any_ev && A + total <= kTwo24 - 1u && (float)(A + total) < tq;
        else
            fast = !any_ev && total < A - lower;
        if (fast) {
            s = grid_value(uu, dir > 0 ? A + total : A - total);
            return -1;
        }
        // Ordered path: find the first event (tie, big, grid change or stop).
        uint32_t incl[kVpt];
        (void)block_incl_scan(inc, incl, sh.red);
        uint32_t first = 0xFFFFFFFFu;
#pragma unroll 1
        for (int i = 0; i < kVpt; ++i) {
            const int li = li_of(i);
            if (li < cnt && li > consumed) {
                bool ev = (ev_local >> i) & 1u;
                if (dir > 0)
                    ev = ev || (A + incl[i] >= kTwo24) || ((float)(A + incl[i]) >= tq);
                else
                    ev = ev || (incl[i] >= A - lower);
                if (ev && (uint32_t)li < first) first = (uint32_t)li;
            }
        }
        first = block_reduce_u32(first, MinU(), sh.red2);
        if (first == 0xFFFFFFFFu) {
            // Only possible when saturation hid nothing: should not happen.
            atomicExch(&sh.misc[7], 1u);
            s = grid_value(uu, dir > 0 ? A + total : A - total);
            return -1;
        }
        // The owner of the event performs the exact operation.
#pragma unroll 1
        for (int i = 0; i < kVpt; ++i) {
            if ((uint32_t)li_of(i) == first) {
                const uint32_t excl = incl[i] - inc[i];
                const float before = grid_value(uu, dir > 0 ? A + excl : A - excl);
                float val = v[i];
                if (!(exact & (1u << i))) {
                    val = exactify(i);
                    v[i] = val;
                    exact |= 1u << i;
                }
                float after;
                bool stop;
                if (dir > 0) {
                    after = __fadd_rn(before, val);
                    stop = after >= thr;
                } else {
                    after = __fsub_rn(before, val);
                    stop = after <= 0.0f;
                }
                sh.fstate = after;
                sh.stop = stop ? (int)first : -1;
                sh.events++;
            }
        }
        csync();
        cur = sh.fstate;
        const int st = sh.stop;
        csync();
        if (st >= 0) {
            s = cur;
            return st;
        }
        consumed = (int)first;
    }
}

// Two-grid tile (see lrs_grid.h): values v in local-position order, positions
// [start, cnt); grid uu = the running value's grid at the tile start.  Used after a
// tile's single-grid fast path found an ordered step.  Values whose `exact` bit is clear
// are approximations within 8 float steps of the exact value; exactify(i) gives the
// exact value.  Same contract as acc_tile.
template <typename Exactify>
__device__ __noinline__ int tile2(float (&v)[kVpt], uint32_t& exact, int start, int cnt, int dir, float& s, float thr,
                     Exactify exactify, RowShared& sh) {
    const int uu = unit_exp(s);
    const int u1 = channel_uu(uu, dir, 1);
    uint32_t inc0[kVpt], inc1[kVpt];
    uint32_t sp0 = 0, sp1 = 0;
#pragma unroll 1
    for (int i = 0; i < kVpt; ++i) {
        const int li = li_of(i);
        inc0[i] = inc1[i] = 0;
        if (li < cnt && li >= start && v[i] != 0.0f) {  // an exact zero adds nothing anywhere
            if (!(exact & (1u << i))) {
                // both grids' increments must be the same for every value within the error bound
                const uint32_t vb = __float_as_uint(v[i]);
                const Cls2 lo = classify2(vb > 8u ? vb - 8u : 0u, uu, dir);
                const Cls2 hi = classify2(vb + 8u, uu, dir);
                const bool ok0 = (lo.inc0 == hi.inc0 && !lo.spec0 && !hi.spec0) || (lo.inc0 == kTwo23 && hi.inc0 == kTwo23);
                const bool ok1 = (lo.inc1 == hi.inc1 && !lo.spec1 && !hi.spec1) || (lo.inc1 == kTwo23 && hi.inc1 == kTwo23);
                if (!ok0 || !ok1) {
                    v[i] = exactify(i);
                    exact |= 1u << i;
                }
            }
            const Cls2 c = classify2(__float_as_uint(v[i]), uu, dir);
            inc0[i] = c.inc0;
            inc1[i] = c.inc1;
            if (c.spec0) sp0 |= 1u << i;
            if (c.spec1) sp1 |= 1u << i;
        }
    }
    uint32_t incl0[kVpt], incl1[kVpt];
    const uint32_t tot0 = block_incl_scan(inc0, incl0, sh.red);
    const uint32_t tot1 = block_incl_scan(inc1, incl1, sh.red);
    int consumed = start - 1;
    float cur = s;
    uint32_t base0 = 0, base1 = 0;
    for (;;) {
        const int ucur = unit_exp(cur);
        const int ch = ucur == uu ? 0 : (ucur == u1 ? 1 : -1);
        if (ch < 0) {  // a second grid change inside the tile
            s = cur;
            return acc_tile(v, exact, cnt, dir, s, thr, exactify, sh, consumed + 1);
        }
        const uint32_t A = grid_count(cur, ucur);
        const uint32_t lower = grid_lower(ucur);
        const float tq = (dir > 0 && thr < __int_as_float(0x7F800000)) ? ldexpf(thr, -ucur) : __int_as_float(0x7F800000);
        const uint32_t base = ch ? base1 : base0;
        const uint32_t spm = ch ? sp1 : sp0;
        uint32_t cand = 0xFFFFFFFFu;
#pragma unroll 1
        for (int i = 0; i < kVpt; ++i) {
            const int li = li_of(i);
            if (li < cnt && li > consumed && (uint32_t)li < cand) {
                const uint32_t incl = ch ? incl1[i] : incl0[i];
                if (needs_step(dir, (spm >> i) & 1u, A, incl - base, lower, tq)) cand = (uint32_t)li;
            }
        }
        const uint32_t first = block_reduce_u32(cand, MinU(), sh.red2);
        if (first == 0xFFFFFFFFu) {
            const uint32_t t = (ch ? tot1 : tot0) - base;
            s = grid_value(ucur, dir > 0 ? A + t : A - t);
            return -1;
        }
#pragma unroll 1
        for (int i = 0; i < kVpt; ++i) {
            if ((uint32_t)li_of(i) == first) {
                const uint32_t incl = ch ? incl1[i] : incl0[i];
                const uint32_t inc = ch ? inc1[i] : inc0[i];
                const uint32_t excl = incl - inc - base;
                const float before = grid_value(ucur, dir > 0 ? A + excl : A - excl);
                float val = v[i];
                if (!(exact & (1u << i))) {
                    // the operation's result must not depend on where in the error bound v lies
                    const uint32_t vb = __float_as_uint(val);
                    const float lo = __uint_as_float(vb > 8u ? vb - 8u : 0u), hi = __uint_as_float(vb + 8u);
                    const float rlo = dir > 0 ? __fadd_rn(before, lo) : __fsub_rn(before, lo);
                    const float rhi = dir > 0 ? __fadd_rn(before, hi) : __fsub_rn(before, hi);
                    if (rlo != rhi) {
                        val = exactify(i);
                        v[i] = val;
                        exact |= 1u << i;
                    }
                }
                const float after = dir > 0 ? __fadd_rn(before, val) : __fsub_rn(before, val);
                const bool stop = dir > 0 ? after >= thr : after <= 0.0f;
                sh.fstate = after;
                sh.stop = stop ? (int)first : -1;
                sh.ev_base0 = incl0[i];
                sh.ev_base1 = incl1[i];
                sh.events++;
            }
        }
        csync();
        cur = sh.fstate;
        const int st = sh.stop;
        base0 = sh.ev_base0;
        base1 = sh.ev_base1;
        if (st >= 0) {
            s = cur;
            return st;
        }
        consumed = (int)first;
    }
}

// Exact sequential run over exact values by the calling thread alone (a short list, or
// the start of the softmax sum where the running value crosses many binades).
// Returns the stop position or -1 (sampler.rs:137-139, 148-151, 156-158).
__device__ __forceinline__ int serial_run(const float* vals, int cnt, int dir, float& s, float thr) {
    float cur = s;
    // eight values loaded at a time (the loads do not wait for the sum)
    for (int i0 = 0; i0 < cnt; i0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = i0 + j < cnt ? vals[i0 + j] : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (i0 + j >= cnt) break;
            cur = dir > 0 ? __fadd_rn(cur, v[j]) : __fsub_rn(cur, v[j]);
            if (dir > 0 ? cur >= thr : cur <= 0.0f) {
                s = cur;
                return i0 + j;
            }
        }
    }
    s = cur;
    return -1;
}

// All-ascending bitonic sort of n 64-bit keys (n <= cap, cap a power of two >= n is
// not required: virtual +inf padding).  `keys` in shared or global memory.
__device__ __noinline__ void bitonic_sort_u64(unsigned long long* keys, uint32_t n) {
    if (n < 2) return;
    uint32_t P = 1;
    while (P < n) P <<= 1;
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t t = threadIdx.x; t < P / 2; t += kThreads) {
                const uint32_t grp = t / stride, off = t % stride;
                uint32_t i, j;
                if (stride == (size >> 1)) {
                    // first step of a merge: compare with the mirrored partner
                    const uint32_t base = (t / stride) * size;
                    i = base + off;
                    j = base + size - 1 - off;
                } else {
                    i = grp * stride * 2 + off;
                    j = i + stride;
                }
                if (j < n) {
                    const unsigned long long a = keys[i], b = keys[j];
                    if (a > b) {
                        keys[i] = b;
                        keys[j] = a;
                    }
                }
            }
            csync();
        }
    }
}

// One warp: the digit d of a radix round (256 counts, digit 255 first) holding the kk-th
// largest key, and kk's rank inside that digit.  Lane l scans digits 255-8l .. 248-8l.
__device__ __forceinline__ void digit_from_top(const uint32_t* hist, uint32_t kk, uint32_t& d, uint32_t& rem) {
    const int lane = threadIdx.x & 31;
    uint32_t c[8], s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        c[e] = hist[255 - 8 * lane - e];
        s += c[e];
    }
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += t;
    }
    const uint32_t excl = incl - s;
    const bool mine = excl < kk && kk <= incl;
    const unsigned own = __ballot_sync(0xFFFFFFFFu, mine);
    uint32_t dd = 0, rr = 0;
    if (mine) {
        uint32_t acc = excl;
        bool found = false;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (!found && acc + c[e] >= kk) {
                dd = (uint32_t)(255 - 8 * lane - e);
                rr = kk - acc;
                found = true;
            }
            acc += c[e];
        }
    }
    const int owner = own ? __ffs(own) - 1 : 0;
    d = __shfl_sync(0xFFFFFFFFu, dd, owner);
    rem = __shfl_sync(0xFFFFFFFFu, rr, owner);
}

// k-th largest key (1-based rank kk) among keys[0..cnt) by radix select.
__device__ __noinline__ uint32_t radix_select_desc(const float* x, uint32_t cnt, uint32_t kk, RowShared& sh) {
    uint32_t prefix = 0;
    for (int round = 0; round < 4; ++round) {
        const int shift = 24 - 8 * round;
        for (int i = threadIdx.x; i < 256; i += kThreads) sh.hist256[i] = 0;
        csync();
        for (uint32_t i0 = 0; i0 < cnt; i0 += kThreads) {
            const uint32_t i = i0 + threadIdx.x;
            uint32_t key = 0;
            bool match = false;
            if (i < cnt) {
                key = fkey(x[i]);
                match = (round == 0) || ((key >> (shift + 8)) == (prefix >> (shift + 8)));
            }
            // warp-aggregated increments: candidates share high key bits
            const unsigned act = __ballot_sync(0xFFFFFFFFu, match);
            if (match) {
                const uint32_t bin = (key >> shift) & 255u;
                const unsigned peers = __match_any_sync(act, bin);
                if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&sh.hist256[bin], (uint32_t)__popc(peers));
            }
        }
        csync();
        if (threadIdx.x < 32) {
            uint32_t d, rem;
            digit_from_top(sh.hist256, kk, d, rem);
            if (threadIdx.x == 0) {
                sh.misc[1] = d;
                sh.misc[2] = rem;
            }
        }
        csync();
        prefix |= sh.misc[1] << shift;
        kk = sh.misc[2];
        csync();
    }
    return prefix;
}

// Margin below the k-th value inside which probabilities may tie: distinct scaled
// logits closer than this can round to the same probability (it is generous by more
// than a factor of 4 over the rounding steps of d = x - max, exp and p = e * inv).
__device__ __forceinline__ float tie_margin(float vk, float m) {
    return ldexpf(fabsf(vk) + fabsf(m) + 1.0f, -18);
}

// Compact the path-K candidate buffer to the elements >= (k-th largest - margin).
__device__ __noinline__ void compact_candidates(float* cx, uint32_t* ci, uint32_t k, float mrun, RowShared& sh) {
    const uint32_t cnt = min(sh.cand_n, (uint32_t)kKCap);
    if (cnt <= k) return;
    const uint32_t key = radix_select_desc(cx, cnt, k, sh);
    const float vk = fkey_inv(key);
    const float delta = tie_margin(vk, mrun);
    const float th = vk - delta;
    // read my entries, then write back compacted
    constexpr int per = (kKCap + kThreads - 1) / kThreads;
    float xv[per];
    uint32_t iv[per];
    int have = 0;
    for (int q = 0; q < per; ++q) {
        const uint32_t i = threadIdx.x + q * kThreads;
        if (i < cnt && cx[i] >= th) {
            xv[have] = cx[i];
            iv[have] = ci[i];
            ++have;
        }
    }
    csync();
    if (threadIdx.x == 0) sh.cand_n = 0;
    csync();
    uint32_t base = atomicAdd(&sh.cand_n, (uint32_t)have);
    for (int q = 0; q < have; ++q) {
        cx[base + q] = xv[q];
        ci[base + q] = iv[q];
    }
    if (threadIdx.x == 0) {
        if (th > sh.theta) sh.theta = th;
        if (delta < sh.delta_min) sh.delta_min = delta;
        sh.vk = vk;
    }
    csync();
}


// Loads a tile of up to kChunk sorted 64-bit keys (p desc, index asc) as probabilities.
__device__ __forceinline__ void load_sorted_tile(const unsigned long long* keys, uint32_t cnt, float (&v)[kVpt]) {
#pragma unroll
    for (int i = 0; i < kVpt; ++i) {
        const int li = li_of(i);
        v[i] = (uint32_t)li < cnt ? __uint_as_float(~(uint32_t)(keys[li] >> 32)) : 0.0f;
    }
}

struct NoExact {  // sorted probability tiles are exact already
    __device__ float operator()(int) const { return 0.0f; }
};

// The scaled, shifted logit d = fl(fl(x * inv_t) - max) of sampler.rs:117 / ops.rs:409.
__device__ __forceinline__ float d_of(float x, float inv_t, float mx) { return __fsub_rn(__fmul_rn(x, inv_t), mx); }

// 2^e for -149 <= e <= 127, from its bits (normal or subnormal).
__device__ __forceinline__ float pow2f(int e) {
    return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(1u << (e + 149));
}
// x * 2^e exactly, for x a multiple of 2^-e below 2^25 2^-e (a grid count): the integer
// count, by two power-of-two products where 2^e alone is not a float.
__device__ __forceinline__ uint32_t grid_units(float x, int e) {
    return e > 127 ? (uint32_t)__fmul_rn(__fmul_rn(x, pow2f(127)), pow2f(e - 127)) : (uint32_t)__fmul_rn(x, pow2f(e));
}

// Largest (penalised) raw logit x with d_of(x) < thr, by bisection over the float order
// (d_of is non-decreasing in x since inv_t >= 0).  -inf if there is none.
__device__ __noinline__ float raw_threshold(float thr, float inv_t, float mx) {
    uint32_t lo = fkey(__int_as_float(0xFF800000)), hi = fkey(__int_as_float(0x7F800000));
    if (!(d_of(fkey_inv(lo), inv_t, mx) < thr)) return __int_as_float(0xFF800000);
    if (d_of(fkey_inv(hi), inv_t, mx) < thr) return fkey_inv(hi);
    while (hi - lo > 1) {  // invariant: d(lo) < thr <= d(hi)
        const uint32_t mid = lo + (hi - lo) / 2;
        if (d_of(fkey_inv(mid), inv_t, mx) < thr) lo = mid; else hi = mid;
    }
    return fkey_inv(lo);
}


// ------------------------------------------------------------- warp helpers ----
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float warp_max_nan(float m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    return m;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float warp_incl_scan_f(float v) {
    const int l = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (l >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ uint32_t warp_incl_scan_plain(uint32_t v) {
    const int l = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (l >= o) v += t;
    }
    return v;
}

// Register slot i of a lane's run holds run offset run_pos(i): float4 number j = i / 4
// is read from offset 4 * ((j + lane) & 7), so the eight lanes of a shared-memory
// phase read eight different bank groups.
__device__ __forceinline__ uint32_t run_pos(int i, int lane) {
    return (uint32_t)((((i >> 2) + lane) & 7) * 4 + (i & 3));
}

// The lane's run of a tile (offsets [32 * lane, 32 * lane + 32)), -inf past nval.
__device__ __forceinline__ void load_run(const float* slot, int lane, uint32_t nval, float (&v)[32]) {
    const float ninf = __int_as_float(0xFF800000);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
        float4 q = make_float4(ninf, ninf, ninf, ninf);
        if (c4 < nval) q = *reinterpret_cast<const float4*>(slot + lane * 32 + c4);
        v[4 * j + 0] = q.x;
        v[4 * j + 1] = q.y;
        v[4 * j + 2] = q.z;
        v[4 * j + 3] = q.w;
    }
}

// Penalty bits of ids [gi0, gi0 + 32) from the row's window bitmap (global, read at L2
// so that the bits set by this CTA's atomics are seen).
__device__ __forceinline__ uint32_t lane_bits(const uint32_t* bm, uint32_t gi0) {
    const uint32_t w = gi0 >> 5, s = gi0 & 31u;
    const uint32_t lo = __ldcg(bm + w);
    if (!s) return lo;
    const uint32_t hi = __ldcg(bm + w + 1);
    return (lo >> s) | (hi << (32u - s));
}

// x > 0 ? x / p : x * p (sampler.rs:96-100).
__device__ __noinline__ float penalise(float x, float p) { return x > 0.0f ? __fdiv_rn(x, p) : __fmul_rn(x, p); }

// Applies the penalty to the register slots whose run offsets have their bit set
// (rare: a window of W ids touches at most W runs of a row).
__device__ __forceinline__ void apply_penalty(float (&v)[32], uint32_t bits, int lane, float pen) {
    while (bits) {
        const int pos = __ffs(bits) - 1;
        bits &= bits - 1u;
        const int slot = ((((pos >> 2) - lane) & 7) << 2) | (pos & 3);
        float x = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i == slot) x = v[i];
        x = penalise(x, pen);
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i == slot) v[i] = x;
    }
}

// Adds, one after the other, the exponentials held by lanes [lo, lo + cnt) to s; every
// lane returns the same sum (ops.rs:408-411).  e is CUDA's expf(d) unless `exact`:
// libm's value (exact_expf(d)) is computed by every such lane at once, before the
// ordered additions, so one table latency is paid per call, not one per element.
__device__ __noinline__ float warp_serial_add(float s, float e, float d, bool exact, int lo, int cnt,
                                              const ExpTable tab) {
    const int lane = threadIdx.x & 31;
    // libm's value only where CUDA's (within 2 ulp) could round differently: s only
    // grows, so its grid at the start (unit 2^uu) is the finest of the run, and every
    // rounding boundary of s + e, on that grid or a coarser one, lies at a multiple of
    // half the unit; a value more than 2^-21 e from all of them adds what libm's adds.
    if (!exact && lane >= lo && lane < lo + cnt) {
        const int uu = unit_exp(s);
        bool amb = true;
        if (uu > -149) {
            const float x = ldexpf(e, 1 - uu);  // e / (half unit), exact below 2^22
            amb = !(x < 4194304.0f) || fabsf(__fsub_rn(x, rintf(x))) <= __fmul_rn(x, 4.76837158203125e-07f);
        }
        if (amb) e = exact_expf(d, tab);
    }
    // (unrolled over all 32 lanes: the shuffles do not wait for the sum, only the adds
    // form the serial chain)
    const int hi = lo + cnt;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float v = __shfl_sync(0xFFFFFFFFu, e, j);
        if (j >= lo && j < hi) s = __fadd_rn(s, v);
    }
    return s;
}

// kk-th largest (1-based) of x[0..cnt) in shared memory, by one warp: radix select on
// the order-preserving key, 8 bits a round.  hist: 256 words owned by the warp.
__device__ __noinline__ float warp_kth_desc(const float* x, uint32_t cnt, uint32_t kk, uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0;
    for (int round = 0; round < 4; ++round) {
        const int shift = 24 - 8 * round;
        for (int b = lane; b < 256; b += 32) hist[b] = 0;
        __syncwarp();
        for (uint32_t i = lane; i < cnt; i += 32) {
            const uint32_t key = fkey(x[i]);
            if (round == 0 || (key >> (shift + 8)) == (prefix >> (shift + 8)))
                atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncwarp();
        uint32_t d, rem;
        digit_from_top(hist, kk, d, rem);
        prefix |= d << shift;
        kk = rem;
        __syncwarp();
    }
    return fkey_inv(prefix);
}

// Path-K state of one warp's streaming filter.
struct WState {
    uint32_t wcnt;  // candidates buffered
    float theta;    // append threshold
    float wdelta;   // smallest compaction margin so far
    uint32_t over;  // ties overflowed the buffer (path N takes the row)
};

// Raise the warp's threshold to (k-th largest buffered - tie margin) and drop the
// buffered entries below it (the warp-scope form of compact_candidates).
__device__ __noinline__ WState warp_compact(float* wx, uint32_t* wi, WState s, uint32_t k, float mrun,
                                            uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    __syncwarp();
    if (s.wcnt <= k) return s;
    const float vk = warp_kth_desc(wx, s.wcnt, k, hist);
    const float delta = tie_margin(vk, mrun);
    const float th = vk - delta;
    s.wdelta = fminf(s.wdelta, delta);
    if (th > s.theta) s.theta = th;
    uint32_t out = 0;
    for (uint32_t b = 0; b < s.wcnt; b += 32) {
        const uint32_t i = b + (uint32_t)lane;
        const bool keep = i < s.wcnt && wx[i] >= th;
        const float xv = keep ? wx[i] : 0.0f;
        const uint32_t iv = keep ? wi[i] : 0u;
        const unsigned m = __ballot_sync(0xFFFFFFFFu, keep);
        __syncwarp();
        if (keep) {
            const uint32_t p = out + (uint32_t)__popc(m & ((1u << lane) - 1u));
            wx[p] = xv;
            wi[p] = iv;
        }
        out += (uint32_t)__popc(m);
        __syncwarp();
    }
    s.wcnt = out;
    return s;
}

// Increments of elements on the two grids a run is classified for (units 2^u0 and
// 2^(u0+1)): e = libm's expf(d) where CUDA's expf (within 2 ulp) could round
// differently; a tie or an element of half a binade or more flags the grid.
struct GridAcc {
    float s0, s1;  // sums of the rounded increments (multiples of the units)
    bool sp0, sp1;
};
__device__ __forceinline__ void classify_elem(float d, float bm0, float bm1, float h0, float h1, GridAcc& g,
                                              const ExpTable tab) {
    bool ex = d == 0.0f;
    float e = ex ? 1.0f : expf(d);
    float i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);  // RN(e / U) U below bm
    float i1 = __fsub_rn(__fadd_rn(bm1, e), bm1);
    if (!ex) {
        const float tol = __fmul_rn(e, 4.76837158203125e-07f);  // 2^-21 e > 2 ulp
        const bool amb = e < 7.8886091e-31f || fabsf(__fsub_rn(e, bm0)) <= tol || fabsf(__fsub_rn(e, bm1)) <= tol ||
                         (e < bm0 && fabsf(__fsub_rn(e, i0)) >= __fsub_rn(h0, tol)) ||
                         (e < bm1 && fabsf(__fsub_rn(e, i1)) >= __fsub_rn(h1, tol));
        if (amb) {
            e = exact_expf(d, tab);
            ex = true;
            i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);
            i1 = __fsub_rn(__fadd_rn(bm1, e), bm1);
        }
    }
    if (e >= bm0) {
        g.sp0 = true;
    } else {
        g.s0 += i0;
        if (ex && h0 > 0.0f && fabsf(__fsub_rn(e, i0)) == h0) g.sp0 = true;
    }
    if (e >= bm1) {
        g.sp1 = true;
    } else {
        g.s1 += i1;
        if (ex && fabsf(__fsub_rn(e, i1)) == h1) g.sp1 = true;
    }
}

// The same on grid u0 alone (runs whose running sum cannot leave u0's binade by the
// estimate; the caller flags grid u0 + 1, so a run that lands there is summed element
// by element).
__device__ __forceinline__ void classify_elem1(float d, float bm0, float h0, GridAcc& g, const ExpTable tab) {
    bool ex = d == 0.0f;
    float e = ex ? 1.0f : expf(d);
    float i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);
    if (!ex) {
        const float tol = __fmul_rn(e, 4.76837158203125e-07f);  // 2^-21 e > 2 ulp
        const bool amb = e < 7.8886091e-31f || fabsf(__fsub_rn(e, bm0)) <= tol ||
                         (e < bm0 && fabsf(__fsub_rn(e, i0)) >= __fsub_rn(h0, tol));
        if (amb) {
            e = exact_expf(d, tab);
            ex = true;
            i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);
        }
    }
    if (e >= bm0) {
        g.sp0 = true;
    } else {
        g.s0 += i0;
        if (ex && h0 > 0.0f && fabsf(__fsub_rn(e, i0)) == h0) g.sp0 = true;
    }
}

// Two elements at once on grid u0 alone (b absent: !vb), straight-line up to the rare
// libm lookups so that the two dependency chains overlap.
__device__ __forceinline__ void classify_pair1(float da, float db, bool vb, float bm0, float h0, GridAcc& g,
                                               const ExpTable tab) {
    bool exa = da == 0.0f, exb = db == 0.0f;
    float ea = exa ? 1.0f : expf(da);
    float eb = exb ? 1.0f : expf(db);
    float ia = __fsub_rn(__fadd_rn(bm0, ea), bm0);
    float ib = __fsub_rn(__fadd_rn(bm0, eb), bm0);
    const float ta = __fmul_rn(ea, 4.76837158203125e-07f), tb = __fmul_rn(eb, 4.76837158203125e-07f);
    const bool amba = !exa && (ea < 7.8886091e-31f || fabsf(__fsub_rn(ea, bm0)) <= ta ||
                               (ea < bm0 && fabsf(__fsub_rn(ea, ia)) >= __fsub_rn(h0, ta)));
    const bool ambb = vb && !exb && (eb < 7.8886091e-31f || fabsf(__fsub_rn(eb, bm0)) <= tb ||
                                     (eb < bm0 && fabsf(__fsub_rn(eb, ib)) >= __fsub_rn(h0, tb)));
    if (amba || ambb) {
        if (amba) {
            ea = exact_expf(da, tab);
            exa = true;
            ia = __fsub_rn(__fadd_rn(bm0, ea), bm0);
        }
        if (ambb) {
            eb = exact_expf(db, tab);
            exb = true;
            ib = __fsub_rn(__fadd_rn(bm0, eb), bm0);
        }
    }
    if (ea >= bm0) {
        g.sp0 = true;
    } else {
        g.s0 += ia;
        if (exa && h0 > 0.0f && fabsf(__fsub_rn(ea, ia)) == h0) g.sp0 = true;
    }
    if (vb) {
        if (eb >= bm0) {
            g.sp0 = true;
        } else {
            g.s0 += ib;
            if (exb && h0 > 0.0f && fabsf(__fsub_rn(eb, ib)) == h0) g.sp0 = true;
        }
    }
}

// Path K, one tile: appends this lane's hits (run offsets in hmask, values re-read from
// the staged run) to the warp buffer in index order, 4 per lane at a time, compacting
// the buffer when a batch would not fit.  mrun: the max of everything seen so far.
__device__ __noinline__ WState topk_tile(const float* run, uint32_t hmask, uint32_t bits, float penalty, float inv_t,
                                        uint32_t gbase, float mrun, uint32_t k, float* wx, uint32_t* wi,
                                        uint32_t* wh, WState ws) {
    const int lane = threadIdx.x & 31;
    // hits in a lane-rotated order: lane L starts at run offset L, so that the lanes'
    // reads (run = lane * 32 + offset) fall in different shared-memory banks
    hmask = __funnelshift_r(hmask, hmask, lane);
    if (ws.wcnt == 0u && ws.theta == -__int_as_float(0x7F800000)) {
        // First tile of the warp: every element is a hit.  The k-th largest of the
        // lanes' four largest values (k <= 128 distinct elements of the tile at or
        // above it) bounds the tile's k-th largest from below; less the tie margin it
        // is the starting threshold, and the hits below it are dropped before any
        // append.  The k-th largest: a radix select over order-preserving keys.
        float top[4] = {-__int_as_float(0x7F800000), -__int_as_float(0x7F800000), -__int_as_float(0x7F800000),
                        -__int_as_float(0x7F800000)};
        for (uint32_t h = hmask; h; h &= h - 1u) {
            const int pos = (__ffs(h) - 1 + lane) & 31;
            float x = run[pos];
            if ((bits >> pos) & 1u) x = penalise(x, penalty);
            float v = __fmul_rn(x, inv_t);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float hi = fmaxf(top[j], v);
                v = fminf(top[j], v);
                top[j] = hi;
            }
        }
        uint32_t key[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t u = __float_as_uint(top[j]);
            key[j] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        }
        uint32_t res = 0;
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t cand = res | (1u << bit);
            uint32_t c = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) c += (uint32_t)__popc(__ballot_sync(0xFFFFFFFFu, key[j] >= cand));
            if (c >= k) res = cand;
        }
        const float kth = __uint_as_float((res & 0x80000000u) ? (res & 0x7FFFFFFFu) : ~res);
        if (kth > -__int_as_float(0x7F800000)) {
            const float delta = tie_margin(kth, mrun);
            const float th = kth - delta;
            if (th > ws.theta) ws.theta = th;
            ws.wdelta = fminf(ws.wdelta, delta);
            uint32_t keep = 0;
            for (uint32_t h = hmask; h; h &= h - 1u) {
                const int bit = __ffs(h) - 1;
                const int pos = (bit + lane) & 31;
                float x = run[pos];
                if ((bits >> pos) & 1u) x = penalise(x, penalty);
                if (__fmul_rn(x, inv_t) >= ws.theta) keep |= 1u << bit;
            }
            hmask = keep;
        }
    }
    while (__any_sync(0xFFFFFFFFu, hmask != 0u)) {
        float xv[4];
        uint32_t gv[4], hm = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            xv[c] = 0.0f;
            gv[c] = 0u;
            if (hmask) {
                const int pos = (__ffs(hmask) - 1 + lane) & 31;
                hmask &= hmask - 1u;
                float x = run[pos];
                if ((bits >> pos) & 1u) x = penalise(x, penalty);
                xv[c] = __fmul_rn(x, inv_t);
                gv[c] = gbase + (uint32_t)pos;
                if (xv[c] >= ws.theta) hm |= 1u << c;
            }
        }
        uint32_t nh = (uint32_t)__popc(hm);
        uint32_t incl = warp_incl_scan_plain(nh);
        uint32_t tot = __shfl_sync(0xFFFFFFFFu, incl, 31);
        if (ws.wcnt + tot > (uint32_t)kWCap) {
            ws = warp_compact(wx, wi, ws, k, mrun, wh);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (!(xv[c] >= ws.theta)) hm &= ~(1u << c);
            nh = (uint32_t)__popc(hm);
            incl = warp_incl_scan_plain(nh);
            tot = __shfl_sync(0xFFFFFFFFu, incl, 31);
            if (ws.wcnt + tot > (uint32_t)kWCap) {  // ties fill the buffer
                ws.over = 1u;
                return ws;
            }
        }
        uint32_t p = ws.wcnt + incl - nh;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if ((hm >> c) & 1u) {
                wx[p] = xv[c];
                wi[p] = gv[c];
                ++p;
            }
        ws.wcnt += tot;
        // hits after a compaction must clear the raised threshold: re-tested next batch
    }
    return ws;
}

// ------------------------------------------------------------ finish phases ----
// Row context of the top-k / top-p / draw phase (sampler.rs:122-162).
struct FinishCtx {
    Geo g;
    const TileRec* tt;              // tile records
    const uint2* lists;             // candidate lists of the sparse tiles: (scaled logit, index)
    const float* lmax;              // per tile t and lane: lmax[64 t + lane], the max of the run's scaled logits
    unsigned long long* scratch;    // path N: gathered (p, index) keys
    const uint32_t* bitmap;         // window bitmap
    uint32_t* hcnt;                 // path N: bucket counts and offsets
    uint32_t* hoff;
    uint32_t* cursor;
    unsigned long long* sbuf;       // path N: bucket sort buffer (aliases cursor)
    float* ring;                    // path N: the (idle) ring, staging area of the gather
    int32_t* err;                   // sticky error word (bounded waits)
    float* cand_x;                  // path K: candidates and sort keys
    uint32_t* cand_i;
    unsigned long long* keys;
    ExpTable exptab;
    uint32_t k, nk;
    float mx, inv_t, inv, S, penalty, top_p, hist_lim;
    bool pen_on, topp_on;
    unsigned long long st;          // PRNG state (advanced by the draw)
    uint32_t cutoff, pos, n_cand;   // results
    float sum, rr, r0;
    unsigned long long chosen;
    long long acc_sort;
};

// Path K: sort the candidates, then top-p, survivor sum and draw on thread 0.
__device__ __noinline__ void finish_path_k(RowShared& sh, FinishCtx& f) {
    const int tid = threadIdx.x;
    const float kInf = __int_as_float(0x7F800000);
    // (the context's fields in registers: loads through `f` go to local memory)
    const uint32_t nk = f.nk;
    const float* const cand_x = f.cand_x;
    const uint32_t* const cand_i = f.cand_i;
    unsigned long long* const keys = f.keys;
    const float mx = f.mx, inv = f.inv;
    const ExpTable exptab = f.exptab;
    for (uint32_t i = tid; i < nk; i += kThreads) {
        const float e = exact_expf(__fsub_rn(cand_x[i], mx), exptab);
        const float p = __fmul_rn(e, inv);
        keys[i] = ((unsigned long long)(~__float_as_uint(p)) << 32) | cand_i[i];
    }
    csync();
    const long long ts = clock64();
    bitonic_sort_u64(keys, nk);  // (p desc, index asc)
    f.acc_sort += clock64() - ts;
    f.n_cand = f.nk;
    for (uint32_t i = tid; i < f.k; i += kThreads) sh.ser[i] = __uint_as_float(~(uint32_t)(f.keys[i] >> 32));
    csync();
    if (tid == 0) {
        // top-p over the first k (sampler.rs:135-146); the survivor sum is the
        // same sequence up to the cutoff (sampler.rs:148-151)
        float cum = 0.0f;
        const int stp = serial_run(sh.ser, (int)f.k, +1, cum, f.topp_on ? f.top_p : kInf);
        const uint32_t cut = stp >= 0 ? (uint32_t)stp + 1 : f.k;
        uint32_t ps = 0;
        float r0 = 0.0f;
        unsigned long long st2 = f.st;
        if (cum > 0.0f) {
            r0 = __fmul_rn(next_f32(&st2), cum);  // sampler.rs:155
            float rv = r0;
            const int w = serial_run(sh.ser, (int)cut, -1, rv, 0.0f);
            ps = w >= 0 ? (uint32_t)w : cut - 1;  // sampler.rs:156-162
        }
        sh.misc[3] = cut;
        sh.misc[4] = ps;
        sh.fstate = cum;
        sh.vk = r0;
    }
    csync();
    f.cutoff = sh.misc[3];
    f.pos = sh.misc[4];
    f.sum = sh.fstate;
    f.rr = sh.vk;
    if (f.sum > 0.0f) {
        (void)next_f32(&f.st);
        f.r0 = f.rr;
    }
    f.chosen = f.keys[f.pos];
    csync();
}

// Path N: gather bucket by bucket, sort lazily, scan with the exact emulation.
__device__ __noinline__ void finish_path_n(RowShared& sh, FinishCtx& f) {
    // The read-only context in registers: loads through `f` go to local memory (the
    // context lives in the kernel's stack frame), which the shared-memory carve-out
    // leaves little L1 for.
    const Geo g = f.g;
    const TileRec* const tt = f.tt;
    const uint2* const lists = f.lists;
    const float* const lmax = f.lmax;
    unsigned long long* const scratch = f.scratch;
    const uint32_t* const bitmap = f.bitmap;
    uint32_t* const hcnt = f.hcnt;
    uint32_t* const hoff = f.hoff;
    uint32_t* const cursor = f.cursor;
    unsigned long long* const sbuf = f.sbuf;
    float* const ring = f.ring;
    int32_t* const err = f.err;
    const ExpTable exptab = f.exptab;
    const uint32_t k = f.k;
    const float mx = f.mx, inv_t = f.inv_t, inv = f.inv, S = f.S, penalty = f.penalty, top_p = f.top_p;
    const float hist_lim = f.hist_lim;
    const bool pen_on = f.pen_on, topp_on = f.topp_on;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const float kInf = __int_as_float(0x7F800000);
    auto penal_g = [&](float x, uint32_t gi) -> float {  // sampler.rs:96-100
        if (pen_on && ((__ldcg(bitmap + (gi >> 5)) >> (gi & 31)) & 1u)) return penalise(x, penalty);
        return x;
    };
    if (warp == 0) {
        // Bucket limit: the first bucket through which the gathered candidates are
        // expected to hold the top-k / top-p survivors (the scan gathers more buckets
        // when it needs them, so this limit only sizes the first gather).  The mass of
        // bucket b lies in [count exp(-(b+1)/kBScale), count exp(-b/kBScale)].  Stop at
        // k candidates, at a lower bound of the head mass of (top_p + margin) S, or
        // where an upper bound of the mass after the bucket (the elements below the
        // histogram range included, each below exp(-18)) is at most (1 - top_p -
        // margin) S.  Past the first bucket whose probabilities are all below 2^-26 the
        // scan ends (once the top-p sum is at least 1/2 nothing after it changes the
        // sum).  One warp, 32 buckets a step.
        const double target = topp_on ? ((double)top_p + kTopPMargin) * (double)S : 1e300;
        const double tail_target = topp_on ? (1.0 - (double)top_p - kTailMargin) * (double)S : -1.0;
        const double exit_e = 1.4901161193847656e-08 * (double)S;
        const double elane = exp(-(double)(lane + 1) / (double)kBScale) * (1.0 - 1e-12);  // (low: a lower bound)
        const double ewidth = exp(1.0 / (double)kBScale) * (1.0 + 1e-9);  // upper / lower bound of a bucket
        const double estep = __shfl_sync(0xFFFFFFFFu, elane, 31);        // exp(-32/kBScale)
        // upper bound of the whole mass (first sweep)
        double utot = 0.0;
        uint32_t ctot = 0;
        {
            double e32 = 1.0;
            for (uint32_t base = 0; base < (uint32_t)kNB - 1; base += 32) {
                const uint32_t b = base + (uint32_t)lane;
                const uint32_t c = b < (uint32_t)kNB - 1 ? hcnt[b] : 0u;
                utot += (double)c * e32 * elane * ewidth;
                ctot += c;
                e32 *= estep;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                utot += __shfl_xor_sync(0xFFFFFFFFu, utot, o);
                ctot += __shfl_xor_sync(0xFFFFFFFFu, ctot, o);
            }
            utot += (double)(g.n - ctot) * 1.5229979744712629e-08;  // exp(-18)
        }
        double e32 = 1.0;  // exp(-32 k / kBScale) at the start of each 32-bucket step
        uint32_t cc = 0, acc = 0, found = (uint32_t)kNB - 1;
        double mass = 0.0, umass = 0.0;
        for (uint32_t base = 0; base < (uint32_t)kNB - 1; base += 32) {
            const uint32_t b = base + (uint32_t)lane;
            const bool in = b < (uint32_t)kNB - 1;
            const uint32_t c = in ? hcnt[b] : 0u;
            const double eb = e32 * elane;
            // inclusive prefixes of counts and masses over the lanes
            uint32_t ci = c;
            double mi = (double)c * eb;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t tc = __shfl_up_sync(0xFFFFFFFFu, ci, o);
                const double tm = __shfl_up_sync(0xFFFFFFFFu, mi, o);
                if (lane >= o) {
                    ci += tc;
                    mi += tm;
                }
            }
            if (in) hoff[b] = acc + ci - c;
            const bool tail_ok = tail_target > 0.0 && utot - (umass + mi * ewidth) <= tail_target;
            const bool stop = in && (cc + ci >= k || mass + mi >= target || tail_ok || eb < exit_e);
            const unsigned m = __ballot_sync(0xFFFFFFFFu, stop);
            if (m && found == (uint32_t)kNB - 1) found = base + (uint32_t)(__ffs(m) - 1);
            cc += __shfl_sync(0xFFFFFFFFu, ci, 31);
            acc += __shfl_sync(0xFFFFFFFFu, ci, 31);
            mass += __shfl_sync(0xFFFFFFFFu, mi, 31);
            umass += __shfl_sync(0xFFFFFFFFu, mi, 31) * ewidth;
            e32 *= estep;
        }
        if (lane == 0) {
            hoff[kNB - 1] = acc;
            hcnt[kNB - 1] = g.n - acc;  // everything below the histogram range
            sh.misc[3] = found;
        }
    }
    csync();
    const uint32_t blim = sh.misc[3];
    // gather exact probabilities of buckets [blo, bhi] into scratch; tiles whose
    // max lies below the range are skipped
    auto gather = [&](uint32_t blo, uint32_t bhi) {
        const bool all = bhi == (uint32_t)kNB - 1;
        uint32_t gph = sh.gph[warp];  // (the warp's staging barrier phase)
        bool gdead = false;           // a staging wait ran out after an abort: wait no more
        const float dlim = -(float)(bhi + 1) / kBScale;
        for (uint32_t q = blo + tid; q <= bhi; q += kThreads) cursor[q] = 0;
        csync();
        // d: the element's d = fl(fl(x * inv_t) - max) (ops.rs:409)
        auto take = [=](uint32_t i, float dd, bool valid) {
            bool tk = false;
            int b = 0;
            if (valid && (dd >= dlim || all)) {
                b = dd >= hist_lim ? (int)fminf(-dd * kBScale, (float)(kNB - 1)) : kNB - 1;
                tk = (uint32_t)b >= blo && (uint32_t)b <= bhi;
            }
            if (tk) {
                // CUDA's expf (within 2 ulp): keys are exactified before a bucket is ordered.
                // A bucket's storage order is free (it is sorted where the order matters).
                const float e = dd == 0.0f ? 1.0f : expf(dd);
                const float pr = __fmul_rn(e, inv);
                const uint32_t slot = hoff[b] + atomicAdd(&cursor[b], 1u);
                scratch[slot] = ((unsigned long long)(~__float_as_uint(pr)) << 32) | i | (dd == 0.0f ? 0u : kApxKey);
            }
        };
        if (warp == 0) {
            const uint32_t edges = g.head + g.tail;
            const bool mine = (uint32_t)lane < edges;
            const uint32_t gi =
                (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
            take(gi, mine ? d_of(penal_g(g.row[gi], gi), inv_t, mx) : 0.0f, mine);
        }
        // The warp's tiles t = warp + kWarps j, 32 at a time (j in lane bits).  Work items
        // of 32 elements, one per lane: a run of a dense tile whose pass-1 run max
        // reaches the range, or 32 list entries of a sparse tile.  The items are listed
        // in shared memory (after the bucket cursors): dense runs from the front, list
        // groups from the back (at most 1024 together).  List groups are read eight at
        // a time with their loads in flight together; dense runs are brought into the
        // warp's part of the ring by bulk copies, kGatherRuns at a time (the ring is
        // idle: the producer streams nothing until this row is done).
        uint32_t* items = reinterpret_cast<uint32_t*>(sbuf) + kGatherItemsOff + (uint32_t)warp * 1024u;
        float* const stage = ring + (size_t)warp * kGatherRuns * 32u;
        uint64_t* const gbar = &sh.gbar[warp];
        const uint64_t pol = policy_evict_first();
        const uint32_t ntw = g.nchunks > (uint32_t)warp ? (g.nchunks - (uint32_t)warp + kWarps - 1) / kWarps : 0u;
        for (uint32_t j0 = 0; j0 < ntw; j0 += 32) {
            const uint32_t nj = min(32u, ntw - j0);
            uint32_t live = 0;  // lane bit j: the lane's run of tile j is an item (dense tiles)
            for (uint32_t j = 0; j < nj; j += 8) {
                float lm[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint32_t t = (uint32_t)warp + kWarps * (j0 + j + (uint32_t)u);
                    lm[u] = -kInf;
                    if (j + (uint32_t)u < nj && (uint32_t)lane * 32u < chunk_count(g, t)) {
                        const TileRec& R = tt[t];
                        if (all)
                            lm[u] = kInf;
                        else if (R.lcnt == kDenseMark && !(__fsub_rn(R.mt, mx) < dlim))
                            lm[u] = __ldcg(lmax + t * 64u + (uint32_t)lane);
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (lm[u] == kInf || __fsub_rn(lm[u], mx) >= dlim) live |= 1u << (j + (uint32_t)u);
            }
            // item = j << 6 | group << 1 | list
            uint32_t nd = 0, nl = 0;
            for (uint32_t j = 0; j < nj; ++j) {
                const uint32_t t = (uint32_t)warp + kWarps * (j0 + j);
                const TileRec& R = tt[t];
                if (!all && R.lcnt != kDenseMark) {
                    const uint32_t ng = __fsub_rn(R.mt, mx) < dlim ? 0u : (R.lcnt + 31u) / 32u;
                    if ((uint32_t)lane < ng) items[1023u - nl - (uint32_t)lane] = (j << 6) | ((uint32_t)lane << 1) | 1u;
                    nl += ng;
                } else {
                    const bool mine = (live >> j) & 1u;
                    const unsigned m = __ballot_sync(0xFFFFFFFFu, mine);
                    if (mine) items[nd + (uint32_t)__popc(m & ((1u << lane) - 1u))] = (j << 6) | ((uint32_t)lane << 1);
                    nd += (uint32_t)__popc(m);
                }
            }
            __syncwarp();
            // list groups: the pass-1 lists hold every element of a sparse tile with
            // d >= hist_lim (scaled, penalised)
            for (uint32_t k0 = 0; k0 < nl; k0 += 8) {
                float xs[8];
                uint32_t gi[8];  // element index (~0u: none)
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    xs[u] = 0.0f;
                    gi[u] = ~0u;
                    if (k0 + (uint32_t)u >= nl) continue;
                    const uint32_t itm = items[1023u - k0 - (uint32_t)u];
                    const uint32_t t = (uint32_t)warp + kWarps * (j0 + (itm >> 6));
                    const uint32_t e = ((itm >> 1) & 31u) * 32u + (uint32_t)lane;
                    const TileRec& R = tt[t];
                    if (e < R.lcnt) {
                        const uint2 en = __ldcg(lists + R.loff + e);
                        xs[u] = __uint_as_float(en.x);
                        gi[u] = en.y;
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (k0 + (uint32_t)u >= nl) break;  // (warp-uniform)
                    const bool ok = gi[u] != ~0u;
                    const float dd = ok ? __fsub_rn(xs[u], mx) : -kInf;
                    if (!all && !__any_sync(0xFFFFFFFFu, dd >= dlim)) continue;
                    take(gi[u], dd, ok);
                }
            }
            // dense runs through the staging area
            for (uint32_t k0 = 0; k0 < nd; k0 += kGatherRuns) {
                if (__any_sync(0xFFFFFFFFu, sh.abort != 0u)) break;  // (aborted: issue no more copies)
                const uint32_t nb = min((uint32_t)kGatherRuns, nd - k0);
                // run k0 + u: its first element and length (a multiple of 4: 16-byte copies)
                auto run_of = [&](uint32_t u, uint32_t& e0, uint32_t& len) {
                    const uint32_t itm = items[k0 + u];
                    const uint32_t t = (uint32_t)warp + kWarps * (j0 + (itm >> 6));
                    const uint32_t o = ((itm >> 1) & 31u) * 32u;
                    e0 = g.head + t * kTile + o;
                    len = min(32u, chunk_count(g, t) - o);
                };
                uint32_t bytes = 0;
                for (uint32_t u = (uint32_t)lane; u < nb; u += 32) {
                    uint32_t e0, len;
                    run_of(u, e0, len);
                    bytes += len * 4u;
                }
                bytes = __reduce_add_sync(0xFFFFFFFFu, bytes);
                if (lane == 0) {
                    fence_proxy_async_smem();  // (the warp's earlier reads of the area come first)
                    mbar_expect_tx(gbar, bytes);
                }
                __syncwarp();
                uint32_t pb0 = 0, pb1 = 0;  // penalty bits of runs lane and lane + 32
                for (uint32_t u = (uint32_t)lane; u < nb; u += 32) {
                    uint32_t e0, len;
                    run_of(u, e0, len);
                    bulk_load(stage + u * 32u, g.row + e0, len * 4u, gbar, pol);
                    if (pen_on) (u < 32u ? pb0 : pb1) = lane_bits(bitmap, e0);
                }
                if (!wait_bar(sh, gbar, gph & 1u, err) && !gdead) {
                    // aborted: still let this warp's copies land before going on (once)
                    const long long t0 = clock64();
                    while (!mbar_try_wait(gbar, gph & 1u))
                        if (clock64() - t0 > kWaitCycles) {
                            gdead = true;
                            break;
                        }
                }
                ++gph;
                for (uint32_t u = 0; u < nb; ++u) {
                    uint32_t e0, len;
                    run_of(u, e0, len);
                    const bool ok = (uint32_t)lane < len && !sh.abort;
                    const uint32_t pb = __shfl_sync(0xFFFFFFFFu, u < 32u ? pb0 : pb1, (int)(u & 31u));  // (all lanes)
                    float dd = -kInf;
                    if (ok) {
                        float x = stage[u * 32u + (uint32_t)lane];
                        if ((pb >> lane) & 1u) x = penalise(x, penalty);
                        dd = d_of(x, inv_t, mx);
                    }
                    if (!all && !__any_sync(0xFFFFFFFFu, dd >= dlim)) continue;
                    take(e0 + (uint32_t)lane, dd, ok);
                }
                __syncwarp();
            }
        }
        if (lane == 0) sh.gph[warp] = gph;
        __threadfence_block();
        csync();
    };
    gather(0, blim);
    uint32_t gathered_to = blim;
    f.n_cand = hoff[blim] + hcnt[blim];
    for (int q = tid; q < (kNB + 31) / 32; q += kThreads) sh.bsorted[q] = 0u;
    csync();
    auto bucket_of = [&](uint32_t pos) -> uint32_t {  // bucket holding sorted position pos
        uint32_t lo = 0, hi = (uint32_t)kNB - 1;
        while (lo < hi) {
            const uint32_t mid = (lo + hi + 1) >> 1;
            if (hoff[mid] <= pos) lo = mid; else hi = mid - 1;
        }
        return lo;
    };
    auto bend = [&](uint32_t q) -> uint32_t { return hoff[q] + hcnt[q]; };
    auto ensure_gathered = [&](uint32_t q) {
        while (q > gathered_to) {
            const uint32_t hi = min((uint32_t)kNB - 1, gathered_to + 1 + 2 * (gathered_to + 1));
            gather(gathered_to + 1, hi);
            gathered_to = hi;
        }
    };
    // exact key of element i: p = fl(libm expf(d) * inv) (sampler.rs:129-131, ops.rs:409-416)
    auto exact_key = [&](uint32_t i) -> unsigned long long {
        const float d = d_of(penal_g(g.row[i], i), inv_t, mx);
        const float pr = __fmul_rn(exact_expf(d, exptab), inv);
        return ((unsigned long long)(~__float_as_uint(pr)) << 32) | i;
    };
    // Bucket q in exact (p desc, index asc) order: exact keys, then a bitonic sort.
    auto ensure_sorted = [&](uint32_t q) {
        ensure_gathered(q);
        if ((sh.bsorted[q >> 5] >> (q & 31)) & 1u) return;
        const long long ts = clock64();
        const uint32_t cnt = hcnt[q];
        unsigned long long* base = scratch + hoff[q];
        for (uint32_t i = tid; i < cnt; i += kThreads) {
            const unsigned long long kk = base[i];
            if ((uint32_t)kk & kApxKey) base[i] = exact_key((uint32_t)kk & ~kApxKey);
        }
        __threadfence_block();
        csync();
        if (cnt > 1) {
            if (cnt <= (uint32_t)kSortCap) {
                for (uint32_t i = tid; i < cnt; i += kThreads) sbuf[i] = base[i];
                csync();
                bitonic_sort_u64(sbuf, cnt);
                for (uint32_t i = tid; i < cnt; i += kThreads) base[i] = sbuf[i];
            } else {
                bitonic_sort_u64(base, cnt);  // rare: one bucket larger than shared memory
            }
            __threadfence_block();
        }
        if (tid == 0) sh.bsorted[q >> 5] |= 1u << (q & 31);
        csync();
        f.acc_sort += clock64() - ts;
    };
    auto is_sorted = [&](uint32_t q) -> bool { return (sh.bsorted[q >> 5] >> (q & 31)) & 1u; };
    // Buckets [qa, qb] (at most kSortCap elements) as one range in exact order: the
    // buckets ahead of the first ordered steps hold a few candidates each, and one
    // sort of all of them replaces a sort per bucket.
    auto sort_range = [&](uint32_t qa, uint32_t qb) {
        ensure_gathered(qb);
        const long long ts = clock64();
        const uint32_t lo = hoff[qa], cnt = bend(qb) - lo;
        unsigned long long* base = scratch + lo;
        for (uint32_t i = tid; i < cnt; i += kThreads) {
            const unsigned long long kk = base[i];
            sbuf[i] = ((uint32_t)kk & kApxKey) ? exact_key((uint32_t)kk & ~kApxKey) : kk;
        }
        csync();
        bitonic_sort_u64(sbuf, cnt);
        for (uint32_t i = tid; i < cnt; i += kThreads) base[i] = sbuf[i];
        __threadfence_block();
        for (uint32_t q = qa + tid; q <= qb; q += kThreads) atomicOr(&sh.bsorted[q >> 5], 1u << (q & 31));
        csync();
        f.acc_sort += clock64() - ts;
    };
    auto pval = [&](uint32_t q) -> float { return __uint_as_float(~(uint32_t)(scratch[q] >> 32)); };
    // Exact sequential run over sorted positions [0, p1) of the candidate sequence
    // (sampler.rs:137-139 / 148-151 / 156-158).  Buckets are in order; inside a bucket
    // the order matters only around an ordered step (a binade crossing, a tie, a big
    // element, the stop), so chunks of whole buckets are summed in storage order on one
    // grid, and only the bucket holding a chunk's first ordered step is made exact,
    // sorted and run in order.  The first kSerial positions go one by one on thread 0.
    // Returns the stop position or -1.
    auto run = [&](uint32_t p1, int dir, float& s, float thr) -> int {
        if (p1 == 0) return -1;
        {   // a limit inside a bucket needs that bucket in order
            const uint32_t q1 = bucket_of(p1 - 1);
            if (bend(q1) > p1) ensure_sorted(q1);
        }
        uint32_t p = 0;
        uint32_t serial_left = kSerial;
        while (p < p1) {
            const uint32_t b = bucket_of(p);
            if (dir > 0) {
                // Every remaining candidate lies in bucket b or a later one; once
                // their probabilities are all below half the sum's grid unit no
                // later addition changes the sum (and none is a tie).
                const float emax = expf(-(float)b / kBScale) * 1.0001f;
                const float pmax = __fmul_rn(emax, inv) * 1.0001f;
                const int uu = unit_exp(s);
                if (uu > -149 && pmax < ldexpf(1.0f, uu - 1)) return -1;
            }
            ensure_gathered(b);
            const bool b_sorted = is_sorted(b);
            if (serial_left > 0) {
                if (!b_sorted) {
                    // every bucket the serial positions reach, in one sort when they fit
                    // (gathered buckets only: the run may stop before it needs more)
                    uint32_t qs = min(bucket_of(min(p1, p + serial_left) - 1u), gathered_to);
                    while (qs > b && bend(qs) - hoff[b] > (uint32_t)kSortCap) --qs;
                    if (qs > b)
                        sort_range(b, qs);
                    else
                        ensure_sorted(b);
                }
                // the sorted stretch from p (whole sorted buckets in a row are in order)
                uint32_t seg_end = bend(b), q = b;
                while (q + 1u < (uint32_t)kNB && seg_end < p1 && seg_end - p < serial_left && is_sorted(q + 1u)) {
                    ++q;
                    seg_end = bend(q);
                }
                seg_end = min(p1, seg_end);
                const uint32_t m = min(seg_end - p, serial_left);
                for (uint32_t q = tid; q < m; q += kThreads) sh.ser[q] = pval(p + q);
                csync();
                if (tid == 0) {
                    float s2 = s;
                    sh.stop = serial_run(sh.ser, (int)m, dir, s2, thr);
                    sh.fstate = s2;
                }
                csync();
                s = sh.fstate;
                const int st0 = sh.stop;
                csync();
                if (st0 >= 0) return (int)p + st0;
                p += m;
                serial_left -= m;
                continue;
            }
            // chunk [p, e): whole buckets, or a piece of a sorted bucket (a bucket larger
            // than a chunk is sorted first)
            uint32_t e;
            if (b_sorted || bend(b) - p > (uint32_t)kChunk) {
                if (!b_sorted) ensure_sorted(b);
                e = min(min(p1, bend(b)), p + (uint32_t)kChunk);
            } else {
                uint32_t q = b;
                e = bend(b);
                while (q + 1 < (uint32_t)kNB && q + 1 <= gathered_to && bend(q + 1) <= p1 &&
                       bend(q + 1) - p <= (uint32_t)kChunk && !((sh.bsorted[(q + 1) >> 5] >> ((q + 1) & 31)) & 1u)) {
                    ++q;
                    e = bend(q);
                }
                e = min(e, p1);
            }
            const uint32_t tc = e - p;
            float v[kVpt];
            load_sorted_tile(scratch + p, tc, v);
            // increments on the running value's grid, exact where an approximate key's
            // error bound could change them
            const int uu = unit_exp(s);
            const uint32_t A = grid_count(s, uu);
            uint32_t inc[kVpt];
            uint32_t t = 0, fl = 0, spm = 0;
#pragma unroll 1
            for (int i = 0; i < kVpt; ++i) {
                inc[i] = 0;
                const int li = li_of(i);
                if ((uint32_t)li < tc) {
                    const unsigned long long kk = scratch[p + li];
                    uint32_t vb = __float_as_uint(v[i]);
                    if ((uint32_t)kk & kApxKey) {
                        const Cls lo = classify(vb > 8u ? vb - 8u : 0u, uu), hi = classify(vb + 8u, uu);
                        if (!(lo.inc == hi.inc && !lo.tie && !hi.tie && !lo.big && !hi.big) && !(lo.big && hi.big)) {
                            const unsigned long long ek = exact_key((uint32_t)kk & ~kApxKey);
                            scratch[p + li] = ek;
                            v[i] = __uint_as_float(~(uint32_t)(ek >> 32));
                            vb = __float_as_uint(v[i]);
                        }
                    }
                    const Cls c = classify(vb, uu);
                    inc[i] = c.inc;
                    t = sat_add(t, c.inc);
                    if (c.tie || c.big) {
                        fl = 1u;
                        spm |= 1u << i;
                    }
                }
            }
            t = block_reduce_u32(t, SatAdd(), sh.red);
            fl = block_reduce_u32(fl, OrOp(), sh.red2);
            const float tq = (dir > 0 && thr < kInf) ? ldexpf(thr, -uu) : kInf;
            const bool fast = dir > 0 ? (!fl && A + t <= kTwo24 - 1u && (float)(A + t) < tq)
                                      : (!fl && t < A - grid_lower(uu));
            if (fast) {
                s = grid_value(uu, dir > 0 ? A + t : A - t);
                p = e;
                continue;
            }
            // the first ordered step in storage order: its bucket is where the order matters
            uint32_t incl[kVpt];
            (void)block_incl_scan(inc, incl, sh.red);
            uint32_t cand = 0xFFFFFFFFu;
            const uint32_t lower = grid_lower(uu);
#pragma unroll 1
            for (int i = 0; i < kVpt; ++i) {
                const int li = li_of(i);
                if ((uint32_t)li < tc && (uint32_t)li < cand &&
                    needs_step(dir, (spm >> i) & 1u, A, incl[i], lower, tq))
                    cand = (uint32_t)li;
            }
            uint32_t first = block_reduce_u32(cand, MinU(), sh.red2);
            if (first >= tc) first = 0;  // (cannot happen: then order the chunk's first bucket)
            const uint32_t qe = bucket_of(p + first);
            const uint32_t bstart = max(p, hoff[qe]);
            // the buckets before qe in this chunk: summed in any order on this grid
            if (bstart > p) {
#pragma unroll 1
                for (int i = 0; i < kVpt; ++i)
                    if ((uint32_t)li_of(i) == bstart - p - 1) sh.fstate = grid_value(uu, dir > 0 ? A + incl[i] : A - incl[i]);
                csync();
                s = sh.fstate;
                csync();
            }
            ensure_sorted(qe);
            // bucket qe (from bstart) in exact order
            uint32_t q0 = bstart;
            const uint32_t qend = min(p1, bend(qe));
            while (q0 < qend) {
                const uint32_t tq2 = min((uint32_t)kChunk, qend - q0);
                float w[kVpt];
                uint32_t ex = 0xFFFFFFFFu;
                load_sorted_tile(scratch + q0, tq2, w);
                const int stp = tile2(w, ex, 0, (int)tq2, dir, s, thr, NoExact(), sh);
                if (stp >= 0) return (int)q0 + stp;
                q0 += tq2;
            }
            p = qend;
        }
        return -1;
    };
    // top-p scan capped at k survivors (sampler.rs:122-146)
    float cum = 0.0f;
    int stp = run(k, +1, cum, topp_on ? top_p : kInf);
    f.cutoff = stp >= 0 ? (uint32_t)stp + 1 : k;
    f.sum = cum;
    // draw (sampler.rs:152-162)
    if (f.sum > 0.0f) {
        f.rr = __fmul_rn(next_f32(&f.st), f.sum);
        f.r0 = f.rr;
        float rv = f.rr;
        stp = run(f.cutoff, -1, rv, 0.0f);
        f.pos = stp >= 0 ? (uint32_t)stp : f.cutoff - 1;
    } else {
        f.pos = 0;
    }
    // The element at the drawn position.  Buckets split the order by d, so elements of
    // equal probability (d a few ulp apart) can sit on both sides of a bucket boundary,
    // each side in index order: such a group is put in index order across the boundary.
    uint32_t qp = bucket_of(f.pos);
    ensure_sorted(qp);
    const uint32_t pk = (uint32_t)(scratch[f.pos] >> 32);
    uint32_t g0 = hoff[qp], g1 = bend(qp);
    while (g0 < f.pos && (uint32_t)(scratch[g0] >> 32) != pk) ++g0;   // (sorted: a short scan of
    while (g1 > f.pos + 1u && (uint32_t)(scratch[g1 - 1u] >> 32) != pk) --g1;  // equal keys is rare)
    bool wide = false;
    // bucket q holds d in (-(q+1)/kBScale, -q/kBScale], so its probabilities lie in
    // [P(-(q+1)/kBScale), P(-q/kBScale)] with P(d) = fl(expf(d) inv) monotone: a
    // neighbour can hold the same probability only if pk reaches that bound
    auto pbound = [&](uint32_t q) -> float {
        return __fmul_rn(exact_expf(-(float)q / kBScale, exptab), inv);
    };
    const float pv = __uint_as_float(~pk);
    const bool look_down = qp > 0u && pv >= pbound(qp);
    const bool look_up = qp + 1u < (uint32_t)kNB && pv <= pbound(qp + 1u);
    for (uint32_t q = qp; look_down && g0 == hoff[q] && q > 0u;) {  // the group reaches the start of bucket q
        --q;
        if (hcnt[q] == 0u) continue;
        ensure_sorted(q);
        if ((uint32_t)(scratch[bend(q) - 1u] >> 32) != pk) break;
        while (g0 > hoff[q] && (uint32_t)(scratch[g0 - 1u] >> 32) == pk) --g0;
        wide = true;
    }
    for (uint32_t q = qp; look_up && g1 == bend(q) && q + 1u < (uint32_t)kNB;) {  // ... or the end of bucket q
        ++q;
        if (hcnt[q] == 0u) continue;
        ensure_sorted(q);
        if ((uint32_t)(scratch[hoff[q]] >> 32) != pk) break;
        while (g1 < bend(q) && (uint32_t)(scratch[g1] >> 32) == pk) ++g1;
        wide = true;
    }
    if (wide) {
        bitonic_sort_u64(scratch + g0, g1 - g0);  // equal high words: index order
        __threadfence_block();
        csync();
    }
    f.chosen = scratch[f.pos];
    csync();
}

// ------------------------------------------------------------------- the kernel ----
extern "C" __global__ void __launch_bounds__(kBlock, 2) lrs_sample_rows(SampleArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ RowShared sh;
    float* ring = reinterpret_cast<float*>(smem_raw);
    unsigned char* regA = smem_raw + kRingBytes;
    unsigned char* regB = regA + kRegionABytes;
    TileRec* ttab_s = reinterpret_cast<TileRec*>(regB + kRegionBBytes);
    float* wbx = reinterpret_cast<float*>(regA);                                  // pass 1, path K
    uint32_t* wbi = reinterpret_cast<uint32_t*>(regA + (size_t)kKCap * 4);
    uint32_t* hcnt = reinterpret_cast<uint32_t*>(regA);                           // pass 2 on, path N
    uint32_t* hoff = reinterpret_cast<uint32_t*>(regA + (size_t)kNB * 4);
    uint32_t* whist = reinterpret_cast<uint32_t*>(regB);                          // pass 1, path K
    float* cand_x = reinterpret_cast<float*>(regB);                               // finish, path K
    uint32_t* cand_i = reinterpret_cast<uint32_t*>(regB + (size_t)kKCap * 4);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(regB + (size_t)kKCap * 8);
    unsigned long long* sbuf = reinterpret_cast<unsigned long long*>(regB);      // finish, path N
    uint32_t* cursor = reinterpret_cast<uint32_t*>(regB);
    unsigned long long* scratch = a.scratch + (uint64_t)blockIdx.x * a.scratch_stride;
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(scratch + a.bitmap_off);
    TileRec* ttab_g = reinterpret_cast<TileRec*>(scratch + a.tiles_off);
    // per tile t (pass 1): lrec[64 t + lane] the lane's candidate exp sum, lrec[64 t + 32 + lane]
    // the max of its run's scaled logits
    float* lrec = reinterpret_cast<float*>(scratch + a.lanes_off);
    uint2* lists = reinterpret_cast<uint2*>(scratch + a.lists_off);  // per warp: sparse tiles' candidates
    const ExpTable exptab{a.exp_index, a.exp_entries, a.exp_near};
    const float kInf = __int_as_float(0x7F800000);
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    if (tid == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&sh.full[i], 1);
            mbar_init(&sh.empty[i], 1);
        }
        for (int i = 0; i < kRowQ; ++i) {
            mbar_init(&sh.rq_full[i], 1);
            mbar_init(&sh.rq_empty[i], 1);
        }
        for (int i = 0; i < kWarps; ++i) {
            mbar_init(&sh.bwait[i], 1);
            mbar_init(&sh.gbar[i], 1);
            sh.gph[i] = 0u;
        }
        sh.abort = 0u;
        sh.bseq = 0xFFFFFFFFu;
        sh.p1done = 0u;
        sh.claim_ok = 0u;
        fence_barrier_init();
    }
    __syncthreads();
    if (warp == kWarps) {  // the producer warp
        if (lane == 0) producer(a, sh, ring);
        return;
    }

    uint32_t qbase = 0;  // loads of earlier rows (same count in every consumer thread)
    uint32_t rqi = 0;
    uint32_t bcnt = 0;   // batons this warp has received (its bwait phase)
    for (;;) {
        if (tid == 0) {
            const uint32_t qs = rqi % kRowQ;
            uint32_t rr = a.rows;
            if (wait_bar(sh, &sh.rq_full[qs], (rqi / kRowQ) & 1u, a.err_flag)) rr = sh.rq_row[qs];
            mbar_arrive(&sh.rq_empty[qs]);
            sh.misc[0] = rr;
        }
        ++rqi;
        csync();
        const uint32_t r = sh.misc[0];
        if (r >= a.rows) break;

        const lrs_params P = a.params[r];
        const Geo g = row_geometry(a, r);
        const uint32_t n = g.n;
        const float temperature = P.temperature;
        const float penalty = P.repetition_penalty;
        const bool greedy = temperature <= 0.0f;              // sampler.rs:62, 104 (NaN -> stochastic)
        const bool fast_greedy = greedy && penalty == 1.0f;   // sampler.rs:62
        const bool pen_on = !fast_greedy && penalty != 1.0f;  // sampler.rs:82
        const uint32_t k = (P.top_k == 0 || P.top_k > n) ? n : P.top_k;  // sampler.rs:122-126
        const bool stochastic = !greedy;
        const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;           // sampler.rs:136
        bool pathK = stochastic && n >= 2 && k < n && k <= (uint32_t)kKMax;
        unsigned long long st = a.state[r];
        const uint32_t passes = row_passes(P, n);
        const bool lists_on = passes == 2;  // candidate lists and dense tiles for pass 2
        const uint32_t q1 = qbase, q2 = qbase + g.nchunks;  // load numbers of pass 1 / pass 2 tile 0
        qbase += g.nchunks;                                  // (+ the dense tiles, after the prep)
        TileRec* const tt = g.nchunks <= (uint32_t)kTilesSmem ? ttab_s : ttab_g;

        lrs_row_info& inf = sh.info;  // written by thread 0 only
        if (tid == 0) {
            inf.status = LRS_OK;
            inf.token = 0;
            inf.path = greedy ? (fast_greedy ? 0u : 1u) : (n == 1 ? 3u : 2u);
            inf.k = k;
            inf.cutoff = 0;
            inf.pos = 0;
            inf.max = 0.0f;
            inf.sum_exp = 0.0f;
            inf.surv_sum = 0.0f;
            inf.r0 = 0.0f;
            inf.prob = 1.0f;
            inf.n_cand = 0;
            inf.events = 0;
            for (int q = 0; q < 8; ++q) inf.cycles[q] = 0;
            inf.reserved = 0;
        }
        long long t_mark = clock64();
        auto sat32 = [](long long d) -> uint32_t { return d > 0xFFFFFFFFll ? 0xFFFFFFFFu : (d < 0 ? 0u : (uint32_t)d); };
        auto lap = [&](int q) {
            const long long now = clock64();
            if (tid == 0) inf.cycles[q] = sat32(now - t_mark);
            t_mark = now;
        };
        long long acc_sort = 0;
        int32_t status = LRS_OK;
        uint32_t token = 0;
        float prob = 1.0f;
        bool advance_state = false;

        // penalty set: distinct ids of the window with id < n (sampler.rs:82-102)
        const uint32_t hlen = a.hist_len ? a.hist_len[r] : 0u;
        const uint32_t* hrow = a.hist ? a.hist + (uint64_t)r * a.hist_ld : nullptr;
        uint32_t hstart = 0;
        if (P.repeat_last_n != 0) hstart = hlen > P.repeat_last_n ? hlen - P.repeat_last_n : 0u;
        if (pen_on && n > 0) {
            for (uint32_t j = hstart + tid; j < hlen; j += kThreads) {
                const uint32_t t = hrow[j];
                if (t < n) atomicOr(&bitmap[t >> 5], 1u << (t & 31));
            }
        }
        if (lists_on)
            for (uint32_t t = tid; t < g.nchunks; t += kThreads) tt[t].tag = kNoTag;
        if (tid == 0) {
            sh.cand_n = 0;
            sh.cand_over = 0;
            sh.theta = -kInf;
            sh.delta_min = kInf;
            sh.ktheta = fkey(-kInf);
            sh.kdelta = __float_as_uint(kInf);
            sh.vk = -kInf;
            sh.misc[7] = 0;
            sh.events = 0;
            sh.wover = 0;
            sh.ndense = 0;
        }
        csync();

        const float inv_t = stochastic ? __fdiv_rn(1.0f, temperature) : 1.0f;  // sampler.rs:115
        auto penal_g = [&](float x, uint32_t gi) -> float {                   // sampler.rs:96-100
            if (pen_on && ((__ldcg(bitmap + (gi >> 5)) >> (gi & 31)) & 1u)) return penalise(x, penalty);
            return x;
        };
        // penalty bits of this lane's run of tile t (loaded one tile ahead of use)
        auto tile_bits = [&](uint32_t t) -> uint32_t {
            const uint32_t c = chunk_count(g, t), o = (uint32_t)lane * 32u;
            const uint32_t nv = o < c ? min(32u, c - o) : 0u;
            if (!pen_on || !nv) return 0u;
            return lane_bits(bitmap, g.head + t * kTile + o) & (nv >= 32u ? 0xFFFFFFFFu : ((1u << nv) - 1u));
        };

        if (n == 0) goto row_done;  // sampler.rs:57-60

        {
            // -------------------------------------------------------- pass 1 ----
            float m_w = -kInf;          // warp: running max of the scaled logits (its own tiles; warp 0: and
                                        // the unaligned head and tail elements)
            float m_pre = -kInf;        // warp: max of elements known to precede its next tile (its own
                                        // earlier tiles; warp 0: the head, never the tail)
            float bv = -kInf;           // lane: greedy best value and index
            uint32_t bi = 0xFFFFFFFFu;
            WState ws{0u, -kInf, kInf, 0u};  // warp: path-K filter
            bool kact = pathK;          // warp: still filtering
            float* wx = wbx + warp * kWCap;
            uint32_t* wi = wbi + warp * kWCap;
            uint32_t* wh = whist + warp * 256;
            // Candidate lists.  S, the exact sum before an element, is at least the exp of the
            // largest d before its tile, e_mp; the prep's grid bound for the tile is then at
            // least grid(e_mp) - 1 (rows of n <= 2^21: delta < 1/4), so an element with
            // d < d_mp - 26 ln 2 - 0.01 adds exactly nothing.  A scaled logit more than
            // theta = 18.1 (+ rounding slack) below a lower bound of the prefix max is such an
            // element, and its d < -18.0999 lies below the path-N bucket range as well.
            const float theta_c = g.n <= (1u << 21) ? 18.1f : 18.8f;
            const uint32_t capw = ((g.nchunks + kWarps - 1) / kWarps) * kDense;
            uint2* wlist = lists + (size_t)warp * capw;
            uint32_t woff = 0;   // warp: entries written to its list
            uint32_t front = 0;  // tiles [0, front) folded into gpm
            float gpm = -kInf;   // max over tiles [0, front) (published by any warp)

            // unaligned head and tail elements (at most 3 + 3), plain loads, warp 0
            if (warp == 0) {
                const uint32_t edges = g.head + g.tail;
                const bool mine = (uint32_t)lane < edges;
                uint32_t gi = 0;
                float x = -kInf;
                if (mine) {
                    gi = (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
                    x = penal_g(g.row[gi], gi);
                }
                if (greedy) {
                    if (mine && (x > bv || (x == bv && gi < bi))) {
                        bv = x;
                        bi = gi;
                    }
                } else {
                    const float xs = __fmul_rn(x, inv_t);
                    m_w = fmax_nan(m_w, warp_max_nan(mine ? xs : -kInf));
                    m_pre = warp_max_nan(mine && (uint32_t)lane < g.head ? xs : -kInf);
                    if (kact) {  // at most 6 entries: the buffer is empty
                        const bool hit = mine && xs >= ws.theta;
                        const unsigned hb = __ballot_sync(0xFFFFFFFFu, hit);
                        if (hit) {
                            const uint32_t p = (uint32_t)__popc(hb & ((1u << lane) - 1u));
                            wx[p] = xs;
                            wi[p] = gi;
                        }
                        ws.wcnt = (uint32_t)__popc(hb);
                    }
                }
            }
            uint32_t bits_nx = (uint32_t)warp < g.nchunks ? tile_bits((uint32_t)warp) : 0u;
            const float2 it2 = make_float2(inv_t, inv_t);
            for (uint32_t t = (uint32_t)warp; t < g.nchunks; t += kWarps) {
                const uint32_t qq = q1 + t, s = qq % kSlots;
                const uint32_t cnt = chunk_count(g, t);
                const uint32_t tb = g.head + t * kTile;
                const uint32_t l0 = (uint32_t)lane * 32u;
                const uint32_t nval = l0 < cnt ? min(32u, cnt - l0) : 0u;
                const uint32_t bits = bits_nx;
                if (t + kWarps < g.nchunks) bits_nx = tile_bits(t + kWarps);
                // candidate threshold from a lower bound of the max before this tile
                float cthr = -kInf;
                if (lists_on) {
                    // fold in the published maxima of earlier tiles: lane u reads the (max, tag)
                    // word of tile front + u, and the leading run of published ones is folded
                    {
                        const uint32_t nb = min(32u, t - front);
                        unsigned long long w = 0ull;
                        if ((uint32_t)lane < nb) w = *reinterpret_cast<volatile unsigned long long*>(&tt[front + lane].mt);
                        const unsigned pub = __ballot_sync(0xFFFFFFFFu, (uint32_t)lane < nb && (uint32_t)(w >> 32) == r);
                        const uint32_t adv = (uint32_t)__clz(__brev(~pub));
                        if (adv != 0u) {
                            const float v = (uint32_t)lane < adv ? __uint_as_float((uint32_t)w) : -kInf;
                            const float vm = fkey_inv(__reduce_max_sync(0xFFFFFFFFu, fkey(v)));
                            gpm = __any_sync(0xFFFFFFFFu, v != v) ? __uint_as_float(0x7FC00000u) : fmax_nan(gpm, vm);
                            front += adv;
                        }
                    }
                    const float mp = fmax_nan(m_pre, gpm);
                    cthr = __fsub_rn(mp, __fmaf_rn(fabsf(mp), 9.5367432e-07f, theta_c));  // slack 2^-20 |mp|
                }
                wait_full(sh, qq, a.err_flag);
                const float* slot = ring + (size_t)s * kTile + l0;
                float ml = -kInf;                // lane: max of its scaled logits
                uint32_t cmask = 0, hmask = 0;   // lane: candidate / top-k hit run offsets
                if (kact) {
                    // every warp's threshold bounds the row's k-th largest from below: take
                    // the largest one published (its margin is in kdelta)
                    const float gth = fkey_inv(*reinterpret_cast<volatile uint32_t*>(&sh.ktheta));
                    if (gth > ws.theta) ws.theta = gth;
                }
                const float theta = kact ? ws.theta : kInf;
                if (greedy) {
#pragma unroll 2
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                        if (c4 >= nval) continue;
                        const float4 q = *reinterpret_cast<const float4*>(slot + c4);
                        float x[4] = {q.x, q.y, q.z, q.w};
                        const uint32_t pb = (bits >> c4) & 15u;
                        if (pb) {
#pragma unroll
                            for (int c = 0; c < 4; ++c)
                                if ((pb >> c) & 1u) x[c] = penalise(x[c], penalty);
                        }
                        // lowest index among the maximal non-NaN values (strict '>' from index 0)
                        const uint32_t gi0 = tb + l0 + c4;
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if (x[c] > bv || (x[c] == bv && gi0 + c < bi)) {
                                bv = x[c];
                                bi = gi0 + c;
                            }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.empty[s]);
                    continue;
                }
                // The penalty (a few ids per row) is applied to the staged run in place, so
                // the loop below and pass 1's later reads of the run see penalised values
                // (pass 2 stages the tile again and applies it itself).
                for (uint32_t pm = bits; pm; pm &= pm - 1u) {
                    float* const px = const_cast<float*>(slot) + (__ffs(pm) - 1);
                    *px = penalise(*px, penalty);
                }
                const uint32_t bits1 = 0u;  // (pass 1 from here on: already applied)
                if (nval == 32u) {
                    // a full run: its max first (packed products, three-input maxima), the
                    // candidate and top-k masks only in lanes whose max reaches a threshold.
                    // The packed products are only compared here: the compiler may fuse a
                    // packed product into a following add even when both are written with
                    // explicit rounding, so every difference of a product (x inv_t - max)
                    // is computed from a scalar __fmul_rn product
                    float ma = -kInf, mb = -kInf;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                        const float4 q = *reinterpret_cast<const float4*>(slot + c4);
                        const float2 lo = __fmul2_rn(make_float2(q.x, q.y), it2);
                        const float2 hi = __fmul2_rn(make_float2(q.z, q.w), it2);
                        ma = fmax3_nan(ma, lo.x, lo.y);
                        mb = fmax3_nan(mb, hi.x, hi.y);
                    }
                    ml = fmax_nan(ma, mb);
                    if (ml >= cthr || ml >= theta) {
#pragma unroll 4
                        for (int j = 0; j < 8; ++j) {
                            const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                            const float4 q = *reinterpret_cast<const float4*>(slot + c4);
                            const float2 lo = __fmul2_rn(make_float2(q.x, q.y), it2);
                            const float2 hi = __fmul2_rn(make_float2(q.z, q.w), it2);
                            const float xs[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                if (xs[c] >= cthr) cmask |= 1u << (c4 + c);
                                if (xs[c] >= theta) hmask |= 1u << (c4 + c);
                            }
                        }
                    }
                } else {
#pragma unroll 4
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                        if (c4 >= nval) continue;
                        const float4 q = *reinterpret_cast<const float4*>(slot + c4);
                        const float x[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float xs = __fmul_rn(x[c], inv_t);
                            ml = fmax_nan(ml, xs);
                            if (xs >= cthr) cmask |= 1u << (c4 + c);
                            if (xs >= theta) hmask |= 1u << (c4 + c);
                        }
                    }
                }
                const float mt = warp_max_nan(ml);
                // path K: the tile's hits join the warp's buffer; a few hits with room in
                // the buffer (the common case once a threshold is set) go straight in
                const uint32_t nhit = kact ? __reduce_add_sync(0xFFFFFFFFu, (uint32_t)__popc(hmask)) : 0u;
                if (nhit != 0u && ws.theta > -kInf && ws.wcnt + nhit <= (uint32_t)kWCap) {
                    const uint32_t nh = (uint32_t)__popc(hmask);
                    uint32_t o = ws.wcnt + warp_incl_scan_plain(nh) - nh;
                    for (uint32_t m = hmask; m; m &= m - 1u) {
                        const int pos = __ffs(m) - 1;
                        wx[o] = __fmul_rn(slot[pos], inv_t);  // (the staged run is penalised)
                        wi[o] = tb + l0 + (uint32_t)pos;
                        ++o;
                    }
                    ws.wcnt += nhit;
                    __syncwarp();
                } else if (nhit != 0u) {
                    const float th_in = ws.theta;
                    ws = topk_tile(slot, hmask, bits1, penalty, inv_t, tb + l0, fmax_nan(m_w, mt), k, wx, wi, wh, ws);
                    if (lane == 0 && ws.theta > th_in && !ws.over) {
                        atomicMin(&sh.kdelta, __float_as_uint(ws.wdelta));  // (before the threshold)
                        __threadfence_block();
                        atomicMax(&sh.ktheta, fkey(ws.theta));
                    }
                    if (ws.over) {
                        kact = false;
                        if (lane == 0) sh.wover = 1u;
                    }
                }
                // The candidates: their exp relative to the lane max (the estimate leaves
                // out the rest, each below 2^-26 of the prefix max's term: the estimate
                // only gets smaller, which keeps its bound), and for a sparse tile the list.
                const uint32_t nc = (uint32_t)__popc(cmask);
                const uint32_t cinc = warp_incl_scan_plain(nc);
                const uint32_t ncand = __shfl_sync(0xFFFFFFFFu, cinc, 31);
                const bool dense = ncand > (uint32_t)kDense;
                float sl = 0.0f;
                if (dense) {
                    // many candidates: one predicated pass over the staged run
                    float sp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                        if (c4 >= nval) continue;
                        const float4 q = *reinterpret_cast<const float4*>(slot + c4);
                        float x[4] = {q.x, q.y, q.z, q.w};
                        const uint32_t pb = (bits1 >> c4) & 15u;
                        if (pb) {
#pragma unroll
                            for (int c = 0; c < 4; ++c)
                                if ((pb >> c) & 1u) x[c] = penalise(x[c], penalty);
                        }
                        const uint32_t cb = cmask >> c4;
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float ev = ex2_approx(__fmul_rn(__fsub_rn(__fmul_rn(x[c], inv_t), ml), kLog2e));
                            sp[c] += ((cb >> c) & 1u) ? ev : 0.0f;
                        }
                    }
                    sl = (sp[0] + sp[1]) + (sp[2] + sp[3]);
                } else {
                    // lane-rotated order (distinct banks); each entry at its index-order place
                    const uint32_t p0 = woff + cinc - nc;
                    uint32_t m = __funnelshift_r(cmask, cmask, lane);
                    while (m) {
                        const int pos = (__ffs(m) - 1 + lane) & 31;
                        m &= m - 1u;
                        float xv = slot[pos];
                        if ((bits1 >> pos) & 1u) xv = penalise(xv, penalty);
                        const float xs = __fmul_rn(xv, inv_t);
                        sl += ex2_approx(__fmul_rn(__fsub_rn(xs, ml), kLog2e));
                        wlist[p0 + (uint32_t)__popc(cmask & ((1u << pos) - 1u))] =
                            make_uint2(__float_as_uint(xs), tb + l0 + (uint32_t)pos);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.empty[s]);
                // tile statistics: max, and per lane its candidates' exp sum relative to the tile max
                const float cl = (ml == -kInf || mt != mt || sl == 0.0f)
                                     ? 0.0f
                                     : __fmul_rn(sl, ex2_approx(__fmul_rn(__fsub_rn(ml, mt), kLog2e)));
                lrec[t * 64u + (uint32_t)lane] = cl;
                lrec[t * 64u + 32u + (uint32_t)lane] = ml;
                const float tot = warp_sum_f(cl);
                if (lane == 0) {
                    TileRec& R = tt[t];
                    R.pt = tot;
                    R.loff = (uint32_t)warp * capw + woff;
                    R.lcnt = dense ? kDenseMark : ncand;
                    if (dense)
                        atomicOr(&sh.dense[t >> 5], 1u << (t & 31));
                    else
                        atomicAnd(&sh.dense[t >> 5], ~(1u << (t & 31)));
                    *reinterpret_cast<volatile unsigned long long*>(&R.mt) =
                        ((unsigned long long)r << 32) | __float_as_uint(mt);  // publishes mt
                    __threadfence_block();
                    atomicAdd(const_cast<uint32_t*>(&sh.p1done), 1u);
                }
                if (!dense) woff += ncand;
                m_w = fmax_nan(m_w, mt);
                m_pre = fmax_nan(m_pre, mt);
            }
            if (greedy) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    sh.gvs[warp] = bv;
                    sh.gis[warp] = bi;
                }
            } else if (lane == 0) {
                sh.wmax[warp] = m_w;
                sh.wcnt[warp] = ws.wcnt;
                sh.wdelta[warp] = ws.wdelta;
            }
            csync();
            lap(0);

            if (greedy) {
                // sampler.rs:62-70 and 104-113; NaN at index 0 -> 0
                float b = sh.gvs[0];
                uint32_t ix = sh.gis[0];
                for (int w = 1; w < kWarps; ++w)
                    if (sh.gvs[w] > b || (sh.gvs[w] == b && sh.gis[w] < ix)) {
                        b = sh.gvs[w];
                        ix = sh.gis[w];
                    }
                const float x0 = penal_g(g.row[0], 0);
                if (x0 != x0 || ix == 0xFFFFFFFFu) ix = 0;
                token = ix;
                prob = 1.0f;
                goto row_done;
            }

            // ---------------------------------------------- stochastic rows ----
            float mx = sh.wmax[0];
            for (int w = 1; w < kWarps; ++w) mx = fmax_nan(mx, sh.wmax[w]);
            if (tid == 0) inf.max = mx;
            // NaN scaled logit or infinite max -> NaN probabilities -> the reference
            // panics at sampler.rs:129/132 (n >= 2)
            const bool bad = (mx != mx) || (fabsf(mx) == kInf);
            if (n == 1) {
                // one logit: one uniform is consumed and the token is 0 (sampler.rs:155-162)
                (void)next_f32(&st);
                advance_state = true;
                token = 0;
                prob = 1.0f;
                goto row_done;
            }
            if (pathK && !bad) {
                if (sh.wover) {
                    pathK = false;
                } else {
                    // the union of the warp buffers, then the final compaction against the row max
                    uint32_t off = 0, tot = 0;
                    for (int w = 0; w < kWarps; ++w) {
                        if (w < warp) off += sh.wcnt[w];
                        tot += sh.wcnt[w];
                    }
                    const uint32_t mine = sh.wcnt[warp];
                    for (uint32_t i = (uint32_t)lane; i < mine; i += 32) {
                        cand_x[off + i] = wx[i];
                        cand_i[off + i] = wi[i];
                    }
                    if (tid == 0) {
                        float dm = kInf;
                        for (int w = 0; w < kWarps; ++w) dm = fminf(dm, sh.wdelta[w]);
                        dm = fminf(dm, __uint_as_float(sh.kdelta));  // thresholds taken from other warps
                        sh.cand_n = tot;
                        sh.delta_min = dm;
                    }
                    csync();
                    compact_candidates(cand_x, cand_i, k, mx, sh);
                    if (sh.cand_over || sh.cand_n > (uint32_t)kKSortMax) pathK = false;
                    // candidates dropped by earlier compactions must lie below every
                    // probability tie of the final k-th value
                    if (pathK && sh.delta_min < kInf && tie_margin(sh.vk, mx) > 4.0f * sh.delta_min) pathK = false;
                    csync();
                }
            }
            const uint32_t nk = sh.cand_n;
            const bool pathN = !pathK;
            const float hist_lim = -(float)(kNB - 1) / kBScale;

            // ---------------------------------------------------------- prep ----
            if (pathN && !bad)
                for (int i = tid; i < kNB; i += kThreads) hcnt[i] = 0;
            if (warp == 0) {
                // pass-2 load numbers of the dense tiles (the producer streams them in order)
                uint32_t dn_acc = 0;
                for (uint32_t base = 0; base < g.nchunks; base += 32) {
                    const uint32_t t = base + (uint32_t)lane;
                    const bool dn = t < g.nchunks && tt[t].lcnt == kDenseMark;
                    const unsigned m = __ballot_sync(0xFFFFFFFFu, dn);
                    if (dn) tt[t].rank = dn_acc + (uint32_t)__popc(m & ((1u << lane) - 1u));
                    dn_acc += (uint32_t)__popc(m);
                }
                if (lane == 0) sh.ndense = dn_acc;
            }
            if (!bad && warp == 0) {
                // the unaligned head elements open the sequential sum (ops.rs:408-411)
                float eh = 0.0f, dh = 0.0f;
                bool exh = true;
                if ((uint32_t)lane < g.head) {
                    dh = d_of(penal_g(g.row[lane], lane), inv_t, mx);
                    exh = dh == 0.0f;
                    eh = exh ? 1.0f : expf(dh);
                }
                const float s0 = warp_serial_add(0.0f, eh, dh, exh, 0, (int)g.head, exptab);
                // Running-sum estimate P at every tile start from the tile statistics.
                // The exact sequential sum there, S, satisfies S >= P (1 - delta) with
                // delta = i 2^-23 + 2^-13 (i elements before the tile): each of the i
                // roundings moves it by at most 2^-24 S, and P's own error (approximate exp
                // of arguments rounded once, f32 summation) is below 2^-14.  So the grid of
                // S is at least ulo = grid(P (1 - delta)) over the whole tile, and an
                // element with d < (ulo - 1) ln 2 - 0.01 adds exactly nothing.
                float run = s0;
                int umin = 0x7FFFFFFF, umax = -0x7FFFFFFF;
                for (uint32_t base = 0; base < g.nchunks; base += 32) {
                    const uint32_t t = base + (uint32_t)lane;
                    const bool in = t < g.nchunks;
                    float mt = -kInf, pt = 0.0f;
                    uint32_t lcnt = 0;
                    if (in) {
                        mt = tt[t].mt;
                        pt = tt[t].pt;
                        lcnt = tt[t].lcnt;
                    }
                    float c = 0.0f;
                    if (in && mt != -kInf) c = __fmul_rn(pt, ex2_approx(__fmul_rn(__fsub_rn(mt, mx), kLog2e)));
                    const float incl = warp_incl_scan_f(c);
                    float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
                    if (lane == 0) excl = 0.0f;
                    const float ptile = __fadd_rn(run, excl);
                    run = __fadd_rn(run, __shfl_sync(0xFFFFFFFFu, incl, 31));
                    const float dl = __fmaf_rn((float)(g.head + t * kTile), 1.1920929e-07f, 1.2207031e-04f);
                    const int ulo = unit_exp(__fmul_rn(ptile, __fsub_rn(1.0f, dl)));
                    const float dmax = __fsub_rn(mt, mx);
                    const float thr = __fsub_rn(__fmul_rn((float)(ulo - 1), 0.69314718f), 0.01f);
                    const bool has = lcnt != 0u;  // a sparse tile without candidates adds nothing
                    const bool sum_live = in && has && dmax >= thr;
                    const bool hist_live = in && has && pathN && dmax >= hist_lim;
                    if (in) {
                        tt[t].pt = ptile;
                        tt[t].flags = (uint32_t)(ulo + 256) | (sum_live ? kSumLive : 0u) | (hist_live ? kHistLive : 0u);
                    }
                    if (sum_live) {
                        umin = min(umin, ulo);
                        umax = max(umax, ulo);
                    }
                }
                // next sum-live tile after each tile (the baton's route)
                uint32_t carry = g.nchunks;
                if (g.nchunks) {
                    for (int base = (int)((g.nchunks - 1) & ~31u); base >= 0; base -= 32) {
                        const uint32_t t = (uint32_t)base + (uint32_t)lane;
                        const bool in = t < g.nchunks;
                        const uint32_t fl = in ? tt[t].flags : 0u;
                        const unsigned m = __ballot_sync(0xFFFFFFFFu, (fl & kSumLive) != 0u);
                        const unsigned above = lane == 31 ? 0u : (m & (0xFFFFFFFFu << (lane + 1)));
                        const uint32_t nxt = above ? (uint32_t)base + (uint32_t)(__ffs(above) - 1) : carry;
                        if (in) tt[t].next = nxt;
                        if (m) carry = (uint32_t)base + (uint32_t)(__ffs(m) - 1);
                    }
                }
                umin = __reduce_min_sync(0xFFFFFFFFu, umin);
                umax = __reduce_max_sync(0xFFFFFFFFu, umax);
                for (int u = umin + lane; u <= umax; u += 32)
                    sh.xthr[u + kUBase] =
                        raw_threshold(__fsub_rn(__fmul_rn((float)(u - 1), 0.69314718f), 0.01f), inv_t, mx);
                if (lane == 0) {
                    sh.xhist = pathN ? raw_threshold(hist_lim, inv_t, mx) : kInf;
                    sh.bval = s0;
                    __threadfence_block();
                    sh.bseq = carry;  // first sum-live tile
                    if (carry < g.nchunks) mbar_arrive(&sh.bwait[carry % kWarps]);  // (release)
                }
            }
            csync();
            qbase += sh.ndense;
            lap(1);

            // -------------------------------------------------------- pass 2 ----
            // exact sequential softmax denominator in index order (ops.rs:408-411)
            float S = 0.0f;
            {
                const float xhist = sh.xhist;
                uint32_t bits_nx = 0;
                float lr_nx = 0.0f;
                float xs_nx[kRunS];      // next sparse tile: this lane's list entries (scaled logits)
                uint32_t i0_nx = 0;      // and the index of its first entry
                // loads of tile t's per-lane inputs, issued one tile ahead of their use
                auto prefetch = [&](uint32_t t) {
                    // dense tiles: penalty bits and lane sums; sparse tiles: the list entries
                    // (runs of ceil(entries / 32) <= kRunS entries, spread over the lanes)
                    const uint32_t lc = tt[t].lcnt;
                    const bool dn = lc == kDenseMark;
                    const uint32_t rs = dn ? 0u : (lc + 31u) >> 5, e0 = (uint32_t)lane * rs;
                    bits_nx = dn ? tile_bits(t) : 0u;
                    lr_nx = dn ? __ldcg(lrec + t * 64u + (uint32_t)lane) : 0.0f;
                    const bool want = !bad && lc != kDenseMark && (tt[t].flags & (kSumLive | kHistLive));
                    const uint2* en = lists + tt[t].loff;
#pragma unroll
                    for (int i = 0; i < kRunS; ++i)
                        xs_nx[i] = (want && (uint32_t)i < rs && e0 + (uint32_t)i < lc) ? __uint_as_float(__ldcg(&en[e0 + i].x)) : -kInf;
                    i0_nx = (want && e0 < lc) ? __ldcg(&en[e0].y) : 0u;
                };
                if ((uint32_t)warp < g.nchunks) prefetch((uint32_t)warp);
                for (uint32_t t = (uint32_t)warp; t < g.nchunks; t += kWarps) {
                    const bool dense = tt[t].lcnt == kDenseMark;
                    const uint32_t fl = bad ? 0u : tt[t].flags;
                    const uint32_t bits = bits_nx;  // this tile's penalty bits, lane sums, list entries
                    const float lr = lr_nx;
                    float xsv[kRunS];
#pragma unroll
                    for (int i = 0; i < kRunS; ++i) xsv[i] = xs_nx[i];
                    const uint32_t i0v = i0_nx;
                    if (t + kWarps < g.nchunks) prefetch(t + kWarps);
                    const bool sum_live = (fl & kSumLive) != 0u;
                    const bool hl = pathN && (fl & kHistLive) != 0u;
                    if (!dense && !sum_live && !hl) continue;  // nothing in this tile can matter
                    const uint32_t cnt = chunk_count(g, t);
                    const uint32_t tb = g.head + t * kTile;
                    const uint32_t l0 = (uint32_t)lane * 32u;
                    const int ulo = (int)(fl & 0xFFFFu) - 256;
                    const float thr_d = __fsub_rn(__fmul_rn((float)(ulo - 1), 0.69314718f), 0.01f);
                    const float xthr = sum_live ? sh.xthr[ulo + kUBase] : kInf;
                    const float ptile = tt[t].pt;
                    const uint32_t lcnt = dense ? 0u : tt[t].lcnt;
                    const uint32_t rs = (lcnt + 31u) >> 5;  // list entries per lane run (sparse)
                    uint32_t s = 0;
                    const float* slot = ring;
                    if (dense) {
                        const uint32_t qq = q2 + tt[t].rank;
                        s = qq % kSlots;
                        slot = ring + (size_t)s * kTile;
                        wait_full(sh, qq, a.err_flag);
                    }
                    // ---- this lane's run: its grid estimate and its increments on two grids
                    GridAcc acc{0.0f, 0.0f, false, false};
                    bool live = false;
                    int u0 = ulo;
                    float bm0 = 0.0f, bm1 = 0.0f, h0 = 0.0f, h1 = 0.0f;
                    bool one = false;  // the run is classified on grid u0 alone
                    auto set_grids = [&](float pl, uint32_t first_index) {
                        const float dl = __fmaf_rn((float)first_index, 1.1920929e-07f, 1.2207031e-04f);
                        u0 = max(unit_exp(__fmul_rn(pl, __fsub_rn(1.0f, dl))), ulo);
                        // an upper estimate (twice the margin: not a bound, a run that lands on
                        // another grid is summed element by element) in the same binade
                        one = unit_exp(__fmul_rn(pl, __fadd_rn(1.0f, __fadd_rn(dl, dl)))) == u0;
                        bm0 = grid_value(u0, kTwo23);
                        bm1 = __fadd_rn(bm0, bm0);
                        h0 = u0 > -149 ? pow2f(u0 - 1) : 0.0f;
                        h1 = pow2f(u0);
                    };
                    if (dense) {
                        // run = 32 consecutive elements of the staged tile
                        const uint32_t nval = l0 < cnt ? min(32u, cnt - l0) : 0u;
                        if (sum_live) {
                            // the running sum at the run start is within (1 +- delta) of its
                            // estimate, so it lies on grid u0 or u0 + 1
                            const float incl = warp_incl_scan_f(lr);
                            float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
                            if (lane == 0) excl = 0.0f;
                            const float scale = ex2_approx(__fmul_rn(__fsub_rn(tt[t].mt, mx), kLog2e));
                            set_grids(__fadd_rn(ptile, __fmul_rn(excl, scale)), tb + l0);
                        }
                        uint32_t lmask = 0;  // live run offsets
                        const float xlow = hl ? fminf(xthr, xhist) : xthr;
#pragma unroll 2
                        for (int j = 0; j < 8; ++j) {
                            const uint32_t c4 = (uint32_t)((j + lane) & 7) * 4u;
                            if (c4 >= nval) continue;
                            const float4 q = *reinterpret_cast<const float4*>(slot + l0 + c4);
                            float x[4] = {q.x, q.y, q.z, q.w};
                            const uint32_t pb = (bits >> c4) & 15u;
                            if (pb) {
#pragma unroll
                                for (int c = 0; c < 4; ++c)
                                    if ((pb >> c) & 1u) x[c] = penalise(x[c], penalty);
                            }
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                if (!(x[c] > xlow)) continue;
                                if (hl && x[c] > xhist)
                                    atomicAdd(&hcnt[(int)fminf(-d_of(x[c], inv_t, mx) * kBScale, (float)(kNB - 1))], 1u);
                                if (x[c] > xthr) lmask |= 1u << (c4 + c);
                            }
                        }
                        live = lmask != 0u;
                        // the live elements only, in a lane-rotated order (distinct banks);
                        // on grid u0 alone when every run of the warp allows it
                        const bool one_w = __all_sync(0xFFFFFFFFu, one);
                        lmask = __funnelshift_r(lmask, lmask, lane);
                        if (one_w) {
                            // two elements an iteration
                            while (lmask) {
                                const int pa = (__ffs(lmask) - 1 + lane) & 31;
                                lmask &= lmask - 1u;
                                const bool vb = lmask != 0u;
                                const int pb = vb ? (__ffs(lmask) - 1 + lane) & 31 : pa;
                                lmask &= lmask - 1u;
                                float xa = slot[l0 + (uint32_t)pa], xb = slot[l0 + (uint32_t)pb];
                                if ((bits >> pa) & 1u) xa = penalise(xa, penalty);
                                if (vb && ((bits >> pb) & 1u)) xb = penalise(xb, penalty);
                                classify_pair1(d_of(xa, inv_t, mx), vb ? d_of(xb, inv_t, mx) : -kInf, vb, bm0, h0, acc,
                                               exptab);
                            }
                            acc.sp1 = true;
                        } else {
                            while (lmask) {
                                const int pos = (__ffs(lmask) - 1 + lane) & 31;
                                lmask &= lmask - 1u;
                                float xv = slot[l0 + (uint32_t)pos];
                                if ((bits >> pos) & 1u) xv = penalise(xv, penalty);
                                classify_elem(d_of(xv, inv_t, mx), bm0, bm1, h0, h1, acc, exptab);
                            }
                        }
                    } else {
                        // run = rs consecutive list entries of the sparse tile (rs = ceil(lcnt / 32)
                        // <= kRunS: the live entries spread over as many lanes as there are)
                        const uint32_t e0 = (uint32_t)lane * rs;
                        float dv[kRunS];
                        float lsum = 0.0f;
#pragma unroll
                        for (int i = 0; i < kRunS; ++i) {
                            dv[i] = -kInf;
                            if ((uint32_t)i < rs && e0 + (uint32_t)i < lcnt) {
                                const float d = __fsub_rn(xsv[i], mx);
                                if (hl && d >= hist_lim) atomicAdd(&hcnt[(int)fminf(-d * kBScale, (float)(kNB - 1))], 1u);
                                if (sum_live && d >= thr_d) {
                                    dv[i] = d;
                                    lsum += ex2_approx(__fmul_rn(d, kLog2e));
                                }
                            }
                        }
                        if (sum_live) {
                            const float incl = warp_incl_scan_f(lsum);
                            float excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
                            if (lane == 0) excl = 0.0f;
                            set_grids(__fadd_rn(ptile, excl), e0 < lcnt ? i0v : tb);
                            const bool one_w = __all_sync(0xFFFFFFFFu, one);
                            // the live entries only (a few per lane), through shared memory: per
                            // warp [entry][lane] in the space of the path-K keys (unused until the finish)
                            float* const wlive = reinterpret_cast<float*>(smem_raw + kRingBytes + kRegionABytes +
                                                                          (size_t)kKCap * 8) +
                                                 (size_t)warp * 32 * kRunS;
                            uint32_t lmk = 0;
#pragma unroll
                            for (int i = 0; i < kRunS; ++i)
                                if (dv[i] != -kInf) {
                                    lmk |= 1u << i;
                                    wlive[i * 32 + lane] = dv[i];
                                }
                            live = lmk != 0u;
                            while (lmk) {
                                const int i = __ffs(lmk) - 1;
                                lmk &= lmk - 1u;
                                const float d = wlive[i * 32 + lane];
                                if (one_w)
                                    classify_elem1(d, bm0, h0, acc, exptab);
                                else
                                    classify_elem(d, bm0, bm1, h0, h1, acc, exptab);
                            }
                            if (one_w) acc.sp1 = true;
                        }
                    }
                    if (sum_live) {
                        // multiples of U summed in f32 are exact below 2^24 U; at or above it the
                        // run leaves the grid anyway (saturated count)
                        const uint32_t c0 = acc.s0 >= __fadd_rn(bm0, bm0) ? kSat : grid_units(acc.s0, -u0);
                        const uint32_t c1 = acc.s1 >= __fadd_rn(bm1, bm1) ? kSat : grid_units(acc.s1, -(u0 + 1));
                        // tile totals for the common case: every run classified on the same grids
                        const unsigned lm = __ballot_sync(0xFFFFFFFFu, live);
                        const int u0w = __shfl_sync(0xFFFFFFFFu, u0, lm ? __ffs(lm) - 1 : 0);
                        const bool uni = __all_sync(0xFFFFFFFFu, !live || u0 == u0w);
                        // (32 counts of at most 2^25 cannot wrap: one hardware sum, then saturate)
                        const uint32_t t0 = min(__reduce_add_sync(0xFFFFFFFFu, live ? c0 : 0u), kSat);
                        const uint32_t t1 = min(__reduce_add_sync(0xFFFFFFFFu, live ? c1 : 0u), kSat);
                        const bool any0 = __any_sync(0xFFFFFFFFu, live && acc.sp0);
                        const bool any1 = __any_sync(0xFFFFFFFFu, live && acc.sp1);
                        // ---- chain step: wait for the exact sum before this tile
                        // Lane 0 alone takes a step that is one add (the common case) and hands
                        // the baton on at once; the warp joins only for a walk over the runs.
                        float Sx = 0.0f;
                        bool done = false;
                        if (lane == 0) {
                            const uint32_t nx = tt[t].next;
                            // the message arrives on this warp's barrier (acquire on completion)
                            wait_bar(sh, &sh.bwait[warp], bcnt & 1u, a.err_flag);
                            ++bcnt;
                            Sx = sh.bval;
                            done = lm == 0u;
                            if (!done && uni) {
                                const int u = unit_exp(Sx);
                                const uint32_t A = grid_count(Sx, u);
                                if (u == u0w && !any0 && A + t0 < kTwo24) {
                                    Sx = grid_value(u, A + t0);
                                    done = true;
                                } else if (u == u0w + 1 && !any1 && A + t1 < kTwo24) {
                                    Sx = grid_value(u, A + t1);
                                    done = true;
                                }
                            }
                            if (done) {
                                sh.bval = Sx;
                                sh.bseq = nx;
                                if (nx < g.nchunks) mbar_arrive(&sh.bwait[nx % kWarps]);  // (release)
                            }
                        }
                        done = __shfl_sync(0xFFFFFFFFu, done, 0);
                        Sx = __shfl_sync(0xFFFFFFFFu, Sx, 0);
                        if (lane == 0 && !done && unit_exp(Sx) < ulo) sh.misc[7] = 1u;  // estimate bound broken
                        const bool walked = !done;
                        uint32_t p = 0;
                        for (int guard = 0; guard <= 32 && !done; ++guard) {
                            const int u = unit_exp(Sx);
                            const uint32_t A = grid_count(Sx, u);
                            const bool act = (uint32_t)lane >= p && live;
                            uint32_t inc = 0;
                            bool ev = false;
                            if (act) {
                                if (u == u0) {
                                    inc = c0;
                                    ev = acc.sp0;
                                } else if (u == u0 + 1) {
                                    inc = c1;
                                    ev = acc.sp1;
                                } else {
                                    ev = true;  // the run starts on a grid it was not classified for
                                }
                            }
                            const uint32_t incl_i = warp_incl_scan(inc);
                            uint32_t excl_i = __shfl_up_sync(0xFFFFFFFFu, incl_i, 1);
                            if (lane == 0) excl_i = 0u;  // (not incl - inc: a lane count may saturate)
                            ev = ev || (act && A + incl_i >= kTwo24);
                            const unsigned m = __ballot_sync(0xFFFFFFFFu, ev);
                            if (!m) {
                                Sx = grid_value(u, A + __shfl_sync(0xFFFFFFFFu, incl_i, 31));
                                break;
                            }
                            // runs before L on the grid, then run L element by element
                            const int L = __ffs(m) - 1;
                            Sx = grid_value(u, A + __shfl_sync(0xFFFFFFFFu, excl_i, L));
                            float e = 0.0f, de = 0.0f;
                            bool exe = true;
                            int len;
                            if (dense) {
                                const uint32_t bL = __shfl_sync(0xFFFFFFFFu, bits, L);
                                const uint32_t pos = (uint32_t)L * 32u + (uint32_t)lane;
                                len = 32;
                                if (pos < cnt) {
                                    float xv = slot[pos];
                                    if ((bL >> lane) & 1u) xv = penalise(xv, penalty);
                                    if (xv > xthr) {  // (at or below: adds exactly nothing on this grid)
                                        de = d_of(xv, inv_t, mx);
                                        exe = de == 0.0f;
                                        e = exe ? 1.0f : expf(de);
                                    }
                                }
                            } else {
                                len = (int)rs;
                                // run L's entries (lane L's prefetched scaled logits, -inf
                                // where absent) to lanes 0 .. rs-1
                                float xl = -kInf;
#pragma unroll
                                for (int i = 0; i < kRunS; ++i) {
                                    const float v = __shfl_sync(0xFFFFFFFFu, xsv[i], L);
                                    if (lane == i) xl = v;
                                }
                                const float d = __fsub_rn(xl, mx);
                                if (xl != -kInf && d >= thr_d) {
                                    de = d;
                                    exe = de == 0.0f;
                                    e = exe ? 1.0f : expf(de);
                                }
                            }
                            Sx = warp_serial_add(Sx, e, de, exe, 0, len, exptab);
                            if (lane == 0) atomicAdd(&sh.events, 1u);
                            p = (uint32_t)L + 1u;
                            if (p >= 32u) break;
                        }
                        if (lane == 0 && walked) {
                            const uint32_t nx = tt[t].next;
                            sh.bval = Sx;
                            sh.bseq = nx;
                            if (nx < g.nchunks) mbar_arrive(&sh.bwait[nx % kWarps]);  // (release)
                        }
                    }
                    if (dense) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sh.empty[s]);
                    }
                }
                csync();
                if (!bad && warp == 0) {
                    // the unaligned tail elements close the sum; head and tail into the buckets
                    const uint32_t edges = g.head + g.tail;
                    float et = 0.0f, dt = 0.0f, xe = -kInf;
                    bool ext = true;
                    if ((uint32_t)lane < edges) {
                        const uint32_t gi =
                            (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
                        xe = penal_g(g.row[gi], gi);
                        if ((uint32_t)lane >= g.head) {
                            dt = d_of(xe, inv_t, mx);
                            ext = dt == 0.0f;
                            et = ext ? 1.0f : expf(dt);
                        }
                    }
                    const float Sx = warp_serial_add(sh.bval, et, dt, ext, (int)g.head, (int)g.tail, exptab);
                    if (pathN && xe > xhist)
                        atomicAdd(&hcnt[(int)fminf(-d_of(xe, inv_t, mx) * kBScale, (float)(kNB - 1))], 1u);
                    if (lane == 0) sh.fstate = Sx;
                }
                csync();
                S = sh.fstate;
            }
            if (tid == 0) inf.sum_exp = S;
            lap(2);
            if (tid == 0 && pathK) sh.claim_ok = rqi;  // a short finish remains: the producer may claim
            if (bad) {
                status = LRS_E_NAN;
                token = LRS_TOKEN_NONE;
                prob = 0.0f;
                goto row_done;
            }

            const float inv = __fdiv_rn(1.0f, S);  // ops.rs:413
            FinishCtx fc;
            fc.g = g;
            fc.tt = tt;
            fc.lists = lists;
            fc.lmax = lrec + 32;
            fc.scratch = scratch;
            fc.bitmap = bitmap;
            fc.hcnt = hcnt;
            fc.hoff = hoff;
            fc.cursor = cursor;
            fc.sbuf = sbuf;
            fc.ring = ring;
            fc.err = a.err_flag;
            fc.cand_x = cand_x;
            fc.cand_i = cand_i;
            fc.keys = keys;
            fc.exptab = exptab;
            fc.k = k;
            fc.nk = nk;
            fc.mx = mx;
            fc.inv_t = inv_t;
            fc.inv = inv;
            fc.S = S;
            fc.penalty = penalty;
            fc.top_p = P.top_p;
            fc.hist_lim = hist_lim;
            fc.pen_on = pen_on;
            fc.topp_on = topp_on;
            fc.st = st;
            fc.cutoff = fc.pos = fc.n_cand = 0;
            fc.sum = fc.rr = fc.r0 = 0.0f;
            fc.chosen = 0;
            fc.acc_sort = 0;
            if (pathK)
                finish_path_k(sh, fc);
            else
                finish_path_n(sh, fc);
            st = fc.st;
            acc_sort = fc.acc_sort;
            if (tid == 0) {
                inf.n_cand = fc.n_cand;
                inf.r0 = fc.r0;
            }
            advance_state = true;
            token = (uint32_t)(fc.chosen & 0xFFFFFFFFu);
            prob = __uint_as_float(~(uint32_t)(fc.chosen >> 32));
            if (tid == 0) {
                inf.cutoff = fc.cutoff;
                inf.pos = fc.pos;
                inf.surv_sum = fc.sum;
            }
            lap(3);
        }

    row_done:
        if (sh.misc[7]) status = LRS_E_INTERNAL;
        if (sh.abort) status = LRS_E_TIMEOUT;
        if (tid == 0) {
            sh.claim_ok = rqi;
            inf.status = status;
            inf.token = token;
            inf.prob = prob;
            inf.events = sh.events;
            inf.cycles[7] = sat32(acc_sort);
            if (status == LRS_OK && advance_state) a.state[r] = st;
            a.tokens[r] = token;
            if (a.probs) a.probs[r] = prob;
            if (a.status) a.status[r] = status;
            if (a.info) a.info[r] = inf;
            if (status == LRS_E_INTERNAL) atomicExch(a.err_flag, LRS_E_INTERNAL);
        }
        if (pen_on && n > 0)
            for (uint32_t j = hstart + tid; j < hlen; j += kThreads) {
                const uint32_t t = hrow[j];
                if (t < n) bitmap[t >> 5] = 0u;
            }
        csync();
    }
}

// --------------------------------------------------------------- row order ----
// The claim order of a launch: rows by estimated cost, longest first (list scheduling of
// rows of unequal length over the persistent CTAs ends sooner when the rows left for the
// end are the short ones).  The cost grows with the temperature (more elements can change
// the exact softmax sum) and with a path-N finish; one-pass rows (greedy) are cheapest.
// Key: 32 temperature bands from 1.5 down to 0.5 (hotter and NaN in band 0, colder in
// band 31) times the two finishes, then the one-pass rows.  One block, a counting sort
// in shared memory; the order inside a key is free (rows are independent).
constexpr int kOrderThreads = 1024;
constexpr uint32_t kOrderKeys = 65;
__device__ __forceinline__ uint32_t order_key(const lrs_params& P, uint32_t n) {
    if (row_passes(P, n) != 2u) return kOrderKeys - 1;
    const uint32_t k = (P.top_k == 0 || P.top_k > n) ? n : P.top_k;
    const bool long_finish = !(k < n && k <= (uint32_t)kKMax);
    const float f = (1.5f - P.temperature) * 32.0f;
    const uint32_t band = !(f > 0.0f) ? 0u : f >= 31.0f ? 31u : (uint32_t)f;
    return band * 2u + (long_finish ? 0u : 1u);
}
__global__ void __launch_bounds__(kOrderThreads) lrs_order_rows(const lrs_params* __restrict__ params, uint32_t rows,
                                                                 uint32_t n, uint32_t* __restrict__ order) {
    __shared__ uint32_t cnt[kOrderKeys];
    for (uint32_t i = threadIdx.x; i < kOrderKeys; i += blockDim.x) cnt[i] = 0u;
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) atomicAdd(&cnt[order_key(params[r], n)], 1u);
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t acc = 0;
        for (uint32_t i = 0; i < kOrderKeys; ++i) {
            const uint32_t c = cnt[i];
            cnt[i] = acc;
            acc += c;
        }
    }
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) order[atomicAdd(&cnt[order_key(params[r], n)], 1u)] = r;
}

#include "lrs_stages.cuh"

}  // namespace lrs

// ------------------------------------------------------------------ host side ----
size_t lrs_kernel_smem_bytes() { return lrs::kDynSmem; }
int lrs_kernel_block_threads() { return lrs::kBlock; }
void lrs_kernel_scratch_layout(uint32_t n, uint64_t* stride, uint64_t* bitmap_off, uint64_t* tiles_off,
                               uint64_t* lanes_off, uint64_t* lists_off) {
    const uint64_t words = (uint64_t)(n + 31) / 32 + 2;  // window bitmap (+ read-ahead word)
    const uint64_t tiles = (uint64_t)n / lrs::kTile + 2;
    const uint64_t wtiles = (tiles + lrs::kWarps - 1) / lrs::kWarps;  // tiles of one consumer warp
    *bitmap_off = n;                                     // [0, n): path-N candidate keys
    *tiles_off = *bitmap_off + (words + 1) / 2;          // tile records, 32 bytes each
    *lanes_off = *tiles_off + 4 * tiles;                 // lane sums and lane maxima, 64 floats per tile
    *lists_off = *lanes_off + 32 * tiles;                // candidate lists, 8 bytes an entry
    *stride = (*lists_off + (uint64_t)lrs::kWarps * wtiles * lrs::kDense + 31) & ~(uint64_t)31;
}
cudaError_t lrs_kernel_set_smem(size_t bytes) {
    return cudaFuncSetAttribute(lrs::lrs_sample_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}
cudaError_t lrs_kernel_occupancy(int* ctas_per_sm, size_t smem) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, lrs::lrs_sample_rows, lrs::kBlock, smem);
}
cudaError_t lrs_kernel_launch(const lrs_kernel_args_t* args, uint32_t grid, size_t smem, cudaStream_t s) {
    cudaError_t e = lrs_kernel_set_smem(smem);
    if (e != cudaSuccess) return e;
    if (args->order && !args->claim_count) {
        lrs::lrs_order_rows<<<1, lrs::kOrderThreads, 0, s>>>(args->params, args->rows, args->n, args->order);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    lrs::lrs_sample_rows<<<grid, lrs::kBlock, smem, s>>>(*args);
    return cudaGetLastError();
}

void lrs_stage_layout(uint32_t rows, uint32_t vocab, lrs_stage_layout_t* L) {
    const uint64_t R = rows ? rows : 1, nt = (uint64_t)(vocab + lrs::kTile - 1) / lrs::kTile + 1;
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = (off + bytes + 255) & ~(uint64_t)255;
        return o;
    };
    L->rows = (uint32_t)R;
    L->nt = (uint32_t)nt;
    L->tstat = take(R * nt * sizeof(float4));
    L->lmax = take(R * nt * 32 * sizeof(float));
    L->tprep = take(R * nt * sizeof(lrs::TilePrep));
    L->tres = take(R * nt * sizeof(lrs::TileRes));
    L->rprep = take(R * sizeof(lrs::RowPrep));
    L->lists = take(R * lrs::kStageListCap * sizeof(uint2));
    L->list_n = take(R * sizeof(uint32_t));
    L->fb_rows = take(R * sizeof(uint32_t));
    L->fb_count = take(sizeof(uint32_t));
    L->live_count = take(sizeof(uint32_t));
    L->big_rows = take(R * sizeof(uint32_t));
    L->big_count = take(sizeof(uint32_t));
    L->big_claim = take(sizeof(uint32_t));
    L->bytes = off;
}

cudaError_t lrs_stage_launch(const lrs_kernel_args_t* args, void* mem, const lrs_stage_layout_t* L,
                             uint32_t fallback_grid, size_t smem, cudaStream_t s) {
    using namespace lrs;
    static int warps_grid[2] = {0, 0};  // persistent grids of the two per-tile stages (blocks)
    if (!warps_grid[0]) {
        int dev = 0, sms = 0, occ0 = 0, occ1 = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ0, lrs_stage_stats, kStageThreads, 0);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, lrs_stage_classify, kClassifyWarps * 32, 0);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(lrs_stage_finish, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kStageFinishSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(lrs_stage_big, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBigSmem);
        if (e != cudaSuccess) return e;
        warps_grid[0] = sms * (occ0 > 0 ? occ0 : 1);
        warps_grid[1] = sms * (occ1 > 0 ? occ1 : 1);
    }
    const uint32_t rows = args->rows;
    char* base = static_cast<char*>(mem);
    StageArgs S;
    S.a = *args;
    S.nt = L->nt;
    S.tstat = reinterpret_cast<float4*>(base + L->tstat);
    S.lmax = reinterpret_cast<float*>(base + L->lmax);
    S.tprep = reinterpret_cast<TilePrep*>(base + L->tprep);
    S.tres = reinterpret_cast<TileRes*>(base + L->tres);
    S.rprep = reinterpret_cast<RowPrep*>(base + L->rprep);
    S.lists = reinterpret_cast<uint2*>(base + L->lists);
    S.list_n = reinterpret_cast<uint32_t*>(base + L->list_n);
    S.fb_rows = reinterpret_cast<uint32_t*>(base + L->fb_rows);
    S.fb_count = reinterpret_cast<uint32_t*>(base + L->fb_count);
    S.live_count = reinterpret_cast<uint32_t*>(base + L->live_count);
    const bool big = args->scratch != nullptr && fallback_grid > 0u;  // (lrs_stage_big's scratch)
    S.big_rows = big ? reinterpret_cast<uint32_t*>(base + L->big_rows) : nullptr;
    S.big_count = reinterpret_cast<uint32_t*>(base + L->big_count);
    S.big_claim = reinterpret_cast<uint32_t*>(base + L->big_claim);
    // (the stats stage zeroes the step's counters and the lists' lengths)
    cudaError_t e;
    lrs_stage_stats<<<warps_grid[0], kStageThreads, 0, s>>>(S);
    lrs_stage_prep<<<rows, kStageThreads, 0, s>>>(S);
    lrs_stage_classify<<<warps_grid[1], kClassifyWarps * 32, 0, s>>>(S);
    lrs_stage_sum<<<(rows + kSumWarps - 1) / kSumWarps, kSumWarps * 32, 0, s>>>(S);
    lrs_stage_finish<<<rows, kThreads, kStageFinishSmem, s>>>(S);
    if (big) lrs_stage_big<<<fallback_grid, kThreads, kBigSmem, s>>>(S);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // the rows the stages left: lrs_sample_rows on the list, in list order
    lrs_kernel_args_t fb = *args;
    fb.order = S.fb_rows;
    fb.claim_count = S.fb_count;
    return lrs_kernel_launch(&fb, fallback_grid, smem, s);
}

cudaError_t lrs_wait_probe_launch(int32_t* err, long long bound, cudaStream_t s) {
    lrs::lrs_wait_probe<<<1, 32, 0, s>>>(err, bound);
    return cudaGetLastError();
}
