// lrs_kernels.cu — the batched token-sampling kernel (sm_100a).
//
// Computes, for every row, exactly what rust-llama's Sampler::sample computes
// (src/sampler.rs:56-163 with ops::softmax_inplace, src/ops.rs:397-419):
//   greedy fast path (sampler.rs:62-70), windowed once-per-token repetition penalty
//   (sampler.rs:82-102), greedy after penalty (104-113), temperature (115-118),
//   softmax (ops.rs:397-419), top-k (122-132), top-p (135-146), survivor sum (148-151)
//   and the categorical draw with the row's xorshift64* state (152-162).
//
// Structure: a persistent CTA (two per SM) takes rows from a global counter.  A row
// is streamed through a 3-stage ring of 16 KB bulk copies (TMA engine, mbarrier
// completion) twice: pass 1 reads it from HBM (L2 evict_last) for the max / argmax
// and a streaming top-k candidate filter; pass 2 re-reads it from L2 (evict_first)
// and computes the softmax denominator with the exact sequential-f32 emulation of
// lrs_device.cuh.  The top-k / top-p / draw phase then works on candidates only:
//   path K (top_k <= kKMax): candidates from the pass-1 filter, sorted in shared memory;
//   path N (top_k off or large): candidates bucketed by (max - x) during pass 2,
//          gathered with exact probabilities into global scratch and sorted bucket by
//          bucket in shared memory as the top-p scan and the draw reach them.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/llamars_sampler.h"
#include "lrs_device.cuh"
#include "lrs_kernels_decl.cuh"

namespace lrs {

constexpr int kKMax = 256;          // path K handles 1 <= k <= kKMax (k < n)
constexpr int kKCap = 4608;         // path K candidate buffer (entries)
constexpr int kKSortMax = 2048;     // path K candidates kept after the final compaction
constexpr int kNB = 2048;           // path N buckets of width 1/32 in (max - x)
constexpr float kBScale = 32.0f;
constexpr int kSortCap = 4096;      // largest bucket sorted in shared memory
constexpr float kTopPMargin = 0.002f;
constexpr int kSerial = 512;        // elements summed one by one at the start of a row or scan
constexpr unsigned long long kWaitLimit = 1ull << 26;

using SampleArgs = lrs_kernel_args_t;

// ---------------------------------------------------------------- shared state ----
struct RowShared {
    uint64_t bar[kStages];
    uint32_t red[kWarps + 2];
    uint32_t red2[kWarps + 2];
    float fstate;          // running exact value broadcast
    int32_t stop;          // stop position broadcast
    uint32_t cand_n;
    uint32_t cand_over;
    float theta;
    float delta_min;
    uint32_t hist256[256];
    uint32_t row;
    uint32_t issued;       // ring loads issued so far (thread 0)
    float vk;              // k-th largest scaled logit at the last compaction
    uint32_t events;       // ordered steps taken by acc_tile for this row
    uint32_t ev_base0, ev_base1;  // tile2: prefixes at the last ordered step
    float xthr;            // pass-2 skip threshold on (penalised) raw logits
    int xthr_uu;           // grid exponent xthr was computed for
    uint32_t misc[8];
};

struct Geo {
    const float* row;
    uint32_t n, head, tail, nchunks;
    uint64_t body;  // elements in the aligned body
};

__device__ __forceinline__ Geo row_geometry(const SampleArgs& a, uint32_t r) {
    Geo g;
    g.row = a.logits + (uint64_t)r * a.ld;
    g.n = a.n;
    const uintptr_t p = (uintptr_t)g.row;
    uint32_t head = (uint32_t)(((16u - (uint32_t)(p & 15u)) & 15u) >> 2);
    if (head > g.n) head = g.n;
    g.head = head;
    g.body = ((uint64_t)(g.n - head) / 4u) * 4u;
    g.tail = g.n - head - (uint32_t)g.body;
    g.nchunks = (uint32_t)((g.body + kChunk - 1) / kChunk);
    return g;
}

__device__ __forceinline__ uint32_t chunk_count(const Geo& g, uint32_t c) {
    const uint64_t left = g.body - (uint64_t)c * kChunk;
    return (uint32_t)(left < (uint64_t)kChunk ? left : (uint64_t)kChunk);
}

// ---------------------------------------------------------------- ring pipeline ----
// Loads of one row are numbered in consumption order: chunk c of pass p is the row's
// load p * nchunks + c; `first` is the CTA-wide number of the row's first load.  Load q
// lands in stage q % kStages and completes phase (q / kStages) & 1 of that stage's
// mbarrier.  Called by thread 0 only; issues while fewer than kStages loads are pending.
__device__ __forceinline__ void ring_issue(RowShared& s, float* ring, const Geo& g, uint32_t first,
                                           uint32_t total, uint32_t consumed) {
    while (s.issued < first + total && s.issued - consumed < (uint32_t)kStages) {
        const uint32_t local = s.issued - first;
        const uint32_t pass = local / g.nchunks, c = local % g.nchunks;
        const uint32_t stage = s.issued % kStages;
        const uint32_t bytes = chunk_count(g, c) * 4u;
        const float* src = g.row + g.head + (uint64_t)c * kChunk;
        fence_proxy_async_smem();
        mbar_expect_tx(&s.bar[stage], bytes);
        bulk_load(ring + (size_t)stage * kChunk, src, bytes, &s.bar[stage],
                  pass == 0 ? policy_evict_last() : policy_evict_first());
        s.issued++;
    }
}

// Wait (bounded) until load number q has landed; returns its stage.
__device__ __forceinline__ int ring_wait(RowShared& s, const SampleArgs& a, uint32_t q, bool& timed_out) {
    const uint32_t stage = q % kStages;
    const uint32_t parity = (q / kStages) & 1u;
    unsigned long long it = 0;
    while (!mbar_try_wait(&s.bar[stage], parity)) {
        if (++it > kWaitLimit) {
            timed_out = true;
            atomicExch(a.err_flag, LRS_E_TIMEOUT);
            break;
        }
    }
    return (int)stage;
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
    __syncthreads();
    if (l == 0) sh[w] = wt;
    __syncthreads();
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
        __syncthreads();
        cur = sh.fstate;
        const int st = sh.stop;
        __syncthreads();
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
        __syncthreads();
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
    for (int i = 0; i < cnt; ++i) {
        cur = dir > 0 ? __fadd_rn(cur, vals[i]) : __fsub_rn(cur, vals[i]);
        if (dir > 0 ? cur >= thr : cur <= 0.0f) {
            s = cur;
            return i;
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
            for (uint32_t t = threadIdx.x; t < P / 2; t += blockDim.x) {
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
            __syncthreads();
        }
    }
}

// k-th largest key (1-based rank kk) among keys[0..cnt) by radix select.
__device__ __noinline__ uint32_t radix_select_desc(const float* x, uint32_t cnt, uint32_t kk, RowShared& sh) {
    uint32_t prefix = 0;
    for (int round = 0; round < 4; ++round) {
        const int shift = 24 - 8 * round;
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.hist256[i] = 0;
        __syncthreads();
        for (uint32_t i0 = 0; i0 < cnt; i0 += blockDim.x) {
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
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t acc = 0;
            int d = 255;
            for (; d >= 0; --d) {
                const uint32_t c = sh.hist256[d];
                if (acc + c >= kk) break;
                acc += c;
            }
            if (d < 0) d = 0;
            sh.misc[1] = (uint32_t)d;
            sh.misc[2] = kk - acc;
        }
        __syncthreads();
        prefix |= sh.misc[1] << shift;
        kk = sh.misc[2];
        __syncthreads();
    }
    return prefix;
}

// Margin below the k-th value inside which probabilities may tie (see DESIGN notes in
// the host documentation): distinct scaled logits closer than this can round to the
// same probability.
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
    __syncthreads();
    if (threadIdx.x == 0) sh.cand_n = 0;
    __syncthreads();
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
    __syncthreads();
}


// Block-wide max of a per-thread value (NaN-propagating).
__device__ __forceinline__ float block_max_nan(float m, float* wsh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) wsh[threadIdx.x >> 5] = m;
    __syncthreads();
    float r = wsh[0];
    for (int w = 1; w < kWarps; ++w) r = fmax_nan(r, wsh[w]);
    return r;
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

// Penalise in place the elements of a staged tile (ids [gbase, gbase + cnt)) whose id
// is in the row's window (sampler.rs:82-102): x > 0 ? x / p : x * p, once per id.
__device__ __forceinline__ void patch_tile(float* t, uint32_t gbase, uint32_t cnt, const uint32_t* bitmap,
                                           float penalty) {
    const uint32_t w0 = gbase >> 5, w1 = (gbase + cnt - 1) >> 5;
    for (uint32_t w = w0 + threadIdx.x; w <= w1; w += kThreads) {
        uint32_t bits = bitmap[w];
        while (bits) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            const uint32_t gi = (w << 5) + (uint32_t)b;
            if (gi >= gbase && gi < gbase + cnt) {
                const float x = t[gi - gbase];
                t[gi - gbase] = x > 0.0f ? __fdiv_rn(x, penalty) : __fmul_rn(x, penalty);
            }
        }
    }
}

// The scaled, shifted logit d = fl(fl(x * inv_t) - max) of sampler.rs:117 / ops.rs:409.
__device__ __forceinline__ float d_of(float x, float inv_t, float mx) { return __fsub_rn(__fmul_rn(x, inv_t), mx); }

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

// ------------------------------------------------------------------- the kernel ----
extern "C" __global__ void __launch_bounds__(kThreads, 2) lrs_sample_rows(SampleArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ RowShared sh;
    __shared__ float wsh[kWarps];
    __shared__ float gvs[kWarps];
    __shared__ uint32_t gis[kWarps];
    __shared__ float red_f[kWarps];
    __shared__ uint32_t red_u[kWarps];
    __shared__ __align__(16) float etile[4];
    float* ring = reinterpret_cast<float*>(smem_raw);
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + (size_t)kStages * kChunk * 4);
    unsigned char* area = smem_raw + (size_t)kStages * kChunk * 4 + (size_t)a.bitmap_words * 4;
    float* cand_x = reinterpret_cast<float*>(area);
    uint32_t* cand_i = reinterpret_cast<uint32_t*>(area + kKCap * 4);
    uint32_t* hcnt = reinterpret_cast<uint32_t*>(area);            // path N bucket counts
    float* hmass = reinterpret_cast<float*>(area + kNB * 4);       // path N bucket mass, then cursors
    uint32_t* hoff = reinterpret_cast<uint32_t*>(area + kNB * 8);  // path N bucket offsets
    unsigned long long* scratch = a.scratch + (uint64_t)blockIdx.x * a.scratch_stride;
    const ExpTable exptab{a.exp_index, a.exp_entries};
    const float kInf = __int_as_float(0x7F800000);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&sh.bar[i], 1);
        fence_barrier_init();
        sh.issued = 0;
    }
    for (uint32_t i = tid; i < a.bitmap_words; i += kThreads) bitmap[i] = 0;
    __syncthreads();
    uint32_t seq = 0;  // ring loads consumed by this CTA (same value in every thread)

    for (;;) {
        if (tid == 0) sh.row = atomicAdd(a.row_counter, 1u);
        __syncthreads();
        const uint32_t r = sh.row;
        __syncthreads();
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

        lrs_row_info inf;
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
        long long t_mark = clock64();
        auto sat32 = [](long long d) -> uint32_t { return d > 0xFFFFFFFFll ? 0xFFFFFFFFu : (d < 0 ? 0u : (uint32_t)d); };
        auto lap = [&](uint32_t& field) {
            const long long now = clock64();
            field = sat32(now - t_mark);
            t_mark = now;
        };
        long long acc_wait = 0, acc_ord = 0, acc_thr = 0, acc_wait1 = 0, acc_sort = 0, acc_loop = 0, acc_red = 0;
        int32_t status = LRS_OK;
        uint32_t token = 0;
        float prob = 1.0f;
        bool timed_out = false;
        bool advance_state = false;

        const bool need_pass2 = stochastic && n >= 2;
        const uint32_t total_loads = n == 0 ? 0u : g.nchunks * (need_pass2 ? 2u : 1u);
        const uint32_t first_load = seq;
        if (tid == 0) {
            ring_issue(sh, ring, g, first_load, total_loads, seq);
            sh.cand_n = 0;
            sh.cand_over = 0;
            sh.theta = -kInf;
            sh.delta_min = kInf;
            sh.vk = -kInf;
            sh.misc[7] = 0;
            sh.events = 0;
            sh.xthr_uu = 1000;
            sh.misc[5] = 0;
            sh.misc[6] = 0;
        }
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
        __syncthreads();

        const float inv_t = stochastic ? __fdiv_rn(1.0f, temperature) : 1.0f;  // sampler.rs:115
        auto penal = [&](float x, uint32_t gi) -> float {                     // sampler.rs:96-100
            if (pen_on && ((bitmap[gi >> 5] >> (gi & 31)) & 1u))
                return x > 0.0f ? __fdiv_rn(x, penalty) : __fmul_rn(x, penalty);
            return x;
        };

        if (n == 0) goto row_done;  // sampler.rs:57-60

        {
            // -------------------------------------------------------- pass 1 ----
            // greedy: argmax (lowest index among maximal values); stochastic: NaN-aware
            // max of the scaled logits and, on path K, the streaming top-k filter.
            float bv = -kInf;
            uint32_t bi = 0xFFFFFFFFu;
            float mx = -kInf;
            float theta = -kInf;
            auto p1_value = [&](float x, uint32_t gi, bool act, bool& hit) {
                if (greedy) {
                    if (act && (x > bv || (x == bv && gi < bi))) {
                        bv = x;
                        bi = gi;
                    }
                    hit = false;
                } else {
                    const float xs = __fmul_rn(x, inv_t);
                    if (act) mx = fmax_nan(mx, xs);
                    hit = act && xs >= theta;
                }
            };
            auto p1_append = [&](float x, uint32_t gi, bool hit) {
                const unsigned m = __ballot_sync(0xFFFFFFFFu, hit);
                if (m) {
                    const int leader = __ffs(m) - 1;
                    uint32_t base = 0;
                    if (lane == leader) base = atomicAdd(&sh.cand_n, (uint32_t)__popc(m));
                    base = __shfl_sync(0xFFFFFFFFu, base, leader);
                    if (hit) {
                        const uint32_t slot = base + __popc(m & ((1u << lane) - 1u));
                        if (slot < (uint32_t)kKCap) {
                            cand_x[slot] = __fmul_rn(x, inv_t);
                            cand_i[slot] = gi;
                        } else {
                            sh.cand_over = 1;
                        }
                    }
                }
            };
            // unaligned head and tail elements, plain loads, warp 0
            if (tid < 32) {
                const uint32_t edges = g.head + g.tail;
                const bool mine = (uint32_t)tid < edges;
                uint32_t gi = 0;
                float x = 0.0f;
                if (mine) {
                    gi = (uint32_t)tid < g.head ? (uint32_t)tid : g.head + (uint32_t)g.body + ((uint32_t)tid - g.head);
                    x = penal(g.row[gi], gi);
                }
                bool hit;
                p1_value(x, gi, mine, hit);
                if (pathK) p1_append(x, gi, hit);
            }
            __syncthreads();
            for (uint32_t c = 0; c < g.nchunks; ++c) {
                const int stage = ring_wait(sh, a, seq, timed_out);
                float* slot = ring + (size_t)stage * kChunk;
                const uint32_t cnt = chunk_count(g, c);
                const uint32_t gbase = g.head + c * kChunk;
                if (pen_on) {
                    patch_tile(slot, gbase, cnt, bitmap, penalty);
                    __syncthreads();
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int li0 = li_of(j * 4);
                    const bool act = (uint32_t)li0 < cnt;
                    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (act) q = *reinterpret_cast<const float4*>(slot + li0);
                    const uint32_t gi = gbase + (uint32_t)li0;
                    bool h0, h1, h2, h3;
                    p1_value(q.x, gi + 0, act, h0);
                    p1_value(q.y, gi + 1, act, h1);
                    p1_value(q.z, gi + 2, act, h2);
                    p1_value(q.w, gi + 3, act, h3);
                    if (pathK && __any_sync(0xFFFFFFFFu, h0 | h1 | h2 | h3)) {
                        p1_append(q.x, gi + 0, h0);
                        p1_append(q.y, gi + 1, h1);
                        p1_append(q.z, gi + 2, h2);
                        p1_append(q.w, gi + 3, h3);
                    }
                }
                __syncthreads();
                ++seq;
                if (tid == 0) ring_issue(sh, ring, g, first_load, total_loads, seq);
                if (pathK) {
                    if (sh.cand_over) {
                        pathK = false;
                    } else if (sh.cand_n > (uint32_t)(kKCap - kChunk)) {
                        const long long tc0 = clock64();
                        const float mb = block_max_nan(mx, wsh);
                        compact_candidates(cand_x, cand_i, k, mb, sh);
                        acc_wait1 += clock64() - tc0;
                        if (sh.cand_n > (uint32_t)(kKCap - kChunk)) pathK = false;
                    }
                    theta = sh.theta;
                    __syncthreads();
                }
            }

            if (greedy) {
                // lowest index among the maximal non-NaN values; NaN at index 0 -> 0
                // (sampler.rs:62-70 and 104-113: strict '>' scanning up from index 0)
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
                    gvs[tid >> 5] = bv;
                    gis[tid >> 5] = bi;
                }
                __syncthreads();
                float b = gvs[0];
                uint32_t ix = gis[0];
                for (int w = 1; w < kWarps; ++w)
                    if (gvs[w] > b || (gvs[w] == b && gis[w] < ix)) {
                        b = gvs[w];
                        ix = gis[w];
                    }
                const float x0 = penal(g.row[0], 0);
                if (x0 != x0 || ix == 0xFFFFFFFFu) ix = 0;
                token = ix;
                prob = 1.0f;
                lap(inf.cycles[0]);
                goto row_done;
            }

            // ---------------------------------------------- stochastic rows ----
            mx = block_max_nan(mx, wsh);
            lap(inf.cycles[0]);
            inf.max = mx;
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
                compact_candidates(cand_x, cand_i, k, mx, sh);
                if (sh.cand_over || sh.cand_n > (uint32_t)kKSortMax) pathK = false;
                // candidates dropped at earlier compactions must lie below every
                // probability tie of the final k-th value
                if (pathK && sh.delta_min < kInf && tie_margin(sh.vk, mx) > 4.0f * sh.delta_min) pathK = false;
                __syncthreads();
            }
            const uint32_t nk = sh.cand_n;
            const bool pathN = !pathK;
            if (pathN && !bad)
                for (int i = tid; i < kNB; i += kThreads) {
                    hcnt[i] = 0;
                    hmass[i] = 0.0f;
                }
            // raw threshold of the path-N histogram: elements with d >= -kNB/kBScale
            const float xhist = (pathN && !bad) ? raw_threshold(-(float)(kNB - 1) / kBScale, inv_t, mx) : kInf;
            __syncthreads();

            // -------------------------------------------------------- pass 2 ----
            // exact sequential softmax denominator in index order (ops.rs:408-411)
            float S = 0.0f;
            auto count_bucket = [&](float x, bool live) {
                // path N: warp-aggregated count of the element's (max - x) bucket
                const bool c = pathN && live && x >= xhist;
                const unsigned act = __ballot_sync(0xFFFFFFFFu, c);
                if (c) {
                    const int b = (int)fminf(-d_of(x, inv_t, mx) * kBScale, (float)(kNB - 1));
                    const unsigned peers = __match_any_sync(act, b);
                    if (lane == __ffs(peers) - 1) atomicAdd(&hcnt[b], (uint32_t)__popc(peers));
                }
            };
            // One tile of values src[li], li in [start, cnt) (local positions = index order).
            auto s_tile = [&](const float* src, uint32_t cnt, uint32_t gbase, uint32_t start) {
                const int uu = unit_exp(S);
                if (uu != sh.xthr_uu) {
                    // elements with e < U/2 add nothing to S at this grid or any later one
                    const long long t0 = clock64();
                    __syncthreads();
                    if (tid == 0) {
                        sh.xthr = raw_threshold((float)(uu - 1) * 0.69314718f - 0.01f, inv_t, mx);
                        sh.xthr_uu = uu;
                    }
                    __syncthreads();
                    acc_thr += clock64() - t0;
                }
                const float xthr = sh.xthr;
                const long long t_start = clock64();
                const float bm = grid_value(uu, kTwo23);                      // magic base 2^23 * U
                const float halfu = uu > -149 ? ldexpf(1.0f, uu - 1) : 0.0f;  // U / 2
                float v[kVpt];
#pragma unroll
                for (int i = 0; i < kVpt; ++i) v[i] = 0.0f;
                uint32_t exact = 0xFFFFFFFFu;  // bit i clear: v[i] approximates libm's expf
                float tot = 0.0f;
                uint32_t nlive = 0;
                uint32_t flags = 0;  // 1: tie or big element on the current grid
                uint32_t live = 0;  // bit i: slot i is above the skip threshold
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int li0 = li_of(j * 4);
                    float4 q = make_float4(-kInf, -kInf, -kInf, -kInf);
                    if ((uint32_t)li0 < cnt && (uint32_t)li0 >= start) {  // start, body cnt: multiples of 4
                        q = *reinterpret_cast<const float4*>(src + li0);
                        if ((uint32_t)li0 + 1 >= cnt) q.y = -kInf;  // edge tiles hold < 4 values
                        if ((uint32_t)li0 + 2 >= cnt) q.z = -kInf;
                        if ((uint32_t)li0 + 3 >= cnt) q.w = -kInf;
                    }
                    if (pathN) {
                        count_bucket(q.x, q.x != -kInf);
                        count_bucket(q.y, q.y != -kInf);
                        count_bucket(q.z, q.z != -kInf);
                        count_bucket(q.w, q.w != -kInf);
                    }
                    live |= (q.x > xthr ? 1u : 0u) << (j * 4);
                    live |= (q.y > xthr ? 2u : 0u) << (j * 4);
                    live |= (q.z > xthr ? 4u : 0u) << (j * 4);
                    live |= (q.w > xthr ? 8u : 0u) << (j * 4);
                }
#pragma unroll 1
                while (live) {
                    const int i = __ffs(live) - 1;
                    live &= live - 1;
                    ++nlive;
                    const float x = src[li_of(i)];
                    const float d = d_of(x, inv_t, mx);
                    float e = d == 0.0f ? 1.0f : expf(d);
                    bool ex = d == 0.0f;
                    if (e >= bm) {
                        flags = 1;  // big: ordered step
                    } else if (halfu > 0.0f) {
                        float inc = __fsub_rn(__fadd_rn(bm, e), bm);
                        float rr = fabsf(__fsub_rn(e, inc));
                        if (!ex && rr >= halfu - __fmul_rn(e, 4.76837158203125e-07f)) {  // 2^-21 > 2.5 ulp
                            // near a rounding midpoint: take libm's exact value
                            e = exact_expf(d, exptab);
                            ex = true;
                            inc = __fsub_rn(__fadd_rn(bm, e), bm);
                            rr = fabsf(__fsub_rn(e, inc));
                            if (e >= bm) flags = 1;
                        }
                        if (ex && rr == halfu) flags = 1;  // tie: parity decides
                        tot = __fadd_rn(tot, inc);
                    } else {
                        tot = __fadd_rn(tot, e);  // unit 2^-149: every float below 2^-125 is on the grid
                    }
                    v[i] = e;
                    if (!ex) exact &= ~(1u << i);
                }
                const long long t_loop = clock64();
                acc_loop += t_loop - t_start;
                if (nlive) atomicAdd(&sh.misc[6], nlive);
                // one reduction of (sum, flags)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    tot = __fadd_rn(tot, __shfl_xor_sync(0xFFFFFFFFu, tot, o));
                    flags |= __shfl_xor_sync(0xFFFFFFFFu, flags, o);
                }
                __syncthreads();
                if (lane == 0) {
                    red_f[tid >> 5] = tot;
                    red_u[tid >> 5] = flags;
                }
                __syncthreads();
                float T = red_f[0];
                uint32_t F = red_u[0];
                for (int w = 1; w < kWarps; ++w) {
                    T = __fadd_rn(T, red_f[w]);
                    F |= red_u[w];
                }
                acc_red += clock64() - t_loop;
                if (!F) {
                    // every increment is a multiple of U below 2^23 U: the float sum is exact
                    // whenever the new value stays below the grid's top
                    const float s2 = __fadd_rn(S, T);
                    if (s2 < __fadd_rn(bm, bm)) {
                        S = s2;
                        return;
                    }
                }
                // a grid change, a tie or a big element inside the tile
                auto exf = [&](int i) -> float {
                    const int li = li_of(i);
                    return exact_expf(d_of(src[li], inv_t, mx), exptab);
                };
                const long long t0 = clock64();
                tile2(v, exact, (int)start, (int)cnt, +1, S, kInf, exf, sh);
                acc_ord += clock64() - t0;
            };
            __shared__ float ser[kSerial + 4];
            // Serial start: the head elements and the first kSerial elements of the first
            // body tile, where the running sum crosses many binades, are added one by one
            // by thread 0 after all threads computed their exact exps.
            auto serial_start = [&](const float* body, uint32_t nbody) {
                const uint32_t nh = g.head;
                for (uint32_t q = tid; q < nh + nbody; q += kThreads) {
                    const float x = q < nh ? penal(g.row[q], q) : body[q - nh];
                    const float d = d_of(x, inv_t, mx);
                    ser[q] = d == 0.0f ? 1.0f : exact_expf(d, exptab);
                }
                __syncthreads();
                if (tid == 0) {
                    float s = 0.0f;
                    (void)serial_run(ser, (int)(nh + nbody), +1, s, kInf);
                    sh.fstate = s;
                }
                __syncthreads();
                S = sh.fstate;
                __syncthreads();
            };
            if (!bad && g.nchunks == 0) serial_start(nullptr, 0);
            for (uint32_t c = 0; c < g.nchunks; ++c) {
                const long long tw = clock64();
                const int stage = ring_wait(sh, a, seq, timed_out);
                acc_wait += clock64() - tw;
                float* slot = ring + (size_t)stage * kChunk;
                const uint32_t cnt = chunk_count(g, c);
                const uint32_t gbase = g.head + c * kChunk;
                if (!bad) {
                    if (pen_on) {
                        patch_tile(slot, gbase, cnt, bitmap, penalty);
                        __syncthreads();
                    }
                    uint32_t start = 0;
                    if (c == 0) {
                        start = min(cnt, (uint32_t)kSerial);
                        serial_start(slot, start);
                        // serial elements are still counted for the path-N histogram
                        if (pathN)
                            for (uint32_t q0 = 0; q0 < start; q0 += kThreads) {
                                const uint32_t q = q0 + tid;
                                count_bucket(q < start ? slot[q] : 0.0f, q < start);
                            }
                    }
                    s_tile(slot, cnt, gbase, start);
                }
                __syncthreads();
                ++seq;
                if (tid == 0) ring_issue(sh, ring, g, first_load, total_loads, seq);
            }
            if (!bad && g.tail) {
                const uint32_t tb = g.head + (uint32_t)g.body;
                if (tid < 4) etile[tid] = tid < (int)g.tail ? penal(g.row[tb + tid], tb + tid) : 0.0f;
                __syncthreads();
                s_tile(etile, g.tail, tb, 0);
                __syncthreads();
            }
            if (!bad && pathN && g.head)  // head elements into the histogram
                if (tid < 32) count_bucket(tid < (int)g.head ? penal(g.row[tid], tid) : 0.0f, tid < (int)g.head);
            inf.sum_exp = S;
            lap(inf.cycles[1]);
            if (bad) {
                status = LRS_E_NAN;
                token = LRS_TOKEN_NONE;
                prob = 0.0f;
                goto row_done;
            }

            const float inv = __fdiv_rn(1.0f, S);  // ops.rs:413
            float sum = 0.0f;
            uint32_t cutoff = 0, pos = 0;
            unsigned long long chosen = 0;
            float rr = 0.0f;
            if (pathK) {
                // -------------------------------------------------------- path K ----
                unsigned long long* keys = reinterpret_cast<unsigned long long*>(ring);
                for (uint32_t i = tid; i < nk; i += kThreads) {
                    const float e = exact_expf(__fsub_rn(cand_x[i], mx), exptab);
                    const float p = __fmul_rn(e, inv);
                    keys[i] = ((unsigned long long)(~__float_as_uint(p)) << 32) | cand_i[i];
                }
                __syncthreads();
                const long long ts = clock64();
                bitonic_sort_u64(keys, nk);  // (p desc, index asc)
                acc_sort += clock64() - ts;
                inf.n_cand = nk;
                for (uint32_t i = tid; i < k; i += kThreads) ser[i] = __uint_as_float(~(uint32_t)(keys[i] >> 32));
                __syncthreads();
                if (tid == 0) {
                    // top-p over the first k (sampler.rs:135-146); the survivor sum is the
                    // same sequence up to the cutoff (sampler.rs:148-151)
                    float cum = 0.0f;
                    const int stp = serial_run(ser, (int)k, +1, cum, topp_on ? P.top_p : kInf);
                    const uint32_t cut = stp >= 0 ? (uint32_t)stp + 1 : k;
                    uint32_t ps = 0;
                    float r0 = 0.0f;
                    unsigned long long st2 = st;
                    if (cum > 0.0f) {
                        r0 = __fmul_rn(next_f32(&st2), cum);  // sampler.rs:155
                        float r = r0;
                        const int w = serial_run(ser, (int)cut, -1, r, 0.0f);
                        ps = w >= 0 ? (uint32_t)w : cut - 1;  // sampler.rs:156-162
                    }
                    sh.misc[3] = cut;
                    sh.misc[4] = ps;
                    sh.fstate = cum;
                    sh.vk = r0;
                }
                __syncthreads();
                cutoff = sh.misc[3];
                pos = sh.misc[4];
                sum = sh.fstate;
                rr = sh.vk;
                if (sum > 0.0f) {
                    (void)next_f32(&st);
                    inf.r0 = rr;
                }
                chosen = keys[pos];
                __syncthreads();
            } else {
                // -------------------------------------------------------- path N ----
                if (tid == 0) {
                    // bucket limit: enough candidates for k and for top_p (+ margin); the
                    // mass of bucket b is at least count * exp(-(b+1)/kBScale) / S
                    uint32_t cc = 0;
                    double mass = 0.0;
                    const double target = topp_on ? ((double)P.top_p + kTopPMargin) * (double)S : 1e300;
                    uint32_t b = 0;
                    for (; b < (uint32_t)kNB - 1; ++b) {
                        cc += hcnt[b];
                        mass += (double)hcnt[b] * exp(-(double)(b + 1) / (double)kBScale);
                        if (cc >= k || mass >= target) break;
                    }
                    sh.misc[3] = b;
                    uint32_t acc = 0;
                    for (int q = 0; q < kNB - 1; ++q) {
                        hoff[q] = acc;
                        acc += hcnt[q];
                    }
                    hoff[kNB - 1] = acc;
                    hcnt[kNB - 1] = n - acc;  // everything below the histogram range
                }
                __syncthreads();
                const uint32_t blim = sh.misc[3];
                uint32_t* cursor = reinterpret_cast<uint32_t*>(hmass);
                for (int q = tid; q < kNB; q += kThreads) cursor[q] = 0;
                __syncthreads();
                // gather exact probabilities of buckets [blo, bhi] into scratch
                auto gather = [&](uint32_t blo, uint32_t bhi) {
                    const float xlo = raw_threshold(-(float)(bhi + 1) / kBScale, inv_t, mx);
                    constexpr int kU = 4;  // independent elements per thread in flight
                    for (uint32_t i0 = 0; i0 < n; i0 += kThreads * kU) {
                        float xs[kU];
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            const uint32_t i = i0 + u * kThreads + tid;
                            xs[u] = i < n ? g.row[i] : -kInf;
                        }
#pragma unroll
                        for (int u = 0; u < kU; ++u) {
                            const uint32_t i = i0 + u * kThreads + tid;
                            bool take = false;
                            int b = 0;
                            float dd = 0.0f;
                            if (i < n) {
                                const float x = penal(xs[u], i);
                                if (x > xlo || bhi == (uint32_t)kNB - 1) {
                                    dd = d_of(x, inv_t, mx);
                                    b = (int)fminf(-dd * kBScale, (float)(kNB - 1));
                                    if (!(x >= xhist)) b = kNB - 1;
                                    take = (uint32_t)b >= blo && (uint32_t)b <= bhi;
                                }
                            }
                            const unsigned act = __ballot_sync(0xFFFFFFFFu, take);
                            if (take) {
                                const float e = exact_expf(dd, exptab);
                                const float pr = __fmul_rn(e, inv);
                                const unsigned peers = __match_any_sync(act, b);
                                const int leader = __ffs(peers) - 1;
                                uint32_t base = 0;
                                if (lane == leader) base = atomicAdd(&cursor[b], (uint32_t)__popc(peers));
                                base = __shfl_sync(act, base, leader);
                                const uint32_t slot = hoff[b] + base + __popc(peers & ((1u << lane) - 1u));
                                scratch[slot] = ((unsigned long long)(~__float_as_uint(pr)) << 32) | i;
                            }
                        }
                    }
                    __threadfence_block();
                    __syncthreads();
                };
                gather(0, blim);
                uint32_t gathered_to = blim;
                inf.n_cand = hoff[blim] + hcnt[blim];
                unsigned long long* sbuf = reinterpret_cast<unsigned long long*>(ring);
                uint32_t sorted_to = 0;  // buckets [0, sorted_to) sorted in scratch
                // Sort bucket b (gathering more buckets first when b is beyond the gathered
                // range, doubling the range each time).  Buckets are sorted in order.
                auto ensure_bucket = [&](uint32_t b) {
                    while (sorted_to <= b) {
                        const uint32_t q = sorted_to;
                        if (q > gathered_to) {
                            const uint32_t hi = min((uint32_t)kNB - 1, gathered_to + 1 + 2 * (gathered_to + 1));
                            gather(gathered_to + 1, hi);
                            gathered_to = hi;
                        }
                        const uint32_t cnt = hcnt[q];
                        if (cnt > 1) {
                            const long long ts = clock64();
                            unsigned long long* base = scratch + hoff[q];
                            if (cnt <= (uint32_t)kSortCap) {
                                for (uint32_t i = tid; i < cnt; i += kThreads) sbuf[i] = base[i];
                                __syncthreads();
                                bitonic_sort_u64(sbuf, cnt);
                                for (uint32_t i = tid; i < cnt; i += kThreads) base[i] = sbuf[i];
                            } else {
                                bitonic_sort_u64(base, cnt);  // rare: one bucket larger than shared memory
                            }
                            __threadfence_block();
                            __syncthreads();
                            acc_sort += clock64() - ts;
                        }
                        ++sorted_to;
                    }
                };
                auto pval = [&](uint32_t q) -> float { return __uint_as_float(~(uint32_t)(scratch[q] >> 32)); };
                // Exact sequential run over sorted positions [0, p1) of the candidate sequence
                // (buckets in order, each sorted when reached): the first kSerial positions
                // one by one on thread 0, then tiles.  Returns the stop position or -1.
                auto run = [&](uint32_t p1, int dir, float& s, float thr) -> int {
                    uint32_t p = 0, b = 0;
                    uint32_t serial_left = kSerial;
                    while (p < p1) {
                        while (b + 1 < (uint32_t)kNB && hoff[b] + hcnt[b] <= p) ++b;
                        if (dir > 0) {
                            // Every remaining candidate lies in bucket b or a later one; once
                            // their probabilities are all below half the sum's grid unit no
                            // later addition changes the sum (and none is a tie).
                            const float emax = expf(-(float)b / kBScale) * 1.0001f;
                            const float pmax = __fmul_rn(emax, inv) * 1.0001f;
                            const int uu = unit_exp(s);
                            if (uu > -149 && pmax < ldexpf(1.0f, uu - 1)) return -1;
                        }
                        ensure_bucket(b);
                        const uint32_t seg_end = min(p1, hoff[b] + hcnt[b]);
                        if (serial_left > 0) {
                            const uint32_t m = min(seg_end - p, serial_left);
                            for (uint32_t q = tid; q < m; q += kThreads) ser[q] = pval(p + q);
                            __syncthreads();
                            if (tid == 0) {
                                float s2 = s;
                                sh.stop = serial_run(ser, (int)m, dir, s2, thr);
                                sh.fstate = s2;
                            }
                            __syncthreads();
                            s = sh.fstate;
                            const int st0 = sh.stop;
                            __syncthreads();
                            if (st0 >= 0) return (int)p + st0;
                            p += m;
                            serial_left -= m;
                            continue;
                        }
                        const uint32_t tc = min((uint32_t)kChunk, seg_end - p);
                        float v[kVpt];
                        uint32_t ex = 0xFFFFFFFFu;
                        load_sorted_tile(scratch + p, tc, v);
                        // single-grid fast check
                        const int uu = unit_exp(s);
                        const uint32_t A = grid_count(s, uu);
                        uint32_t t = 0, f = 0;
#pragma unroll
                        for (int i = 0; i < kVpt; ++i) {
                            if ((uint32_t)li_of(i) < tc) {
                                const Cls c = classify(__float_as_uint(v[i]), uu);
                                t = sat_add(t, c.inc);
                                f |= (c.tie || c.big) ? 1u : 0u;
                            }
                        }
                        t = block_reduce_u32(t, SatAdd(), sh.red);
                        f = block_reduce_u32(f, OrOp(), sh.red2);
                        const float tq = (dir > 0 && thr < kInf) ? ldexpf(thr, -uu) : kInf;
                        const bool fast = dir > 0 ? (!f && A + t <= kTwo24 - 1u && (float)(A + t) < tq)
                                                  : (!f && t < A - grid_lower(uu));
                        if (fast) {
                            s = grid_value(uu, dir > 0 ? A + t : A - t);
                        } else {
                            const int stp = tile2(v, ex, 0, (int)tc, dir, s, thr, NoExact(), sh);
                            if (stp >= 0) return (int)p + stp;
                        }
                        p += tc;
                    }
                    return -1;
                };
                // top-p scan capped at k survivors (sampler.rs:122-146)
                float cum = 0.0f;
                int stp = run(k, +1, cum, topp_on ? P.top_p : kInf);
                cutoff = stp >= 0 ? (uint32_t)stp + 1 : k;
                sum = cum;
                // draw (sampler.rs:152-162)
                if (sum > 0.0f) {
                    rr = __fmul_rn(next_f32(&st), sum);
                    inf.r0 = rr;
                    float r = rr;
                    stp = run(cutoff, -1, r, 0.0f);
                    pos = stp >= 0 ? (uint32_t)stp : cutoff - 1;
                } else {
                    pos = 0;
                }
                {
                    uint32_t b = 0;
                    while (b + 1 < (uint32_t)kNB && hoff[b] + hcnt[b] <= pos) ++b;
                    ensure_bucket(b);
                }
                chosen = scratch[pos];
                __syncthreads();
            }
            advance_state = true;
            token = (uint32_t)(chosen & 0xFFFFFFFFu);
            prob = __uint_as_float(~(uint32_t)(chosen >> 32));
            inf.cutoff = cutoff;
            inf.pos = pos;
            inf.surv_sum = sum;
            lap(inf.cycles[2]);
        }

    row_done:
        if (sh.misc[7]) status = LRS_E_INTERNAL;
        if (timed_out) status = LRS_E_TIMEOUT;
        if (tid == 0) {
            inf.status = status;
            inf.token = token;
            inf.prob = prob;
            inf.events = sh.events;
            inf.cycles[3] = sat32(acc_wait1);
            inf.cycles[4] = sat32(acc_ord);
            inf.cycles[6] = sat32(acc_loop);
            inf.reserved = sat32(acc_red) / 16u * 0 + sh.misc[5];
            inf.cycles[5] = sat32(acc_red);
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
                if (t < n) bitmap[t >> 5] = 0;
            }
        __syncthreads();
    }
}

}  // namespace lrs

// ------------------------------------------------------------------ host side ----
size_t lrs_kernel_ring_bytes() { return (size_t)lrs::kStages * lrs::kChunk * sizeof(float); }
size_t lrs_kernel_area_bytes() {
    const size_t k = (size_t)lrs::kKCap * 8, nb = (size_t)lrs::kNB * 12;
    return k > nb ? k : nb;
}
cudaError_t lrs_kernel_set_smem(size_t bytes) {
    return cudaFuncSetAttribute(lrs::lrs_sample_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}
cudaError_t lrs_kernel_occupancy(int* ctas_per_sm, size_t smem) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, lrs::lrs_sample_rows, lrs::kThreads, smem);
}
cudaError_t lrs_kernel_launch(const lrs_kernel_args_t* args, uint32_t grid, size_t smem, cudaStream_t s) {
    cudaError_t e = lrs_kernel_set_smem(smem);
    if (e != cudaSuccess) return e;
    lrs::lrs_sample_rows<<<grid, lrs::kThreads, smem, s>>>(*args);
    return cudaGetLastError();
}
