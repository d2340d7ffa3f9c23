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
__device__ __forceinline__ void block_incl_scan(const uint32_t (&inc)[kVpt], uint32_t (&incl)[kVpt],
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
    uint32_t off = 0;
    for (int i = 0; i < w; ++i) off = sat_add(off, sh[i]);
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
__device__ int acc_tile(float (&v)[kVpt], uint32_t& exact, int cnt, int dir, float& s, float thr,
                        Exactify exactify, RowShared& sh) {
    int consumed = -1;
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
#pragma unroll
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
                    if (lo.inc == hi.inc && !lo.tie && !hi.tie && !lo.big && !hi.big) {
                        c = lo;
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
        block_incl_scan(inc, incl, sh.red);
        uint32_t first = 0xFFFFFFFFu;
#pragma unroll
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
#pragma unroll
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

// All-ascending bitonic sort of n 64-bit keys (n <= cap, cap a power of two >= n is
// not required: virtual +inf padding).  `keys` in shared or global memory.
__device__ void bitonic_sort_u64(unsigned long long* keys, uint32_t n) {
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
__device__ uint32_t radix_select_desc(const float* x, uint32_t cnt, uint32_t kk, RowShared& sh) {
    uint32_t prefix = 0;
    for (int round = 0; round < 4; ++round) {
        const int shift = 24 - 8 * round;
        for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.hist256[i] = 0;
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
            const uint32_t key = fkey(x[i]);
            const bool match = (round == 0) || ((key >> (shift + 8)) == (prefix >> (shift + 8)));
            if (match) atomicAdd(&sh.hist256[(key >> shift) & 255u], 1u);
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
__device__ void compact_candidates(float* cx, uint32_t* ci, uint32_t k, float mrun, RowShared& sh) {
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

// ------------------------------------------------------------------- the kernel ----
extern "C" __global__ void __launch_bounds__(kThreads, 2) lrs_sample_rows(SampleArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ RowShared sh;
    __shared__ float wsh[kWarps];
    __shared__ float gvs[kWarps];
    __shared__ uint32_t gis[kWarps];
    __shared__ float etile[4];
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
        auto xs_of = [&](float x, uint32_t gi) -> float { return __fmul_rn(penal(x, gi), inv_t); };

        if (n == 0) goto row_done;  // sampler.rs:57-60

        {
            // -------------------------------------------------------- pass 1 ----
            float bv = -kInf;
            uint32_t bi = 0xFFFFFFFFu;
            float mx = -kInf;
            float theta = -kInf;
            auto p1_elem = [&](float x, uint32_t gi, bool active) {
                if (greedy) {
                    if (active) {
                        const float xp = penal(x, gi);
                        if (xp > bv || (xp == bv && gi < bi)) {
                            bv = xp;
                            bi = gi;
                        }
                    }
                } else {
                    float xs = 0.0f;
                    if (active) {
                        xs = xs_of(x, gi);
                        mx = fmax_nan(mx, xs);
                    }
                    if (pathK) {
                        const bool hit = active && xs >= theta;
                        const unsigned m = __ballot_sync(0xFFFFFFFFu, hit);
                        if (m) {
                            const int leader = __ffs(m) - 1;
                            uint32_t base = 0;
                            if (lane == leader) base = atomicAdd(&sh.cand_n, (uint32_t)__popc(m));
                            base = __shfl_sync(0xFFFFFFFFu, base, leader);
                            if (hit) {
                                const uint32_t slot = base + __popc(m & ((1u << lane) - 1u));
                                if (slot < (uint32_t)kKCap) {
                                    cand_x[slot] = xs;
                                    cand_i[slot] = gi;
                                } else {
                                    sh.cand_over = 1;
                                }
                            }
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
                    x = g.row[gi];
                }
                p1_elem(x, gi, mine);
            }
            __syncthreads();
            for (uint32_t c = 0; c < g.nchunks; ++c) {
                const int stage = ring_wait(sh, a, seq, timed_out);
                const float* slot = ring + (size_t)stage * kChunk;
                const uint32_t cnt = chunk_count(g, c);
                const uint32_t gbase = g.head + c * kChunk;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int li0 = li_of(j * 4);
                    const bool act = (uint32_t)li0 < cnt;
                    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (act) q = *reinterpret_cast<const float4*>(slot + li0);
                    p1_elem(q.x, gbase + li0 + 0, act);
                    p1_elem(q.y, gbase + li0 + 1, act);
                    p1_elem(q.z, gbase + li0 + 2, act);
                    p1_elem(q.w, gbase + li0 + 3, act);
                }
                __syncthreads();
                ++seq;
                if (tid == 0) ring_issue(sh, ring, g, first_load, total_loads, seq);
                if (pathK) {
                    if (sh.cand_over) {
                        pathK = false;
                    } else if (sh.cand_n > (uint32_t)(kKCap - kChunk)) {
                        const float mb = block_max_nan(mx, wsh);
                        compact_candidates(cand_x, cand_i, k, mb, sh);
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
                goto row_done;
            }

            // ---------------------------------------------- stochastic rows ----
            mx = block_max_nan(mx, wsh);
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
            __syncthreads();

            // -------------------------------------------------------- pass 2 ----
            // exact sequential softmax denominator in index order (ops.rs:408-411)
            float S = 0.0f;
            auto s_tile = [&](const float* src, uint32_t cnt, uint32_t gbase) {
                float v[kVpt];
                uint32_t exact = 0;
                const int uu0 = unit_exp(S);
                // e < U/2 adds nothing to S now or later in the row (U only grows)
                const float thr_skip = pathN ? -kInf : (float)(uu0 - 1) * 0.69314718f - 0.01f;
#pragma unroll
                for (int i = 0; i < kVpt; ++i) {
                    const int li = li_of(i);
                    v[i] = 0.0f;
                    if ((uint32_t)li < cnt) {
                        const float dd = __fsub_rn(xs_of(src[li], gbase + li), mx);
                        if (dd < thr_skip) {
                            exact |= 1u << i;
                        } else {
                            if (dd == 0.0f) {
                                v[i] = 1.0f;
                                exact |= 1u << i;
                            } else {
                                v[i] = expf(dd);
                            }
                            if (pathN) {
                                const int b = (int)fminf(-dd * kBScale, (float)(kNB - 1));
                                atomicAdd(&hcnt[b], 1u);
                                atomicAdd(&hmass[b], v[i]);
                            }
                        }
                    }
                }
                auto exf = [&](int i) -> float {
                    const int li = li_of(i);
                    return exact_expf(__fsub_rn(xs_of(src[li], gbase + li), mx), exptab);
                };
                acc_tile(v, exact, (int)cnt, +1, S, kInf, exf, sh);
            };
            if (!bad && g.head) {
                if (tid < 4) etile[tid] = tid < (int)g.head ? g.row[tid] : 0.0f;
                __syncthreads();
                s_tile(etile, g.head, 0);
                __syncthreads();
            }
            for (uint32_t c = 0; c < g.nchunks; ++c) {
                const int stage = ring_wait(sh, a, seq, timed_out);
                const float* slot = ring + (size_t)stage * kChunk;
                if (!bad) s_tile(slot, chunk_count(g, c), g.head + c * kChunk);
                __syncthreads();
                ++seq;
                if (tid == 0) ring_issue(sh, ring, g, first_load, total_loads, seq);
            }
            if (!bad && g.tail) {
                const uint32_t tb = g.head + (uint32_t)g.body;
                if (tid < 4) etile[tid] = tid < (int)g.tail ? g.row[tb + tid] : 0.0f;
                __syncthreads();
                s_tile(etile, g.tail, tb);
                __syncthreads();
            }
            inf.sum_exp = S;
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
            bool drew = false;
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
                bitonic_sort_u64(keys, nk);  // (p desc, index asc)
                inf.n_cand = nk;
                float v[kVpt];
                uint32_t ex = 0xFFFFFFFFu;
                load_sorted_tile(keys, k, v);
                float cum = 0.0f;
                auto noex = [&](int i) -> float { return v[i]; };
                int stp = acc_tile(v, ex, (int)k, +1, cum, topp_on ? P.top_p : kInf, noex, sh);
                cutoff = stp >= 0 ? (uint32_t)stp + 1 : k;  // sampler.rs:135-146
                sum = cum;                                   // sampler.rs:148-151 (same sequence)
                if (sum > 0.0f) {
                    rr = __fmul_rn(next_f32(&st), sum);      // sampler.rs:155
                    inf.r0 = rr;
                    float w[kVpt];
                    uint32_t ex2 = 0xFFFFFFFFu;
                    load_sorted_tile(keys, cutoff, w);
                    auto noex2 = [&](int i) -> float { return w[i]; };
                    stp = acc_tile(w, ex2, (int)cutoff, -1, rr, 0.0f, noex2, sh);
                    pos = stp >= 0 ? (uint32_t)stp : cutoff - 1;  // sampler.rs:156-162
                    drew = true;
                } else {
                    pos = 0;  // sampler.rs:152-154
                }
                chosen = keys[pos];
                __syncthreads();
            } else {
                // -------------------------------------------------------- path N ----
                if (tid == 0) {
                    uint32_t cc = 0;
                    double mass = 0.0;
                    const double target = topp_on ? ((double)P.top_p + kTopPMargin) * (double)S : 1e300;
                    uint32_t b = 0;
                    for (; b < (uint32_t)kNB; ++b) {
                        cc += hcnt[b];
                        mass += (double)hmass[b];
                        if (cc >= k || mass >= target) break;
                    }
                    sh.misc[3] = b < (uint32_t)kNB ? b : (uint32_t)(kNB - 1);
                    uint32_t acc = 0;
                    for (int q = 0; q < kNB; ++q) {
                        hoff[q] = acc;
                        acc += hcnt[q];
                    }
                }
                __syncthreads();
                const uint32_t blim = sh.misc[3];
                uint32_t* cursor = reinterpret_cast<uint32_t*>(hmass);
                for (int q = tid; q < kNB; q += kThreads) cursor[q] = 0;
                __syncthreads();
                // gather exact probabilities of buckets [blo, bhi] into scratch
                auto gather = [&](uint32_t blo, uint32_t bhi) {
                    for (uint32_t i = tid; i < n; i += kThreads) {
                        const float dd = __fsub_rn(xs_of(g.row[i], i), mx);
                        const int b = (int)fminf(-dd * kBScale, (float)(kNB - 1));
                        if ((uint32_t)b >= blo && (uint32_t)b <= bhi) {
                            const float e = exact_expf(dd, exptab);
                            const float p = __fmul_rn(e, inv);
                            const uint32_t slot = hoff[b] + atomicAdd(&cursor[b], 1u);
                            scratch[slot] = ((unsigned long long)(~__float_as_uint(p)) << 32) | i;
                        }
                    }
                    __threadfence_block();
                    __syncthreads();
                };
                gather(0, blim);
                uint32_t gathered_to = blim;
                inf.n_cand = hoff[blim] + hcnt[blim];
                unsigned long long* sbuf = reinterpret_cast<unsigned long long*>(ring);
                auto sort_bucket = [&](uint32_t b) {
                    const uint32_t cnt = hcnt[b];
                    unsigned long long* base = scratch + hoff[b];
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
                };
                // top-p scan over sorted buckets, capped at k survivors (sampler.rs:122-146)
                float cum = 0.0f;
                uint32_t done = 0;
                bool stopped = false;
                uint32_t sorted_to = 0;
                for (uint32_t b = 0; b < (uint32_t)kNB && !stopped && done < k; ++b) {
                    if (b > gathered_to) {
                        gather(gathered_to + 1, kNB - 1);
                        gathered_to = kNB - 1;
                    }
                    const uint32_t cnt = hcnt[b];
                    sorted_to = b + 1;
                    if (cnt == 0) continue;
                    sort_bucket(b);
                    const unsigned long long* base = scratch + hoff[b];
                    for (uint32_t t0 = 0; t0 < cnt && !stopped && done < k; t0 += kChunk) {
                        uint32_t tc = min((uint32_t)kChunk, cnt - t0);
                        if (tc > k - done) tc = k - done;
                        float v[kVpt];
                        uint32_t ex = 0xFFFFFFFFu;
                        load_sorted_tile(base + t0, tc, v);
                        auto noex = [&](int i) -> float { return v[i]; };
                        const int stp = acc_tile(v, ex, (int)tc, +1, cum, topp_on ? P.top_p : kInf, noex, sh);
                        if (stp >= 0) {
                            stopped = true;
                            done += (uint32_t)stp + 1;
                        } else {
                            done += tc;
                        }
                    }
                }
                cutoff = done;
                sum = cum;
                // draw (sampler.rs:152-162)
                if (sum > 0.0f) {
                    rr = __fmul_rn(next_f32(&st), sum);
                    inf.r0 = rr;
                    drew = true;
                }
                uint32_t seen = 0;
                bool found = false;
                for (uint32_t b = 0; b < (uint32_t)kNB && !found && seen < cutoff; ++b) {
                    const uint32_t cnt = hcnt[b];
                    if (cnt == 0) continue;
                    if (b >= sorted_to) {
                        if (b > gathered_to) {
                            gather(gathered_to + 1, kNB - 1);
                            gathered_to = kNB - 1;
                        }
                        sort_bucket(b);
                        sorted_to = b + 1;
                    }
                    const unsigned long long* base = scratch + hoff[b];
                    for (uint32_t t0 = 0; t0 < cnt && !found && seen < cutoff; t0 += kChunk) {
                        uint32_t tc = min((uint32_t)kChunk, cnt - t0);
                        if (tc > cutoff - seen) tc = cutoff - seen;
                        if (!drew) {  // sum <= 0: the first survivor (sampler.rs:152-154)
                            found = true;
                            pos = 0;
                            chosen = base[t0];
                            break;
                        }
                        float v[kVpt];
                        uint32_t ex = 0xFFFFFFFFu;
                        load_sorted_tile(base + t0, tc, v);
                        auto noex = [&](int i) -> float { return v[i]; };
                        const int stp = acc_tile(v, ex, (int)tc, -1, rr, 0.0f, noex, sh);
                        if (stp >= 0) {
                            found = true;
                            pos = seen + (uint32_t)stp;
                            chosen = base[t0 + stp];
                        } else {
                            chosen = base[t0 + tc - 1];
                            seen += tc;
                        }
                    }
                }
                if (!found) pos = cutoff - 1;  // sampler.rs:162: the last survivor
                __syncthreads();
            }
            (void)drew;
            advance_state = true;
            token = (uint32_t)(chosen & 0xFFFFFFFFu);
            prob = __uint_as_float(~(uint32_t)(chosen >> 32));
            inf.cutoff = cutoff;
            inf.pos = pos;
            inf.surv_sum = sum;
        }

    row_done:
        if (sh.misc[7]) status = LRS_E_INTERNAL;
        if (timed_out) status = LRS_E_TIMEOUT;
        if (tid == 0) {
            inf.status = status;
            inf.token = token;
            inf.prob = prob;
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
