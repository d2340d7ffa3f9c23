// lrs_stages.cuh — the staged sampling pipeline (sm_100a), included by lrs_kernels.cu.
//
// The same computation as lrs_sample_rows (rust-llama src/sampler.rs:56-163 with
// ops::softmax_inplace, src/ops.rs:397-419), split into five launches whose work items
// are independent, so that every SM streams, classifies or finishes whatever is ready
// instead of one CTA carrying one row through every phase:
//
//   stats     one warp per tile (1024 floats) of every row: the tile's max of the scaled
//             logits x' = fl(pen(x) * inv_t) (sampler.rs:82-118), its sum of exp relative to
//             that max (approximate, for estimates only), the 32 lane maxima, and for greedy
//             rows the argmax (sampler.rs:62-70, 104-113).
//   prep      one CTA per row: the row max M; greedy rows and rows whose probabilities are
//             NaN finish here.  From the tile statistics, an estimate P_t of the sequential
//             softmax sum at every tile start with a proven relative error bound, hence the
//             lowest binade grid the exact sum can be on there (dead elements below it add
//             exactly nothing) and the two grids a tile is classified on.  The candidate
//             threshold of the finish: from the k-th largest lane maximum for top-k (k <= 128),
//             or for top-p alone a depth below M that holds the nucleus's mass.
//   classify  one warp per tile: the increments of the tile's live elements on its two
//             grids (lrs_grid.h), per block of 128 elements, and the candidates appended to
//             the row's list.
//   sum       one warp per row: the exact running sum in tile order, a tile in one step
//             where the sum stays on a grid it was classified for, else block by block,
//             walking element by element only a block where the sum crosses a binade or
//             meets a tie or an element of half a binade.
//   finish    one CTA per row: the candidates' exact probabilities, sorted (p desc, index
//             asc), the top-p cut, survivor sum and draw (sampler.rs:122-162).
//
// Rows the stages do not take (top-p off with top-k off or above kKMax, rows longer than
// kStageMaxTiles tiles, a top-k list overflowing with ties, a nucleus larger than the list
// capacity) are flagged and sampled by lrs_sample_rows afterwards, from the same inputs
// (its results are the same bits).
//
// Tile layout in registers: lane L holds elements 128 j + 4 L + c (block j = 0..7, c = 0..3)
// of the tile, so every warp-wide 16-byte load is one contiguous 512-byte block.

constexpr int kStageThreads = 256;                 // stats / prep / classify blocks (8 warps)
constexpr int kStageWarps = kStageThreads / 32;
constexpr uint32_t kStageListCap = 8192;           // candidate-list entries per row
// the finish's dynamic shared memory: the keys, then the sort's two 16-bit permutations
constexpr size_t kStageFinishSmem = kStageListCap * sizeof(unsigned long long) + 2 * kStageListCap * sizeof(uint16_t);
constexpr int kStageNucleusBuckets = 580;          // mass buckets of width 1/32 in (M - x')
constexpr float kStageNucleusFill = 0.73f;         // top-p lists: the share of the capacity aimed at
constexpr uint32_t kStageMaxTiles = 256;           // tiles of the longest stochastic row the stages take (n <= 262,144)
// flags of a row's prep record
constexpr uint32_t kRowDone = 1u;        // outputs written by the prep (greedy, NaN, n <= 1)
constexpr uint32_t kRowFallback = 2u;    // sampled by lrs_sample_rows afterwards
constexpr uint32_t kRowPathK = 4u;       // top-k list (k <= kKMax)
constexpr uint32_t kRowPathN = 8u;       // top-p nucleus list
constexpr uint32_t kRowBig = 16u;        // top-p nucleus deeper than a list: lrs_stage_big
// flags of a tile's prep / result records
constexpr uint32_t kTileWalk = 1u;       // prep: the estimate allows more than two grids
constexpr uint32_t kTileOne = 2u;        // prep: the estimate allows grid u0 alone
constexpr uint32_t kTileLive = 4u;       // result: some element can change the sum
constexpr uint32_t kTileSp0 = 8u;        // result: a tie or big element on grid u0
constexpr uint32_t kTileSp1 = 16u;       // ... on grid u0 + 1
constexpr uint32_t kTileLikelyWalk = 32u;  // prep: the estimate crosses a binade inside the tile

struct RowPrep {            // prep -> classify / sum / finish (64 bytes)
    uint32_t flags;
    float M;                // max of the scaled logits (ops.rs:401-406)
    float inv_t;            // 1 / temperature (sampler.rs:115)
    float cand;             // path K: scaled-logit threshold of the list; path N: d threshold
    uint32_t k;             // effective top-k (sampler.rs:122-126)
    float cand_raw;         // the same threshold on the raw (penalised) logit, for quick tests
    uint32_t pad[2];        // sum -> finish: the exact softmax sum (bits) and its ordered steps
    uint32_t cyc_prep;      // diagnostics: SM cycles of the prep and the sum, blocks walked
    uint32_t cyc_sum;
    uint32_t walks;
    uint32_t pad2[5];
};
struct TilePrep {           // prep -> classify / sum (16 bytes)
    int32_t u0;             // lowest grid exponent of the exact sum over the tile (rigorous)
    uint32_t flags;
    float xthr;             // raw (penalised) logits at or below this add exactly nothing from this tile on
    float dthr;             // the same bound on d = fl(x' - M)
};
struct TileRes {            // classify -> sum (80 bytes)
    uint32_t t0, t1;        // increment totals on grids u0 and u0 + 1 (saturating)
    uint32_t flags;
    uint32_t bflags;        // per block of 128 elements: bit b live, 8 + b a tie or big element on
                            // grid u0, 16 + b the same on grid u0 + 1
    uint32_t b0[8], b1[8];  // per block: increment totals on grids u0 and u0 + 1
};

struct StageArgs {
    lrs_kernel_args_t a;    // inputs, outputs and the libm-expf table (shared with lrs_sample_rows)
    uint32_t nt;            // tile slots per row (>= every row's tile count)
    float4* tstat;          // [rows][nt]  (mt, pt, greedy value, greedy index bits)
    float* lmax;            // [rows][nt][32] lane maxima
    TilePrep* tprep;        // [rows][nt]
    TileRes* tres;          // [rows][nt]
    RowPrep* rprep;         // [rows]
    uint2* lists;           // [rows][kStageListCap] (scaled logit bits, index)
    uint32_t* list_n;       // [rows] entries appended (may exceed the capacity: overflow)
    uint32_t* fb_rows;      // rows left to lrs_sample_rows
    uint32_t* fb_count;
    uint32_t* live_count;   // rows prep leaves to classify (0: classify and sum have nothing to do)
    uint32_t* big_rows;     // rows for lrs_stage_big (null: none; such rows go to lrs_sample_rows)
    uint32_t* big_count;
    uint32_t* big_claim;    // lrs_stage_big: the next entry of big_rows a CTA takes
};

__device__ __forceinline__ void stage_fallback(const StageArgs& S, uint32_t r) {
    const uint32_t i = atomicAdd(S.fb_count, 1u);
    S.fb_rows[i] = r;
}

// The row's window as bits of the tile's elements [g0, g0 + cnt): the penalty set of
// sampler.rs:82-102 (distinct ids of recent[start..] below n; ids of the tile are below n).
// Built in the warp's 32 shared words; returns true if any bit is set.
__device__ __forceinline__ bool tile_window(const uint32_t* hrow, uint32_t hstart, uint32_t hlen, uint32_t g0,
                                            uint32_t cnt, uint32_t* wb) {
    const int lane = threadIdx.x & 31;
    wb[lane] = 0u;
    __syncwarp();
    for (uint32_t j = hstart + (uint32_t)lane; j < hlen; j += 32) {
        const uint32_t o = hrow[j] - g0;
        if (o < cnt) atomicOr(&wb[o >> 5], 1u << (o & 31));
    }
    __syncwarp();
    return __any_sync(0xFFFFFFFFu, wb[lane] != 0u);
}

// The penalty on the window's elements of a tile in the block layout (wb: the window's bits).
__device__ __forceinline__ void penalise_tile_blocks(const uint32_t* wb, float penalty, float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t b4 = (wb[4 * j + (lane >> 3)] >> (4 * (lane & 7))) & 15u;
        if (b4) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if ((b4 >> c) & 1u) v[4 * j + c] = penalise(v[4 * j + c], penalty);
        }
    }
}

// The warp's tile in the block layout: v[4 j + c] = element 128 j + 4 L + c (-inf past cnt),
// the penalty applied to the window's elements (sampler.rs:96-100).
__device__ __forceinline__ void load_tile_blocks(const float* base, uint32_t cnt, bool pen, const uint32_t* wb,
                                                 float penalty, float (&v)[32]) {
    const int lane = threadIdx.x & 31;
    const float ninf = __int_as_float(0xFF800000);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t e0 = 128u * j + 4u * lane;
        float4 q = make_float4(ninf, ninf, ninf, ninf);
        if (e0 < cnt) q = __ldg(reinterpret_cast<const float4*>(base + e0));
        v[4 * j + 0] = q.x;
        v[4 * j + 1] = q.y;
        v[4 * j + 2] = q.z;
        v[4 * j + 3] = q.w;
    }
    if (pen) penalise_tile_blocks(wb, penalty, v);
}

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ uint32_t window_start(const lrs_params& P, uint32_t hlen) {
    return (P.repeat_last_n != 0 && hlen > P.repeat_last_n) ? hlen - P.repeat_last_n : 0u;  // sampler.rs:84-88
}

// ------------------------------------------------------------------ stats ----
__global__ void __launch_bounds__(kStageThreads) lrs_stage_stats(const StageArgs S) {
    __shared__ uint32_t wbits[kStageThreads];
    const lrs_kernel_args_t& a = S.a;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* wb = wbits + warp * 32;
    const float kInf = __int_as_float(0x7F800000);
    const uint64_t tasks = (uint64_t)a.rows * S.nt;
    const uint64_t stride = (uint64_t)gridDim.x * kStageWarps;
    // the step's counters start from zero (the later stages read them in stream order)
    if (blockIdx.x == 0 && threadIdx.x < kLrsRowCounters) a.row_counter[threadIdx.x] = 0u;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        *S.fb_count = 0u;
        *S.live_count = 0u;
        if (S.big_rows) {
            *S.big_count = 0u;
            *S.big_claim = 0u;
        }
    }
    for (uint64_t task = (uint64_t)blockIdx.x * kStageWarps + warp; task < tasks; task += stride) {
        const uint32_t r = (uint32_t)(task / S.nt), t = (uint32_t)(task % S.nt);
        if (t == 0 && lane == 0) S.list_n[r] = 0u;
        const Geo g = row_geometry(a, r);
        if (t >= g.nchunks) continue;
        const lrs_params P = a.params[r];
        const bool greedy = P.temperature <= 0.0f;
        const bool pen_on = !(greedy && P.repetition_penalty == 1.0f) && P.repetition_penalty != 1.0f;
        if (row_passes(P, g.n) == 2u && g.nchunks > kStageMaxTiles) continue;  // (long rows: lrs_sample_rows)
        const uint32_t cnt = chunk_count(g, t);
        const uint32_t g0 = g.head + t * kTile;
        bool pen = false;
        if (pen_on && a.hist_len) {
            const uint32_t hlen = a.hist_len[r];
            pen = tile_window(a.hist + (uint64_t)r * a.hist_ld, window_start(P, hlen), hlen, g0, cnt, wb);
        }
        float v[32];
        load_tile_blocks(g.row + g0, cnt, pen, wb, P.repetition_penalty, v);
        float4* out = S.tstat + (uint64_t)r * S.nt + t;
        if (greedy) {
            // lowest index among the maximal non-NaN values (strict '>' from index 0)
            float bv = -kInf;
            uint32_t bi = 0xFFFFFFFFu;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t gi = g0 + 128u * (i >> 2) + 4u * lane + (i & 3);
                if (v[i] > bv || (v[i] == bv && gi < bi && v[i] != -kInf)) {
                    bv = v[i];
                    bi = gi;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) *out = make_float4(bv, 0.0f, 0.0f, __uint_as_float(bi));
            continue;
        }
        const float inv_t = __fdiv_rn(1.0f, P.temperature);
        const float2 it2 = make_float2(inv_t, inv_t);
        float ma = -kInf, mb = -kInf;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float2 lo = __fmul2_rn(make_float2(v[4 * j], v[4 * j + 1]), it2);
            const float2 hi = __fmul2_rn(make_float2(v[4 * j + 2], v[4 * j + 3]), it2);
            v[4 * j] = lo.x;
            v[4 * j + 1] = lo.y;
            v[4 * j + 2] = hi.x;
            v[4 * j + 3] = hi.y;
            ma = fmax3_nan(ma, lo.x, lo.y);
            mb = fmax3_nan(mb, hi.x, hi.y);
        }
        const float ml = fmax_nan(ma, mb);
        const float mt = warp_max_nan(ml);
        // approximate sum of exp(x' - mt) (estimates only; the error is bounded in the prep)
        float sl = 0.0f;
        if (mt > -kInf && mt < kInf) {
            float s2[2] = {0.0f, 0.0f};
#pragma unroll
            for (int i = 0; i < 32; ++i) s2[i & 1] += ex2_approx(__fmul_rn(__fsub_rn(v[i], mt), kLog2e));
            sl = s2[0] + s2[1];
        }
        const float pt = warp_sum_f(sl);
        S.lmax[((uint64_t)r * S.nt + t) * 32u + lane] = ml;
        if (lane == 0) *out = make_float4(mt, pt, 0.0f, 0.0f);
    }
}

// ------------------------------------------------------------------- prep ----
// Is id gi in the row's window?  (the whole warp looks)
__device__ __forceinline__ bool in_window(const uint32_t* hrow, uint32_t hstart, uint32_t hlen, uint32_t gi) {
    bool hit = false;
    for (uint32_t j = hstart + (threadIdx.x & 31); j < hlen; j += 32) hit |= hrow[j] == gi;
    return __any_sync(0xFFFFFFFFu, hit);
}

struct PrepShared {
    float vals[kStageMaxTiles * 32 + 32];  // the row's lane maxima, then its edge elements (or -inf)
    uint32_t hist[256];
    float mass[kStageNucleusBuckets];
    float xt[kNU];                         // raw dead thresholds by grid exponent (u - umin)
    double wsum[kStageWarps];
    float wf[kStageWarps];
    uint32_t wu[kStageWarps];
    int wi[2 * kStageWarps];
    uint32_t bc[4];
    float bf[4];
    double bd[2];
};

// kk-th largest (1-based) of vals[0..cnt) in shared memory, by the block: radix select on
// order-preserving keys, 8 bits a round, with warp-aggregated counter increments (the
// values share their high bits).  kk <= cnt.
__device__ __noinline__ float block_select_desc(const float* vals, uint32_t cnt, uint32_t kk, PrepShared& ps) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint32_t prefix = 0;
    for (int round = 0; round < 4; ++round) {
        const int shift = 24 - 8 * round;
        for (int b = tid; b < 256; b += kStageThreads) ps.hist[b] = 0u;
        __syncthreads();
        for (uint32_t i0 = 0; i0 < cnt; i0 += kStageThreads) {
            const uint32_t i = i0 + (uint32_t)tid;
            const uint32_t key = i < cnt ? fkey(vals[i]) : 0u;
            const bool match = i < cnt && (round == 0 || (key >> (shift + 8)) == (prefix >> (shift + 8)));
            const uint32_t bin = match ? (key >> shift) & 255u : 256u;
            const unsigned peers = __match_any_sync(0xFFFFFFFFu, bin);
            if (match && lane == __ffs(peers) - 1) atomicAdd(&ps.hist[bin], (uint32_t)__popc(peers));
        }
        __syncthreads();
        if (tid < 32) {
            uint32_t d, rem;
            digit_from_top(ps.hist, kk, d, rem);
            if (tid == 0) {
                ps.bc[0] = d;
                ps.bc[1] = rem;
            }
        }
        __syncthreads();
        prefix |= ps.bc[0] << shift;
        kk = ps.bc[1];
        __syncthreads();
    }
    return fkey_inv(prefix);
}

__device__ __forceinline__ void write_row(const lrs_kernel_args_t& a, uint32_t r, int32_t status, uint32_t token,
                                          float prob, bool advance, unsigned long long st, const lrs_row_info& inf) {
    if (status == LRS_OK && advance) a.state[r] = st;
    a.tokens[r] = token;
    if (a.probs) a.probs[r] = prob;
    if (a.status) a.status[r] = status;
    if (a.info) a.info[r] = inf;
}

__device__ __forceinline__ lrs_row_info blank_info(uint32_t path, uint32_t k) {
    lrs_row_info inf;
    inf.status = LRS_OK;
    inf.token = 0;
    inf.path = path;
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
    return inf;
}

// One CTA per row.
__global__ void __launch_bounds__(kStageThreads) lrs_stage_prep(const StageArgs S) {
    __shared__ PrepShared ps;
    const lrs_kernel_args_t& a = S.a;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float kInf = __int_as_float(0x7F800000);
    const uint32_t r = blockIdx.x;
    const long long t_start = clock64();
    const lrs_params P = a.params[r];
    const Geo g = row_geometry(a, r);
    const uint32_t n = g.n;
    const bool greedy = P.temperature <= 0.0f;  // sampler.rs:62, 104 (NaN -> stochastic)
    const bool fast_greedy = greedy && P.repetition_penalty == 1.0f;
    const bool pen_on = !fast_greedy && P.repetition_penalty != 1.0f;
    const uint32_t k = (P.top_k == 0 || P.top_k > n) ? n : P.top_k;  // sampler.rs:122-126
    const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;            // sampler.rs:136
    const uint32_t path = greedy ? (fast_greedy ? 0u : 1u) : (n == 1 ? 3u : 2u);
    const uint32_t ntile = g.nchunks;
    RowPrep rp;
    rp.flags = 0;
    rp.M = 0.0f;
    rp.inv_t = 1.0f;
    rp.cand = -kInf;
    rp.k = k;
    rp.cand_raw = -kInf;
    rp.pad[0] = rp.pad[1] = 0;
    rp.cyc_prep = rp.cyc_sum = rp.walks = 0;
    for (int q = 0; q < 5; ++q) rp.pad2[q] = 0;
    lrs_row_info inf = blank_info(path, k);
    auto leave = [&](uint32_t flags) {  // (thread 0 writes the record; every thread returns)
        if (tid == 0) {
            rp.flags = flags;
            S.rprep[r] = rp;
            if (flags & kRowFallback) stage_fallback(S, r);
        }
    };
    if (n == 0) {  // sampler.rs:57-60
        if (tid == 0) write_row(a, r, LRS_OK, 0u, 1.0f, false, 0ull, inf);
        leave(kRowDone);
        return;
    }
    if (row_passes(P, n) == 2u && ntile > kStageMaxTiles) {  // long rows: lrs_sample_rows
        leave(kRowFallback);
        return;
    }
    const uint32_t hlen = (pen_on && a.hist_len) ? a.hist_len[r] : 0u;
    const uint32_t* hrow = a.hist ? a.hist + (uint64_t)r * a.hist_ld : nullptr;
    const uint32_t hstart = window_start(P, hlen);
    // the unaligned edge elements (at most 3 + 3): warp 0, lanes 0 .. edges-1
    const uint32_t edges = g.head + g.tail;
    const bool mine = warp == 0 && (uint32_t)lane < edges;
    const uint32_t egi = (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
    float ex = -kInf;
    if (warp == 0) {
        if (mine) ex = g.row[egi];
        for (uint32_t e = 0; e < edges; ++e) {  // (penalty: each is looked up in the window by the warp)
            const uint32_t gi = __shfl_sync(0xFFFFFFFFu, egi, (int)e);
            const bool hit = pen_on && in_window(hrow, hstart, hlen, gi);
            if (hit && (uint32_t)lane == e) ex = penalise(ex, P.repetition_penalty);
        }
    }
    if (greedy) {
        // lowest index among the maximal non-NaN values (sampler.rs:62-70, 104-113)
        float bv = -kInf;
        uint32_t bi = 0xFFFFFFFFu;
        if (mine && ex == ex && ex != -kInf) {
            bv = ex;
            bi = egi;
        }
        for (uint32_t t = (uint32_t)tid; t < ntile; t += kStageThreads) {
            const float4 q = S.tstat[(uint64_t)r * S.nt + t];
            const uint32_t qi = __float_as_uint(q.w);
            if (q.x > bv || (q.x == bv && qi < bi)) {
                bv = q.x;
                bi = qi;
            }
        }
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
            ps.wf[warp] = bv;
            ps.wu[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kStageWarps; ++w)
                if (ps.wf[w] > bv || (ps.wf[w] == bv && ps.wu[w] < bi)) {
                    bv = ps.wf[w];
                    bi = ps.wu[w];
                }
            const float x0 = g.row[0];  // NaN at index 0 -> 0 (the penalty keeps a NaN a NaN)
            if (x0 != x0 || bi == 0xFFFFFFFFu) bi = 0;
            inf.token = bi;
            inf.cycles[4] = 1u;  // (finished by the staged pipeline)
            write_row(a, r, LRS_OK, bi, 1.0f, false, 0ull, inf);
        }
        leave(kRowDone);
        return;
    }
    const float inv_t = __fdiv_rn(1.0f, P.temperature);  // sampler.rs:115
    const float exs = mine ? __fmul_rn(ex, inv_t) : -kInf;
    // the row max (ops.rs:401-406, NaN-propagating)
    float mx = exs;
    for (uint32_t t = (uint32_t)tid; t < ntile; t += kStageThreads) mx = fmax_nan(mx, S.tstat[(uint64_t)r * S.nt + t].x);
    mx = warp_max_nan(mx);
    if (lane == 0) ps.wf[warp] = mx;
    __syncthreads();
    float M = ps.wf[0];
    for (int w = 1; w < kStageWarps; ++w) M = fmax_nan(M, ps.wf[w]);
    __syncthreads();
    inf.max = M;
    if (n == 1) {  // one uniform is consumed and the token is 0 (sampler.rs:155-162)
        if (tid == 0) {
            unsigned long long st = a.state[r];
            (void)next_f32(&st);
            inf.cycles[4] = 1u;
            write_row(a, r, LRS_OK, 0u, 1.0f, true, st, inf);
        }
        leave(kRowDone);
        return;
    }
    if (M != M || fabsf(M) == kInf) {  // NaN probabilities: the reference panics (sampler.rs:129/132)
        if (tid == 0) {
            inf.status = LRS_E_NAN;
            inf.token = LRS_TOKEN_NONE;
            inf.prob = 0.0f;
            inf.cycles[4] = 1u;
            write_row(a, r, LRS_E_NAN, LRS_TOKEN_NONE, 0.0f, false, 0ull, inf);
        }
        leave(kRowDone);
        return;
    }
    rp.M = M;
    rp.inv_t = inv_t;
    const bool pathK = k < n && k <= (uint32_t)kKMax;
    if (!pathK && !topp_on) {  // every element survives: the survivor sum runs over the whole row
        leave(kRowFallback);
        return;
    }
    // ---- running-sum estimates and the grids of every tile (one tile a thread) ----
    // P_t: the head's exp sum plus the tile sums before t, each rescaled to M.  The exact
    // sequential sum there, S_t, lies within P_t (1 +- delta_t) with delta_t = i 2^-23 +
    // 2^-13 (i elements before the tile): each of the i f32 roundings moves it by at most
    // 2^-24 S_t, and P's own error (approximate exps of once-rounded arguments, the f32 tile
    // sums) is far below 2^-13.  So the exact sum is on grid u0 = grid(P_t (1 - delta_t)) or
    // above over the whole tile, and elements with d < (u0 - 1) ln 2 - 0.01 add exactly nothing.
    if (warp == 0) {
        double eh = 0.0, et = 0.0;
        if (mine) ((uint32_t)lane < g.head ? eh : et) = exp((double)__fsub_rn(exs, M));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            eh += __shfl_xor_sync(0xFFFFFFFFu, eh, o);
            et += __shfl_xor_sync(0xFFFFFFFFu, et, o);
        }
        if (lane == 0) {
            ps.bd[0] = eh;
            ps.bd[1] = et;
        }
    }
    const uint32_t t = (uint32_t)tid;  // (ntile <= kStageMaxTiles == kStageThreads)
    const bool tin = t < ntile;
    double c = 0.0;
    if (tin) {
        const float4 q = S.tstat[(uint64_t)r * S.nt + t];
        if (q.x > -kInf) c = (double)q.y * exp((double)q.x - (double)M);
    }
    double incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double tv = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += tv;
    }
    if (lane == 31) ps.wsum[warp] = incl;
    __syncthreads();
    double before = ps.bd[0];
    for (int w = 0; w < warp; ++w) before += ps.wsum[w];
    double s_total = ps.bd[0] + ps.bd[1];
    for (int w = 0; w < kStageWarps; ++w) s_total += ps.wsum[w];
    bool big = false;
    if (!pathK && topp_on && k > kStageListCap) {
        // Every probability is at most 1/S (the max's exp is 1), so the nucleus holds at least
        // top_p S elements, S above s_total (1 - delta) (the bound of the tile estimates over
        // the whole row): a nucleus that cannot fit in the list goes to lrs_sample_rows now.
        const double delta = (double)n * 0x1p-23 + 0x1p-13;
        if ((double)P.top_p * s_total * (1.0 - delta) > 1.01 * (double)kStageListCap) {
            if (!S.big_rows || n > kStageMaxTiles * (uint32_t)kTile) {  // (the window bitmap's bound)
                leave(kRowFallback);
                return;
            }
            big = true;  // (lrs_stage_big samples it once the sum stage has its denominator)
        }
    }
    TilePrep tp{0, 0u, 0.0f, 0.0f};
    int umin = 0x7FFFFFFF, umax = -0x7FFFFFFF;
    if (tin) {
        const double pt0 = before + incl - c, pt1 = before + incl;
        const double i0 = (double)(g.head + t * kTile), i1 = i0 + (double)chunk_count(g, t);
        const double lo = pt0 * (1.0 - (i0 * 0x1p-23 + 0x1p-13));
        const double hi = pt1 * (1.0 + (i1 * 0x1p-23 + 0x1p-13));
        const int u0 = unit_exp(__double2float_rd(lo));
        const int uh = unit_exp(__double2float_ru(hi));
        tp.u0 = u0;
        tp.flags = uh > u0 + 1 ? kTileWalk : (uh == u0 ? kTileOne : 0u);
        // (a likely walk: the central estimate crosses a binade inside the tile)
        if (unit_exp((float)pt0) != unit_exp((float)pt1)) tp.flags |= kTileLikelyWalk;
        tp.dthr = __fsub_rn(__fmul_rn((float)(u0 - 1), 0.69314718f), 0.01f);
        umin = umax = u0;
    }
    umin = __reduce_min_sync(0xFFFFFFFFu, umin);
    umax = __reduce_max_sync(0xFFFFFFFFu, umax);
    if (lane == 0) {
        ps.wi[warp] = umin;
        ps.wi[kStageWarps + warp] = umax;
    }
    __syncthreads();
    umin = ps.wi[0];
    umax = ps.wi[kStageWarps];
    for (int w = 1; w < kStageWarps; ++w) {
        umin = min(umin, ps.wi[w]);
        umax = max(umax, ps.wi[kStageWarps + w]);
    }
    // the raw dead thresholds, one bisection per distinct grid of the row's tiles
    for (int u = umin + tid; u <= umax; u += kStageThreads)
        ps.xt[u - umin] = raw_threshold(__fsub_rn(__fmul_rn((float)(u - 1), 0.69314718f), 0.01f), inv_t, M);
    // the lane maxima and the edge elements, staged for the selections below
    const uint32_t nl = ntile * 32u;
    const float* lm = S.lmax + (uint64_t)r * S.nt * 32u;
    for (uint32_t i = (uint32_t)tid; i < nl; i += kStageThreads) ps.vals[i] = lm[i];
    if (warp == 0) ps.vals[nl + lane] = exs;  // (lane e: edge element e, or -inf)
    __syncthreads();
    if (tin) {
        tp.xthr = ps.xt[tp.u0 - umin];
        S.tprep[(uint64_t)r * S.nt + t] = tp;
    }
    const uint32_t nv = nl + 32u;
    // ---- the candidate threshold of the finish ----
    if (pathK) {
        // k-th largest of the lane maxima (k <= kKMax of them are distinct elements at or
        // above it, so it bounds the row's k-th largest scaled logit from below); less the
        // tie margin (generous for both the bound and the final k-th value), every element
        // whose probability can reach the k-th probability lies above it.
        float th;
        if (k <= ntile && nv + 32u + ntile <= kStageMaxTiles * 32u + 32u) {
            // A tile's max is one of its lane maxima, so the k-th largest of the tile maxima and
            // the edge elements bounds the k-th largest of all from below: select it among
            // those, keep the values at or above it (in the free end of ps.vals), select there.
            float* tv = ps.vals + nv;  // (tile maxima, then the edge elements)
            for (uint32_t t2 = (uint32_t)tid; t2 < ntile; t2 += kStageThreads)
                tv[t2] = S.tstat[(uint64_t)r * S.nt + t2].x;
            if (warp == 0) tv[ntile + lane] = ps.vals[nl + lane];
            __syncthreads();
            const float th0 = block_select_desc(tv, ntile + 32u, k, ps);
            if (tid == 0) ps.bc[2] = 0u;
            __syncthreads();
            float* kept = ps.vals + nv;  // (the tile maxima are done with)
            for (uint32_t i0 = 0; i0 < nv; i0 += kStageThreads) {
                const uint32_t i = i0 + (uint32_t)tid;
                const float x = i < nv ? ps.vals[i] : -kInf;
                const bool keep = i < nv && x >= th0;
                const unsigned m = __ballot_sync(0xFFFFFFFFu, keep);
                uint32_t o = 0;
                if (lane == 0 && m) o = atomicAdd(&ps.bc[2], (uint32_t)__popc(m));
                o = __shfl_sync(0xFFFFFFFFu, o, 0) + (uint32_t)__popc(m & ((1u << lane) - 1u));
                if (keep && o < kStageMaxTiles * 32u + 32u - nv) kept[o] = x;
            }
            __syncthreads();
            const uint32_t nk = ps.bc[2];
            __syncthreads();
            th = nk <= kStageMaxTiles * 32u + 32u - nv ? block_select_desc(kept, nk, k, ps)
                                                       : block_select_desc(ps.vals, nv, k, ps);
        } else {
            th = block_select_desc(ps.vals, nv, k, ps);
        }
        float cand = -kInf;
        if (th > -kInf) cand = __fsub_rn(th, __fmul_rn(__fadd_rn(__fadd_rn(fabsf(th), fabsf(M)), 1.0f), 0x1p-17f));
        rp.flags = kRowPathK;
        rp.cand = cand;
        rp.cand_raw = cand > -kInf ? raw_threshold(cand, inv_t, 0.0f) : -kInf;
    } else if (big) {  // no list: classify and sum only give the denominator
        rp.flags = kRowPathN | kRowBig;
        rp.cand = kInf;
        rp.cand_raw = kInf;
    } else {
        // The nucleus (sampler.rs:135-146) is the head of the sorted probabilities up to mass
        // top_p.  The list takes every element with d >= theta, theta the shallower of two
        // guesses: the first bucket edge (width 1/32) where the mass of the lane maxima above
        // it reaches (top_p + 2^-16) times the estimated sum (lane maxima are distinct
        // elements, so the mass of all elements there is at least that), and the depth of
        // the lane maximum of a rank that fills about kStageNucleusFill of the list.
        // The finish checks that the cut lies inside the list, and gathers a deeper list
        // from the row where it does not.
        for (int b = tid; b < kStageNucleusBuckets; b += kStageThreads) ps.mass[b] = 0.0f;
        __syncthreads();
        for (uint32_t i = (uint32_t)tid; i < nv; i += kStageThreads) {
            const float d = __fsub_rn(ps.vals[i], M);
            if (d >= -(float)(kStageNucleusBuckets - 1) / 32.0f)
                atomicAdd(&ps.mass[(int)fminf(-d * 32.0f, (float)(kStageNucleusBuckets - 2))], expf(d));
        }
        __syncthreads();
        if (warp == 0) {
            const double target = ((double)P.top_p + 0x1p-16) * s_total;
            double acc = 0.0;
            int found = -1;
            for (int base = 0; base < kStageNucleusBuckets - 1 && found < 0; base += 32) {
                const int b = base + lane;
                double m = b < kStageNucleusBuckets - 1 ? (double)ps.mass[b] : 0.0;
                double mi = m;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const double tv = __shfl_up_sync(0xFFFFFFFFu, mi, o);
                    if (lane >= o) mi += tv;
                }
                const unsigned hit = __ballot_sync(0xFFFFFFFFu, b < kStageNucleusBuckets - 1 && acc + mi >= target);
                if (hit) found = base + __ffs(hit) - 1;
                acc += __shfl_sync(0xFFFFFFFFu, mi, 31);
            }
            if (lane == 0) ps.bf[0] = found >= 0 ? -(float)(found + 1) / 32.0f : -kInf;
        }
        __syncthreads();
        const float th_mass = ps.bf[0];
        // The rank: with the elements of a row in no particular order, a fraction f of the lanes
        // (32 elements each) whose maximum is at or above a threshold means about
        // 32 nl (1 - (1 - f)^(1/32)) elements there; the rank is the f that makes that
        // kStageNucleusFill of the list's capacity.
        // (A row that fits whole takes every element.)
        const double fill = (double)kStageNucleusFill * kStageListCap;
        float th_rank = -kInf;
        if (fill < 32.0 * nl) {
            const double f = 1.0 - pow(1.0 - fill / (32.0 * nl), 32.0);
            uint32_t rank = (uint32_t)(f * nl);
            rank = rank < 1u ? 1u : (rank > nv ? nv : rank);
            const float x_rank = block_select_desc(ps.vals, nv, rank, ps);
            th_rank = x_rank > -kInf ? __fsub_rn(x_rank, M) : -kInf;
        }
        rp.flags = kRowPathN;
        rp.cand = fmaxf(th_mass, th_rank);  // elements with d >= this (d = fl(x' - M))
        rp.cand_raw = rp.cand > -kInf ? raw_threshold(rp.cand, inv_t, M) : -kInf;  // largest raw x with d below it
    }
    if (warp == 0) {
        // the edge elements that qualify join the list (the tiles' candidates come from classify)
        const bool cq = mine && ((rp.flags & kRowPathK) ? exs >= rp.cand : __fsub_rn(exs, M) >= rp.cand);
        const unsigned cm = __ballot_sync(0xFFFFFFFFu, cq);
        uint32_t base = 0;
        if (lane == 0 && cm) base = atomicAdd(S.list_n + r, (uint32_t)__popc(cm));
        base = __shfl_sync(0xFFFFFFFFu, base, 0) + (uint32_t)__popc(cm & ((1u << lane) - 1u));
        if (cq && base < kStageListCap) S.lists[(uint64_t)r * kStageListCap + base] = make_uint2(__float_as_uint(exs), egi);
    }
    if (tid == 0) {
        const long long dt = clock64() - t_start;
        rp.cyc_prep = dt > 0xFFFFFFFFll ? 0xFFFFFFFFu : (uint32_t)dt;
        S.rprep[r] = rp;
        atomicAdd(S.live_count, 1u);
        if (big) S.big_rows[atomicAdd(S.big_count, 1u)] = r;
    }
}

// --------------------------------------------------------------- classify ----
// One element's increments (integer units) on grids u0 and u0 + 1 (unit 2^u0, binade base
// bm0 = 2^(u0 + 23), half unit h0; the same for u0 + 1), from CUDA's expf where it cannot
// round differently from libm's (within 2 ulp: more than 2^-21 e from every rounding boundary
// of either grid), else from libm's value; sp: a tie (exact half unit) or an element of half a
// binade or more on that grid (an ordered step).  one: grid u0 alone (channel 1 is flagged).
struct ElemCls {
    uint32_t c0, c1;
    bool sp0, sp1;
};
__device__ __forceinline__ ElemCls classify_units(float d, int u0, float bm0, float bm1, float h0, float h1, bool one,
                                                  const ExpTable tab) {
    ElemCls r{0u, 0u, false, one};
    bool ex = d == 0.0f;
    float e = ex ? 1.0f : expf(d);
    float i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);  // RN(e / U) U below bm0
    float i1 = one ? 0.0f : __fsub_rn(__fadd_rn(bm1, e), bm1);
    if (!ex) {
        const float tol = __fmul_rn(e, 4.76837158203125e-07f);  // 2^-21 e > 2 ulp
        bool amb = e < 7.8886091e-31f || fabsf(__fsub_rn(e, bm0)) <= tol ||
                   (e < bm0 && fabsf(__fsub_rn(e, i0)) >= __fsub_rn(h0, tol));
        if (!one)
            amb = amb || fabsf(__fsub_rn(e, bm1)) <= tol || (e < bm1 && fabsf(__fsub_rn(e, i1)) >= __fsub_rn(h1, tol));
        if (amb) {
            e = exact_expf(d, tab);
            ex = true;
            i0 = __fsub_rn(__fadd_rn(bm0, e), bm0);
            i1 = one ? 0.0f : __fsub_rn(__fadd_rn(bm1, e), bm1);
        }
    }
    if (e >= bm0) {
        r.sp0 = true;
    } else {
        r.c0 = grid_units(i0, -u0);
        if (ex && h0 > 0.0f && fabsf(__fsub_rn(e, i0)) == h0) r.sp0 = true;
    }
    if (!one) {
        if (e >= bm1) {
            r.sp1 = true;
        } else {
            r.c1 = grid_units(i1, -(u0 + 1));
            if (ex && fabsf(__fsub_rn(e, i1)) == h1) r.sp1 = true;
        }
    }
    return r;
}

constexpr int kClassifyWarps = 4;  // warps per block of the classify stage

// One warp per tile (grid-stride over every row's tiles).  The tile stays in registers in the
// block layout (lane L: elements 128 j + 4 L + c, j the block of 128); a lane queues its live
// elements' d values (x' > xthr) with their blocks in shared memory, then classifies its queue
// in block order, adding each block's increments once per change of block.  Candidates of the
// finish go to the row's list under one reservation per warp.
__global__ void __launch_bounds__(kClassifyWarps * 32) lrs_stage_classify(const StageArgs S) {
    __shared__ uint32_t wbits[kClassifyWarps * 32];
    __shared__ float qd[kClassifyWarps * 32 * 32];    // per warp: queue slot k of lane L at 32 k + L
    __shared__ uint8_t qb[kClassifyWarps * 32 * 32];  // ... and the element's block
    __shared__ uint32_t bcount[kClassifyWarps * 16];  // per warp: block increment totals (grids u0, u0 + 1)
    const lrs_kernel_args_t& a = S.a;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* wb = wbits + warp * 32;
    float* wq = qd + warp * 1024;
    uint8_t* wqb = qb + warp * 1024;
    uint32_t* bc = bcount + warp * 16;
    const ExpTable exptab{a.exp_index, a.exp_entries, a.exp_near};
    if (*(volatile const uint32_t*)S.live_count == 0u) return;  // (every row finished in prep or left)
    const uint64_t tasks = (uint64_t)a.rows * S.nt;
    const uint64_t stride = (uint64_t)gridDim.x * kClassifyWarps;
    uint64_t task = (uint64_t)blockIdx.x * kClassifyWarps + warp;
    uint32_t r = (uint32_t)(task / S.nt), t = (uint32_t)(task % S.nt);  // (then stepped)
    const uint32_t sq = (uint32_t)(stride / S.nt), sr = (uint32_t)(stride % S.nt);
    for (; task < tasks; task += stride, r += sq, t += sr) {
        if (t >= S.nt) {
            t -= S.nt;
            ++r;
        }
        const Geo g = row_geometry(a, r);
        if (t >= g.nchunks) continue;
        const uint32_t cnt = chunk_count(g, t);
        const uint32_t g0 = g.head + t * kTile;
        // the tile's raw values first: their latency overlaps the records' (nearly every tile
        // of a row holds live elements)
        float v[32];
        load_tile_blocks(g.row + g0, cnt, false, wb, 1.0f, v);
        {  // (the warp's next tile into L2, a line per lane)
            uint32_t tn = t + sr, rn = r + sq;
            if (tn >= S.nt) {
                tn -= S.nt;
                ++rn;
            }
            if (task + stride < tasks && tn < g.nchunks && (uint32_t)lane * 32u < chunk_count(g, tn))
                prefetch_l2(a.logits + (uint64_t)rn * a.ld + g.head + tn * kTile + lane * 32u);
        }
        const uint64_t ti = (uint64_t)r * S.nt + t;
        const RowPrep rp = S.rprep[r];
        const TilePrep tp = S.tprep[ti];
        const float mt = S.tstat[ti].x;
        const lrs_params P = a.params[r];
        const uint32_t hlen = a.hist_len ? a.hist_len[r] : 0u;
        if (rp.flags & (kRowDone | kRowFallback)) continue;
        const float M = rp.M, inv_t = rp.inv_t;
        const bool pathK = rp.flags & kRowPathK;
        const float dmax = __fsub_rn(mt, M);
        const bool sum_live = !(dmax < tp.dthr);
        const bool cand_live = pathK ? !(mt < rp.cand) : !(dmax < rp.cand);
        if (!sum_live && !cand_live) {
            if (lane == 0) {
                S.tres[ti].flags = 0u;
                S.tres[ti].bflags = 0u;
            }
            continue;
        }
        if (P.repetition_penalty != 1.0f && hlen) {
            if (tile_window(a.hist + (uint64_t)r * a.hist_ld, window_start(P, hlen), hlen, g0, cnt, wb))
                penalise_tile_blocks(wb, P.repetition_penalty, v);
        }
        const float xthr = sum_live ? tp.xthr : __int_as_float(0x7F800000);
        const float craw = cand_live ? rp.cand_raw : __int_as_float(0x7F800000);
        // the lane's live elements (x' > xthr) into its queue (in block order); its candidates
        // (x' > craw: d, or the scaled logit, at or above the list threshold)
        uint32_t nq = 0, cm = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            cm |= (v[i] > craw ? 1u : 0u) << i;
            if (v[i] > xthr) {
                wq[nq * 32u + lane] = d_of(v[i], inv_t, M);
                wqb[nq * 32u + lane] = (uint8_t)(i >> 2);
                ++nq;
            }
        }
        if (__any_sync(0xFFFFFFFFu, cm != 0u)) {  // the candidates: one reservation per warp
            const uint32_t nc = (uint32_t)__popc(cm);
            const uint32_t incl = warp_incl_scan_plain(nc);
            uint32_t base = 0;
            if (lane == 31) base = atomicAdd(S.list_n + r, incl);
            base = __shfl_sync(0xFFFFFFFFu, base, 31) + incl - nc;
            uint2* lst = S.lists + (uint64_t)r * kStageListCap;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if ((cm >> i) & 1u) {
                    const uint32_t gi = g0 + 128u * (uint32_t)(i >> 2) + 4u * (uint32_t)lane + (uint32_t)(i & 3);
                    if (base < kStageListCap) lst[base] = make_uint2(__float_as_uint(__fmul_rn(v[i], inv_t)), gi);
                    ++base;
                }
            }
        }
        uint32_t t0v = 0, t1v = 0, fl = 0, bf = 0;
        if (__any_sync(0xFFFFFFFFu, nq != 0u)) {
            // increments of the live elements on grids u0 and u0 + 1, per block of 128
            const int u0 = tp.u0;
            const bool one = tp.flags & kTileOne;
            if (lane < 16) bc[lane] = 0u;
            __syncwarp();
            const float bm0 = grid_value(u0, kTwo23), bm1 = __fadd_rn(bm0, bm0);
            const float h0 = u0 > -149 ? pow2f(u0 - 1) : 0.0f, h1 = pow2f(u0);
            uint32_t cb = 8u, a0 = 0u, a1 = 0u, bfl = 0u;
            for (uint32_t k = 0; k < nq; ++k) {
                const float d = wq[k * 32u + lane];
                const uint32_t b = wqb[k * 32u + lane];
                if (b != cb) {
                    if (cb < 8u) {
                        atomicAdd(&bc[cb], a0);
                        atomicAdd(&bc[8u + cb], a1);
                    }
                    cb = b;
                    a0 = a1 = 0u;
                }
                const ElemCls c = classify_units(d, u0, bm0, bm1, h0, h1, one, exptab);
                a0 += c.c0;  // (a block's count is at most 128 * 2^23 < 2^32)
                a1 += c.c1;
                bfl |= (1u << b) | (c.sp0 ? 0x100u << b : 0u) | (c.sp1 ? 0x10000u << b : 0u);
            }
            if (cb < 8u) {
                atomicAdd(&bc[cb], a0);
                atomicAdd(&bc[8u + cb], a1);
            }
            __syncwarp();
            // (saturated where a block leaves the grid)
            const uint32_t c0 = lane < 8 ? min(bc[lane], kSat) : 0u, c1 = lane < 8 ? min(bc[8 + lane], kSat) : 0u;
            bf = __reduce_or_sync(0xFFFFFFFFu, bfl);
            t0v = min(__reduce_add_sync(0xFFFFFFFFu, c0), kSat);
            t1v = min(__reduce_add_sync(0xFFFFFFFFu, c1), kSat);
            fl = kTileLive | ((bf >> 8) & 0xFFu ? kTileSp0 : 0u) | ((bf >> 16) & 0xFFu ? kTileSp1 : 0u);
            if (lane < 8) {
                S.tres[ti].b0[lane] = c0;
                S.tres[ti].b1[lane] = c1;
            }
        }
        if (lane == 0) {
            TileRes* out = S.tres + ti;
            out->t0 = t0v;
            out->t1 = t1v;
            out->flags = fl;
            out->bflags = bf;
        }
        __syncwarp();  // (the queue and counts are reused by the next tile)
    }
}

// ----------------------------------------------------------------- walks ----
// Exact sequential sum s <- fl(s + e) (ops.rs:408-411) over one block of 128 elements in
// index order, by one warp: lane L holds positions 4 L .. 4 L + 3, with libm's values.  A
// round classifies the remaining positions on the grid of the running sum and the next one
// (lrs_grid.h); ordered steps (a binade crossing, a tie, an element of half a binade or
// more) are found by prefix sums on the channel of the sum's current grid and added
// exactly; only a sum that leaves both grids is classified again.  A sum that starts from
// zero crosses many binades in its first elements: such a block is added one by one.
// The block's 128 values added to s one after another by lane 0 from the warp's shared buffer
// (ser: 128 floats), the result on every lane.
__device__ __forceinline__ float warp_serial128(const float (&e)[4], float* ser, float s) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int c = 0; c < 4; ++c) ser[4 * lane + c] = e[c];
    __syncwarp();
    if (lane == 0) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = ser[j];
        for (int i = 0; i < 128; i += 8) {
            float nx[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) nx[j] = i + 8 + j < 128 ? ser[i + 8 + j] : 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[j]);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = nx[j];
        }
    }
    s = __shfl_sync(0xFFFFFFFFu, s, 0);
    __syncwarp();  // (the buffer is read no more)
    return s;
}

__device__ __noinline__ float warp_walk_block(float4 q, uint32_t pen4, float penalty,
                                              float inv_t, float M, float xthr, float s, const ExpTable tab,
                                              uint32_t* events, float* ser) {
    const int lane = threadIdx.x & 31;
    float e[4];
    {
        float x[4] = {q.x, q.y, q.z, q.w};  // (the lane's four raw values; -inf past the block)
        // (the four exps side by side; the table only where the rounded double exp is too
        // close to a rounding midpoint)
        float d[4];
        bool ok[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if ((pen4 >> c) & 1u) x[c] = penalise(x[c], penalty);
            d[c] = x[c] > xthr ? d_of(x[c], inv_t, M) : -1.0f;
            ok[c] = expf_rounded(d[c], tab, e[c]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (!ok[c]) e[c] = exact_expf_table(d[c], tab, e[c]);
            if (!(x[c] > xthr)) e[c] = 0.0f;
            else if (d[c] == 0.0f) e[c] = 1.0f;
        }
    }
    if (s == 0.0f) {  // (the sum starts here: one lane adds all 128 in order)
        if (lane == 0) *events += 128u;
        return warp_serial128(e, ser, s);
    }
    int consumed = -1;
    for (int round = 0; round < 129; ++round) {
        const int uu = unit_exp(s), u1 = uu + 1;  // (the sum only grows)
        uint32_t a0[4], a1[4], sp0 = 0, sp1 = 0, t0 = 0, t1 = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            a0[c] = a1[c] = 0u;
            if (4 * lane + c > consumed && e[c] != 0.0f) {
                const Cls2 k = classify2(__float_as_uint(e[c]), uu, +1);
                a0[c] = k.inc0;
                a1[c] = k.inc1;
                sp0 |= (uint32_t)k.spec0 << c;
                sp1 |= (uint32_t)k.spec1 << c;
            }
            t0 = sat_add(t0, a0[c]);
            t1 = sat_add(t1, a1[c]);
        }
        const uint32_t l0 = warp_incl_scan(t0), l1 = warp_incl_scan(t1);
        uint32_t x0 = __shfl_up_sync(0xFFFFFFFFu, l0, 1), x1 = __shfl_up_sync(0xFFFFFFFFu, l1, 1);
        if (lane == 0) x0 = x1 = 0u;  // (not l - t: the scans saturate)
        const uint32_t tot0 = __shfl_sync(0xFFFFFFFFu, l0, 31), tot1 = __shfl_sync(0xFFFFFFFFu, l1, 31);
        if (round == 0 && (grid_count(s, uu) + tot0 >= 2u * kTwo24 ||
                           __popc(__ballot_sync(0xFFFFFFFFu, sp0 != 0u)) >= 4)) {
            // (a block whose sum crosses two binades or more, or that holds several ordered
            // steps: one lane adds all 128 in order, cheaper than a warp step per event)
            if (lane == 0) *events += 128u;
            return warp_serial128(e, ser, s);
        }
        uint32_t base0 = 0, base1 = 0;  // channel prefixes at the last ordered step
        bool again = false;
        for (int step = 0; step < 129; ++step) {
            const int uc = unit_exp(s);
            const int ch = uc == uu ? 0 : (uc == u1 ? 1 : -1);
            if (ch < 0) {  // a second grid change: classify the rest again
                again = true;
                break;
            }
            const uint32_t A = grid_count(s, uc);
            const uint32_t bse = ch ? base1 : base0;
            const uint32_t spm = ch ? sp1 : sp0;
            uint32_t run = ch ? x1 : x0, r0 = x0, r1 = x1;
            uint32_t cand = 0xFFFFFFFFu, pre = 0, cb0 = 0, cb1 = 0;
            float val = 0.0f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t pr = run;
                run = sat_add(run, ch ? a1[c] : a0[c]);
                r0 = sat_add(r0, a0[c]);
                r1 = sat_add(r1, a1[c]);
                if (cand == 0xFFFFFFFFu && 4 * lane + c > consumed &&
                    (((spm >> c) & 1u) || A + (run - bse) >= kTwo24)) {
                    cand = (uint32_t)(4 * lane + c);
                    pre = pr;
                    cb0 = r0;
                    cb1 = r1;
                    val = e[c];
                }
            }
            const uint32_t first = __reduce_min_sync(0xFFFFFFFFu, cand);
            if (first == 0xFFFFFFFFu) {
                s = grid_value(uc, A + ((ch ? tot1 : tot0) - bse));  // (below 2^24: no crossing)
                break;
            }
            const int owner = (int)(first >> 2);
            const float after = __fadd_rn(grid_value(uc, A + (pre - bse)), val);  // (meaningful in the owner)
            s = __shfl_sync(0xFFFFFFFFu, after, owner);
            base0 = __shfl_sync(0xFFFFFFFFu, cb0, owner);
            base1 = __shfl_sync(0xFFFFFFFFu, cb1, owner);
            consumed = (int)first;
            if (lane == 0) ++*events;
        }
        if (!again) break;
    }
    return s;
}

// ------------------------------------------------------------------- sum ----

constexpr int kSumWarps = 4;  // rows per block of the sum stage (one warp each)

// The running sum over tile t (its grid records from classify): block by block, each block
// added in one step where the sum stays on a grid it was classified for, else walked.  The
// tile's values are loaded first, side by side with its records, so that a walk finds its
// block in registers.
__device__ __noinline__ float warp_tile_blocks(const StageArgs& S, const Geo& g, uint32_t r, uint32_t t, float s,
                                               const lrs_params& P, float inv_t, float M, const uint32_t* hrow,
                                               uint32_t hstart, uint32_t hlen, uint32_t* wb, const ExpTable tab,
                                               uint32_t* events, uint32_t* walks, float* ser) {
    const int lane = threadIdx.x & 31;
    const uint64_t ti = (uint64_t)r * S.nt + t;
    const uint32_t cnt = chunk_count(g, t);
    const uint32_t g0 = g.head + t * kTile;
    float4 tq[8];  // (lane L: elements 128 j + 4 L .. + 3 of the tile, -inf past its end)
    {
        const float ninf = __int_as_float(0xFF800000);
        const float* tb = g.row + g0 + 4 * lane;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            tq[j] = 128u * (uint32_t)j + 4u * (uint32_t)lane < cnt ? __ldg(reinterpret_cast<const float4*>(tb + 128 * j))
                                                                  : make_float4(ninf, ninf, ninf, ninf);
    }
    const TilePrep tp = S.tprep[ti];
    const uint32_t bflags = S.tres[ti].bflags;
    uint32_t c0 = 0, c1 = 0;
    if (lane < 8) {
        c0 = S.tres[ti].b0[lane];
        c1 = S.tres[ti].b1[lane];
    }
    const bool pen_on = P.repetition_penalty != 1.0f;
    bool pen = false;
    if (pen_on && hlen) pen = tile_window(hrow, hstart, hlen, g0, cnt, wb);
    const uint32_t nb = (cnt + 127u) / 128u;
    for (uint32_t b0 = 0; b0 < nb;) {
        const uint32_t b = (uint32_t)lane;
        const bool in = b >= b0 && b < nb;
        const bool live = in && ((bflags >> b) & 1u);
        const int uu = unit_exp(s);
        const uint32_t A = grid_count(s, uu);
        uint32_t inc = 0;
        bool ok = !live;
        if (live) {
            if (uu == tp.u0 && !((bflags >> (8 + b)) & 1u)) {
                inc = c0;
                ok = true;
            } else if (uu == tp.u0 + 1 && !((bflags >> (16 + b)) & 1u)) {
                inc = c1;
                ok = true;
            }
        }
        const uint32_t incl = warp_incl_scan(inc);
        const unsigned m = __ballot_sync(0xFFFFFFFFu, in && (!ok || A + incl >= kTwo24));
        if (!m) {
            s = grid_value(uu, A + __shfl_sync(0xFFFFFFFFu, incl, 31));
            break;
        }
        const int L = __ffs(m) - 1;
        uint32_t excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
        if (lane == 0) excl = 0u;
        s = grid_value(uu, A + __shfl_sync(0xFFFFFFFFu, excl, L));
        const uint32_t bw = (uint32_t)L;
        const uint32_t pen4 = pen ? (wb[4 * bw + (lane >> 3)] >> (4 * (lane & 7))) & 15u : 0u;
        float4 q = tq[0];
#pragma unroll
        for (int j = 1; j < 8; ++j)
            if ((uint32_t)j == bw) q = tq[j];
        s = warp_walk_block(q, pen4, P.repetition_penalty, inv_t, M, tp.xthr, s, tab, events, ser);
        ++*walks;
        b0 = bw + 1;
    }
    return s;
}

// One warp per row: the exact softmax denominator (ops.rs:408-411) in index order, from the
// tile results where the running sum stays on a grid a tile was classified for, stepping
// through the tile's blocks otherwise.  Writes S (or a failed bound: the row goes to
// lrs_sample_rows).
__global__ void __launch_bounds__(kSumWarps * 32) lrs_stage_sum(const StageArgs S) {
    __shared__ uint32_t wbits[kSumWarps * 32];
    __shared__ float wser[kSumWarps * 128];  // (a warp's block values for a one-lane sum)
    const lrs_kernel_args_t& a = S.a;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t r = blockIdx.x * kSumWarps + warp;
    if (r >= a.rows || *(volatile const uint32_t*)S.live_count == 0u) return;
    RowPrep* rpp = S.rprep + r;
    const uint32_t flags = rpp->flags;
    if (flags & (kRowDone | kRowFallback)) return;
    const long long t_start = clock64();
    uint32_t walks = 0, events = 0;
    const ExpTable exptab{a.exp_index, a.exp_entries, a.exp_near};
    const lrs_params P = a.params[r];
    const Geo g = row_geometry(a, r);
    const float M = rpp->M, inv_t = rpp->inv_t;
    const bool pen_on = P.repetition_penalty != 1.0f;
    const uint32_t hlen = (pen_on && a.hist_len) ? a.hist_len[r] : 0u;
    const uint32_t* hrow = a.hist ? a.hist + (uint64_t)r * a.hist_ld : nullptr;
    const uint32_t hstart = window_start(P, hlen);
    uint32_t* wb = wbits + warp * 32;
    const uint32_t edges = g.head + g.tail;
    const bool mine = (uint32_t)lane < edges;
    const uint32_t egi = (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
    float ex = mine ? g.row[egi] : 0.0f;
    for (uint32_t e = 0; e < edges; ++e) {
        const uint32_t gi = __shfl_sync(0xFFFFFFFFu, egi, (int)e);
        const bool hit = pen_on && in_window(hrow, hstart, hlen, gi);
        if (hit && (uint32_t)lane == e) ex = penalise(ex, P.repetition_penalty);
    }
    float de = 0.0f, ee = 0.0f;
    bool exe = true;
    if (mine) {
        de = d_of(ex, inv_t, M);
        exe = de == 0.0f;
        ee = exe ? 1.0f : expf(de);
    }
    const uint32_t nt = g.nchunks;
    // the tiles likely to be stepped through, brought into L2 ahead of the scan (a lane a 128-byte line)
    for (uint32_t t0 = 0; t0 < nt; t0 += 32) {
        const uint32_t t = t0 + (uint32_t)lane;
        bool want = false;
        if (t < nt) {
            const uint32_t pf = S.tprep[(uint64_t)r * S.nt + t].flags, rf = S.tres[(uint64_t)r * S.nt + t].flags;
            want = t == 0 || (pf & (kTileWalk | kTileLikelyWalk)) ||
                   ((rf & kTileLive) && (rf & (kTileSp0 | kTileSp1)) == (kTileSp0 | kTileSp1));
        }
        for (unsigned m = __ballot_sync(0xFFFFFFFFu, want); m; m &= m - 1u) {
            const uint32_t tw = t0 + (uint32_t)(__ffs(m) - 1);
            if ((uint32_t)lane * 32u < chunk_count(g, tw)) prefetch_l2(g.row + g.head + tw * kTile + lane * 32u);
        }
    }
    // the head opens the sum
    float s = warp_serial_add(0.0f, ee, de, exe, 0, (int)g.head, exptab);
    bool bad = false;
    for (uint32_t t0 = 0; t0 < nt;) {
        const uint32_t t = t0 + (uint32_t)lane;
        const bool in = t < nt;
        uint32_t rflags = 0, rt0 = 0, rt1 = 0;
        int u0 = 0;
        if (in) {
            const TileRes* rs = S.tres + (uint64_t)r * S.nt + t;
            rflags = rs->flags;
            rt0 = rs->t0;
            rt1 = rs->t1;
            u0 = S.tprep[(uint64_t)r * S.nt + t].u0;
        }
        const int uu = unit_exp(s);
        const uint32_t A = grid_count(s, uu);
        // a tile applies in one step when the running sum stays on a grid it was classified for
        uint32_t inc = 0;
        bool ok = !in || !(rflags & kTileLive);
        if (in && (rflags & kTileLive)) {
            if (uu == u0 && !(rflags & kTileSp0)) {
                inc = rt0;
                ok = true;
            } else if (uu == u0 + 1 && !(rflags & kTileSp1)) {
                inc = rt1;
                ok = true;
            }
        }
        const uint32_t incl = warp_incl_scan(inc);
        // a tile whose rigorous lower grid lies above the running sum's breaks the bound that
        // made its dead elements dead: checked below with the exact sum
        const bool stop = in && (!ok || A + incl >= kTwo24 || u0 > uu);
        const unsigned m = __ballot_sync(0xFFFFFFFFu, stop);
        if (!m) {
            s = grid_value(uu, A + __shfl_sync(0xFFFFFFFFu, incl, 31));
            t0 += 32;
            continue;
        }
        const int L = __ffs(m) - 1;
        uint32_t excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
        if (lane == 0) excl = 0u;
        s = grid_value(uu, A + __shfl_sync(0xFFFFFFFFu, excl, L));
        const uint32_t tw = t0 + (uint32_t)L;
        if (unit_exp(s) < __shfl_sync(0xFFFFFFFFu, u0, L)) {  // the estimate's lower bound failed
            bad = true;
            break;
        }
        s = warp_tile_blocks(S, g, r, tw, s, P, inv_t, M, hrow, hstart, hlen, wb, exptab, &events, &walks,
                             wser + warp * 128);
        t0 = tw + 1;
    }
    // the tail closes the sum
    if (!bad) s = warp_serial_add(s, ee, de, exe, (int)g.head, (int)g.tail, exptab);
    if (lane == 0) {
        if (bad) {
            rpp->flags = flags | kRowFallback;
            stage_fallback(S, r);
        } else {
            rpp->pad[0] = __float_as_uint(s);
            rpp->pad[1] = events;
        }
        const long long dt = clock64() - t_start;
        rpp->cyc_sum = dt > 0xFFFFFFFFll ? 0xFFFFFFFFu : (uint32_t)dt;
        rpp->walks = walks;
    }
}

// ----------------------------------------------------------------- finish ----
// A top-p row whose nucleus the finish cannot hold goes to lrs_stage_big when it can take it,
// else to lrs_sample_rows.
__device__ __forceinline__ void stage_big_or_fallback(const StageArgs& S, uint32_t r, uint32_t n) {
    if (S.big_rows && n <= kStageMaxTiles * (uint32_t)kTile) {
        S.rprep[r].flags |= kRowBig;
        S.big_rows[atomicAdd(S.big_count, 1u)] = r;
    } else {
        stage_fallback(S, r);
    }
}

// A top-p row whose nucleus is deeper than its list (sampler.rs:135-146): the CTA counts the
// row's elements by d = fl(x' - M) in buckets of 1/4 over d in (-18, 0] and gathers the exact
// keys (p desc, index asc) of every element above the deepest bucket edge whose elements fit
// in the list's capacity (level 0).  If the nucleus reaches past that edge, level 1 counts the
// next bucket in steps of 1/32 and gathers down to the deepest of those edges that fits.
// Returns the number of keys (cand: the edge), or 0xFFFFFFFF if no deeper edge fits.  The
// finish checks that the nucleus lies inside them.  The counts are private to each thread (a
// column of the keys area per thread, no atomics); split and base (the bucket that overflows
// and the count above it) carry from level 0 to level 1.
constexpr int kRgCoarse = 72;  // buckets of 1/4: d in (-18, 0]
__device__ __noinline__ uint32_t regather_nucleus(const StageArgs& S, uint32_t r, const lrs_params& P, float M, float inv,
                                                  const ExpTable tab, unsigned long long* keys, RowShared& sh,
                                                  float& cand, int level, int& split, uint32_t& base) {
    static_assert(kRgCoarse * kThreads + kRgCoarse + 8 <= 2 * (int)kStageListCap, "regather counts fit the keys");
    const lrs_kernel_args_t& a = S.a;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Geo g = row_geometry(a, r);
    const float inv_t = __fdiv_rn(1.0f, P.temperature);
    const bool pen_on = P.repetition_penalty != 1.0f;
    const uint32_t hlen = (pen_on && a.hist_len) ? a.hist_len[r] : 0u;
    const uint32_t* hrow = a.hist ? a.hist + (uint64_t)r * a.hist_ld : nullptr;
    const uint32_t hstart = window_start(P, hlen);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(keys);  // [bucket][kThreads]
    uint32_t* tot = cnt + kRgCoarse * kThreads;          // [kRgCoarse] coarse totals, then [8] fine
    uint32_t* wb = sh.hist256 + warp * 32;                // (the warp's window words)
    if (level == 0) {
        // the whole row into L2 ahead of the passes (a thread a 128-byte line at a time)
        for (uint64_t q = (uint64_t)tid * 32u; q < g.n; q += (uint64_t)kThreads * 32u) prefetch_l2(g.row + q);
    }
    // floor(-d * sc) for d in (-18, 0] (sc a power of two: the product is exact), from the
    // bits of fl_rd(-d * sc + 2^23); 0xFFFF past -18 and for NaN
    auto bucket = [](float d, float sc) -> uint32_t {
        return d > -18.0f ? (__float_as_uint(__fadd_rd(__fmul_rn(d, -sc), 8388608.0f)) & 0x7FFFFFu) : 0xFFFFu;
    };
    // mode 0: coarse counts; mode 1: fine counts in coarse bucket cb; mode 2: gather d >= th
    auto visit = [&](int mode, uint32_t cb, float th) {
        // the tiles, then the edge elements as item nchunks (lanes 0 .. edges-1); warp w takes
        // items w, w + 7, ...
        const uint32_t edges = g.head + g.tail;
        for (uint32_t t = (uint32_t)warp; t <= g.nchunks; t += kWarps) {
            const bool edge = t == g.nchunks;
            float v[32];
            uint32_t g0 = 0;
            if (!edge) {
                // the warp's next tile into L1 while this one is counted (a line per lane)
                const uint32_t tn = t + kWarps;
                if (tn < g.nchunks && (uint32_t)lane * 32u < chunk_count(g, tn))
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(g.row + g.head + tn * kTile + lane * 32u));
                const uint32_t c = chunk_count(g, t);
                g0 = g.head + t * kTile;
                bool pen = false;
                if (pen_on && hlen) pen = tile_window(hrow, hstart, hlen, g0, c, wb);
                load_tile_blocks(g.row + g0, c, pen, wb, P.repetition_penalty, v);
            } else {
                const uint32_t egi = (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
                float x = (uint32_t)lane < edges ? g.row[egi] : __int_as_float(0xFF800000);
                for (uint32_t e = 0; e < edges; ++e) {
                    const uint32_t gi = __shfl_sync(0xFFFFFFFFu, egi, (int)e);
                    const bool hit = pen_on && in_window(hrow, hstart, hlen, gi);
                    if (hit && (uint32_t)lane == e) x = penalise(x, P.repetition_penalty);
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __int_as_float(0xFF800000);
                v[0] = x;
            }
            if (mode == 0) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const uint32_t b = bucket(d_of(v[i], inv_t, M), 4.0f);
                    if (b < (uint32_t)kRgCoarse) ++cnt[b * kThreads + tid];
                }
            } else if (mode == 1) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const uint32_t b = bucket(d_of(v[i], inv_t, M), 32.0f);
                    if ((b >> 3) == cb) ++cnt[(b & 7u) * kThreads + tid];
                }
            } else {
                // count, one reservation per warp and tile, then the writes in the lane's order
                uint32_t mine = 0;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    v[i] = d_of(v[i], inv_t, M);
                    mine += v[i] >= th ? 1u : 0u;
                }
                const uint32_t incl = warp_incl_scan_plain(mine);
                const uint32_t wtot = __shfl_sync(0xFFFFFFFFu, incl, 31);
                if (wtot == 0u) continue;
                uint32_t wbase = 0;
                if (lane == 31) wbase = atomicAdd(&sh.misc[1], wtot);
                uint32_t o = __shfl_sync(0xFFFFFFFFu, wbase, 31) + incl - mine;
                if (mine == 0u) continue;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (v[i] >= th) {
                        uint32_t gi;
                        if (!edge)
                            gi = g0 + 128u * (i >> 2) + 4u * lane + (i & 3);
                        else
                            gi = (uint32_t)lane < g.head ? (uint32_t)lane : g.head + g.body + ((uint32_t)lane - g.head);
                        if (o < kStageListCap)  // (d now; its key once every element is in)
                            keys[o] = ((unsigned long long)__float_as_uint(v[i]) << 32) | gi;
                        ++o;
                    }
                }
            }
        }
    };
    // the totals of nb private columns into out[0 .. nb) (a warp per bucket)
    auto reduce = [&](int nb, uint32_t* out) {
        for (int b = warp; b < nb; b += kWarps) {
            uint32_t c = 0;
#pragma unroll
            for (int q = 0; q < kWarps; ++q) c += cnt[b * kThreads + lane + 32 * q];
            c = __reduce_add_sync(0xFFFFFFFFu, c);
            if (lane == 0) out[b] = c;
        }
    };
    // warp 0: the deepest bucket of c[0 .. nb) whose prefix count, from base0, fits in the list
    auto deepest = [&](const uint32_t* c, int nb, uint32_t base0) -> int {
        uint32_t acc = base0;
        int best = -1;
        for (int b0 = 0; b0 < nb; b0 += 32) {
            const int b = b0 + lane;
            const uint32_t ci = warp_incl_scan_plain(b < nb ? c[b] : 0u) + acc;
            const unsigned fit = __ballot_sync(0xFFFFFFFFu, b < nb && ci <= kStageListCap);
            if (fit) best = b0 + 31 - __clz(fit);
            acc = __shfl_sync(0xFFFFFFFFu, ci, 31);
            if (acc > kStageListCap) break;
        }
        return best;
    };
    if (tid == 0) sh.misc[1] = 0u;  // (the gather's key counter)
    int edge_b;  // the deepest fine bucket (1/32) above the edge
    if (level == 0) {
#pragma unroll
        for (int b = 0; b < kRgCoarse; ++b) cnt[b * kThreads + tid] = 0u;  // (its own column)
        visit(0, 0u, 0.0f);
        csync();
        reduce(kRgCoarse, tot);
        csync();
        if (warp == 0) {
            const int cb = deepest(tot, kRgCoarse, 0u);  // buckets 0 .. cb fit
            uint32_t bs = 0;
            for (int b = lane; b <= cb; b += 32) bs += tot[b];
            bs = __reduce_add_sync(0xFFFFFFFFu, bs);
            if (lane == 0) {
                sh.misc[0] = (uint32_t)(cb + 1);  // the coarse bucket that overflows (kRgCoarse: none)
                sh.misc[2] = bs;
            }
        }
        csync();
        split = (int)sh.misc[0];
        base = sh.misc[2];
        edge_b = split * 8 - 1;
    } else {
        edge_b = -1;
    }
    // level 1, or level 0 when no coarse bucket fits: split the overflowing bucket by 1/32
    if (edge_b < 0 || level == 1) {
        if (split >= kRgCoarse) return 0xFFFFFFFFu;
#pragma unroll
        for (int b = 0; b < 8; ++b) cnt[b * kThreads + tid] = 0u;
        visit(1, (uint32_t)split, 0.0f);
        csync();
        reduce(8, tot + kRgCoarse);
        csync();
        if (warp == 0) {
            const int f = deepest(tot + kRgCoarse, 8, base);
            if (lane == 0) sh.misc[3] = (uint32_t)(f + 1);
        }
        csync();
        const int f = (int)sh.misc[3] - 1;
        if (f < 0) return 0xFFFFFFFFu;  // (no edge deeper than level 0's)
        edge_b = split * 8 + f;
        if (level == 0) split = kRgCoarse;  // (level 0 took the fine edge: level 1 has none deeper)
    }
    cand = -(float)(edge_b + 1) / 32.0f;
    csync();  // (the counts are dead: the gather writes keys)
    visit(2, 0u, cand);
    csync();
    const uint32_t nkeys = sh.misc[1];
    if (nkeys > kStageListCap) return 0xFFFFFFFFu;
    // the keys (p desc, index asc) from the gathered d values, p = fl(libm expf(d) * inv)
    // (four a thread side by side)
    for (uint32_t i0 = tid; i0 < nkeys; i0 += 4u * kThreads) {
        unsigned long long k[4];
        float ev[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t i = i0 + (uint32_t)u * kThreads;
            k[u] = i < nkeys ? keys[i] : 0ull;
            ok[u] = expf_rounded(__uint_as_float((uint32_t)(k[u] >> 32)), tab, ev[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t i = i0 + (uint32_t)u * kThreads;
            if (i < nkeys) {
                const float d = __uint_as_float((uint32_t)(k[u] >> 32));
                const float e = ok[u] ? ev[u] : exact_expf_table(d, tab, ev[u]);
                keys[i] = ((unsigned long long)(~__float_as_uint(__fmul_rn(e, inv))) << 32) | (k[u] & 0xFFFFFFFFull);
            }
        }
    }
    csync();
    return nkeys;
}

// ------------------------------------------------------------------ sort ----
// Ascending sort of n <= kStageListCap 64-bit keys in shared memory by the block.  A warp
// sorts runs of 32 * KPL keys in registers with a bitonic network (lane L holds keys
// KPL L .. KPL L + KPL - 1; every compare-exchange pairs i with i ^ m, m = 2^ls - 1 opening the
// merge of size 2^ls with the mirrored partner, m = 2^lt cleaning; m < KPL pairs registers of
// a lane, larger m pairs lanes by shuffles).  Runs of 256 are then merged pairwise by merge
// path into 16-bit permutations, and the final order is written back through global scratch.
__host__ __device__ constexpr int hibit(int x) { return x >= 2 ? 2 * hibit(x >> 1) : x; }

template <int M, int KPL>
__device__ __forceinline__ void seg_stage(unsigned long long (&k)[KPL], uint32_t lane) {
    if constexpr (M >= KPL) {
        constexpr int mL = M / KPL, mj = M % KPL;      // partner lane lane ^ mL, register j ^ mj
        constexpr uint32_t h = (uint32_t)hibit(mL);    // the lane bit that decides the pair
        const bool lower = (lane & h) == 0u;
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            if constexpr (mj == 0) {
                const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, k[j], mL), x = k[j];
                k[j] = lower ? (o < x ? o : x) : (o < x ? x : o);
            } else if (j < (j ^ mj)) {  // (both registers of a pair are read before either is written)
                const unsigned long long o1 = __shfl_xor_sync(0xFFFFFFFFu, k[j ^ mj], mL);
                const unsigned long long o2 = __shfl_xor_sync(0xFFFFFFFFu, k[j], mL);
                const unsigned long long x1 = k[j], x2 = k[j ^ mj];
                k[j] = lower ? (o1 < x1 ? o1 : x1) : (o1 < x1 ? x1 : o1);
                k[j ^ mj] = lower ? (o2 < x2 ? o2 : x2) : (o2 < x2 ? x2 : o2);
            }
        }
    } else {
        constexpr int H = hibit(M);
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            if (!(j & H)) {
                const unsigned long long x = k[j], y = k[j ^ M];
                k[j] = x < y ? x : y;
                k[j ^ M] = x < y ? y : x;
            }
        }
    }
}

template <int LT, int KPL>
__device__ __forceinline__ void seg_clean(unsigned long long (&k)[KPL], uint32_t lane) {
    if constexpr (LT >= 0) {
        seg_stage<(1 << LT), KPL>(k, lane);
        seg_clean<LT - 1, KPL>(k, lane);
    }
}

// The merges of sizes 2^LS .. 32 KPL: a full sort of the run from LS = 1.
template <int LS, int KPL>
__device__ __forceinline__ void seg_sort(unsigned long long (&k)[KPL], uint32_t lane) {
    if constexpr ((1 << LS) <= 32 * KPL) {
        seg_stage<(1 << LS) - 1, KPL>(k, lane);
        seg_clean<LS - 2, KPL>(k, lane);
        seg_sort<LS + 1, KPL>(k, lane);
    }
}

// The warp sorts keys[b, b + 32 KPL) in place; positions at or past n read as ~0 and are
// written back only below `store`.
template <int KPL>
__device__ __forceinline__ void warp_sort_run(unsigned long long* keys, uint32_t b, uint32_t n, uint32_t store) {
    const uint32_t lane = threadIdx.x & 31u;
    unsigned long long k[KPL];
#pragma unroll
    for (int j = 0; j < KPL; ++j) {
        const uint32_t i = b + KPL * lane + (uint32_t)j;
        k[j] = i < n ? keys[i] : ~0ull;
    }
    seg_sort<1, KPL>(k, lane);
#pragma unroll
    for (int j = 0; j < KPL; ++j) {
        const uint32_t i = b + KPL * lane + (uint32_t)j;
        if (i < store) keys[i] = k[j];
    }
}

// The warp sorts k[0, c) in place, ascending, c <= 1024: a bitonic network over the next power
// of two in shared memory, every compare-exchange ascending (a merge opens with mirrored
// partners), so the positions past c act as +inf and are never read or written.  Loops over
// any c (the big-nucleus buckets); the finish's fixed runs of 256 keep the register network.
__device__ __noinline__ void warp_sort_smem(unsigned long long* k, uint32_t c) {
    const uint32_t lane = threadIdx.x & 31u;
    if (c < 2u) return;
    uint32_t lp = 1;
    while ((1u << lp) < c) ++lp;
    const uint32_t pairs = 1u << (lp - 1);
    for (uint32_t ls = 1; ls <= lp; ++ls) {
        for (int lt = (int)ls - 1; lt >= 0; --lt) {
            const bool open = lt == (int)ls - 1;  // (the merge's first stage: mirrored partners)
            for (uint32_t q = lane; q < pairs; q += 32u) {
                const uint32_t i = ((q >> lt) << (lt + 1)) | (q & ((1u << lt) - 1u));
                const uint32_t j = open ? (i | ((1u << (lt + 1)) - 1u)) - (i & ((1u << lt) - 1u)) : i + (1u << lt);
                if (j < c) {
                    const unsigned long long a = k[i], b = k[j];
                    if (b < a) {
                        k[i] = b;
                        k[j] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// The sorted order: position i holds keys[perm[i]] (keys[i] when perm is null).
struct SortedKeys {
    const unsigned long long* keys;
    const uint16_t* perm;
    __device__ __forceinline__ unsigned long long operator[](uint32_t i) const { return keys[perm ? (uint32_t)perm[i] : i]; }
    __device__ __forceinline__ float p(uint32_t i) const { return __uint_as_float(~(uint32_t)((*this)[i] >> 32)); }
};

// Sorts keys[0, n) (p desc, index asc as an ascending key): returns the order as a view.
__device__ __noinline__ SortedKeys stage_sort_u64(unsigned long long* keys, uint32_t n, uint16_t* pa, uint16_t* pb) {
    const int tid = threadIdx.x, warp = tid >> 5;
    if (n <= 256u) {
        if (n >= 2u && warp == 0) {
            if (n <= 64u)
                warp_sort_run<2>(keys, 0u, n, n);
            else
                warp_sort_run<8>(keys, 0u, n, n);
        }
        csync();
        return SortedKeys{keys, nullptr};
    }
    const uint32_t n2 = (n + 255u) & ~255u;  // (runs of 256; the pads sort last)
    for (uint32_t sg = (uint32_t)warp; sg < (n2 >> 8); sg += kWarps) warp_sort_run<8>(keys, sg << 8, n, n2);
    csync();
    // Merge levels: runs of L into runs of 2L.  A thread writes E consecutive outputs, E odd
    // so that the threads' positions fall in different shared-memory banks (a thread's range
    // may cross from one pair of runs into the next).
    uint32_t E = (n2 + kThreads - 1) / kThreads;
    E |= 1u;
    const uint16_t* src = nullptr;  // (level 1 reads the runs in place)
    uint16_t* dst = pa;
    for (uint32_t L = 256; L < n2; L <<= 1) {
        auto key_at = [&](uint32_t q) -> unsigned long long { return keys[src ? (uint32_t)src[q] : q]; };
        const uint32_t q_begin = (uint32_t)tid * E, q_end = q_begin + E < n2 ? q_begin + E : n2;
        for (uint32_t q = q_begin; q < q_end;) {
            const uint32_t base = q & ~(2u * L - 1u), k0 = q - base;
            const uint32_t len = n2 - base < 2u * L ? n2 - base : 2u * L;
            const uint32_t lenA = len < L ? len : L, lenB = len - lenA;
            const uint32_t A = base, B = base + lenA;
            const uint32_t cnt = (q_end < base + len ? q_end : base + len) - q;
            // merge path: i elements of A among the first k0 outputs of the pair (ties: A first)
            uint32_t lo = k0 > lenB ? k0 - lenB : 0u, hi = k0 < lenA ? k0 : lenA;
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (key_at(A + mid) <= key_at(B + k0 - 1u - mid)) lo = mid + 1u; else hi = mid;
            }
            uint32_t i = lo, j = k0 - lo;
            unsigned long long ka = i < lenA ? key_at(A + i) : 0ull, kb = j < lenB ? key_at(B + j) : 0ull;
            for (uint32_t e = 0; e < cnt; ++e) {
                const bool takeA = i < lenA && (j >= lenB || ka <= kb);
                const uint32_t qq = takeA ? A + i : B + j;
                dst[q + e] = (uint16_t)(src ? (uint32_t)src[qq] : qq);
                if (takeA) {
                    ++i;
                    ka = i < lenA ? key_at(A + i) : 0ull;
                } else {
                    ++j;
                    kb = j < lenB ? key_at(B + j) : 0ull;
                }
            }
            q += cnt;
        }
        csync();
        src = dst;
        dst = dst == pa ? pb : pa;
    }
    // the order into place: every thread holds its keys in registers across the barrier
    constexpr int kPer = (int)((kStageListCap + kThreads - 1) / kThreads);
    unsigned long long v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = (uint32_t)tid + (uint32_t)j * kThreads;
        v[j] = i < n ? keys[src[i]] : 0ull;
    }
    csync();
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const uint32_t i = (uint32_t)tid + (uint32_t)j * kThreads;
        if (i < n) keys[i] = v[j];
    }
    csync();
    return SortedKeys{keys, nullptr};
}

// Exclusive prefix of small per-thread counts in thread order over the block; total: the sum.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t c, uint32_t* shw, uint32_t& total) {
    const uint32_t incl = warp_incl_scan_plain(c);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    csync();
    if (l == 31) shw[w] = incl;
    csync();
    uint32_t before = 0, tot = 0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) {
        const uint32_t x = shw[i];
        before += i < w ? x : 0u;
        tot += x;
    }
    total = tot;
    return before + incl - c;
}

// A long top-p list (sampler.rs:135-146) before its sort: the mass of its keys by probability
// bucket (1/8 binade below the row's largest probability inv), the first bucket where the
// mass reaches top_p + 2^-11, and the keys of the buckets down to the next one moved to the
// front (in no particular order).  Returns their number m (n: every key stays), and in
// p_left the largest probability of a key left out.  The finish checks that the cut lies
// among the first m in sorted order, above p_left; the buckets only choose m.  hist: 7 x 256
// floats of shared memory.
constexpr uint32_t kPrefilterMin = 512;  // lists shorter than this are sorted whole
__device__ __noinline__ uint32_t nucleus_prefilter(unsigned long long* keys, uint32_t n, float top_p, float inv,
                                                   float* hist, RowShared& sh, float& p_left) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t ib = __float_as_uint(inv);
    auto bucket = [ib](unsigned long long k) -> uint32_t {
        const uint32_t pb = ~(uint32_t)(k >> 32);
        const uint32_t b = ib > pb ? (ib - pb) >> 20 : 0u;
        return b < 255u ? b : 255u;
    };
    for (int i = tid; i < kWarps * 256; i += kThreads) hist[i] = 0.0f;
    csync();
    float* wh = hist + warp * 256;
    for (uint32_t i = tid; i < n; i += kThreads) {
        const unsigned long long k = keys[i];
        atomicAdd(&wh[bucket(k)], __uint_as_float(~(uint32_t)(k >> 32)));
    }
    csync();
    for (int b = tid; b < 256; b += kThreads) {  // (column b: only this thread reads or writes it)
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) t += hist[w * 256 + b];
        hist[b] = t;
    }
    csync();
    if (warp == 0) {
        const double target = (double)top_p + 0x1p-11;
        double acc = 0.0;
        int found = 255;
        for (int b0 = 0; b0 < 256; b0 += 32) {
            double mi = (double)hist[b0 + lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double tv = __shfl_up_sync(0xFFFFFFFFu, mi, o);
                if (lane >= o) mi += tv;
            }
            const unsigned hit = __ballot_sync(0xFFFFFFFFu, acc + mi >= target);
            if (hit) {
                found = b0 + __ffs(hit) - 1;
                break;
            }
            acc += __shfl_sync(0xFFFFFFFFu, mi, 31);
        }
        if (lane == 0) sh.misc[4] = (uint32_t)(found + 1);  // (one bucket of margin)
    }
    csync();
    const uint32_t bsel = sh.misc[4];
    if (bsel >= 255u) return n;
    // compaction in waves of 8 keys a thread: every key of a wave is read before any is
    // written, and a wave writes only below its own end
    uint32_t m = 0, pl = 0;
    for (uint32_t w0 = 0; w0 < n; w0 += 8u * kThreads) {
        unsigned long long v[8];
        uint32_t c = 0, selm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t i = w0 + 8u * tid + (uint32_t)j;
            v[j] = i < n ? keys[i] : 0ull;
            const bool in = i < n;
            const bool sel = in && bucket(v[j]) <= bsel;
            if (sel) {
                selm |= 1u << j;
                ++c;
            } else if (in) {
                const uint32_t pb = ~(uint32_t)(v[j] >> 32);
                pl = pb > pl ? pb : pl;
            }
        }
        uint32_t total;
        uint32_t o = m + block_excl_scan(c, sh.red, total);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (selm & (1u << j)) keys[o++] = v[j];
        m += total;
        csync();
    }
    pl = __reduce_max_sync(0xFFFFFFFFu, pl);
    if (lane == 0) sh.red2[warp] = pl;
    csync();
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) r = sh.red2[i] > r ? sh.red2[i] : r;
    csync();
    p_left = __uint_as_float(r);  // (positive floats order as their bits)
    return m;
}

// The sequential f32 run over keys[0, cnt) (p in the high word, inverted) by thread 0, eight
// values a step with their loads issued a step ahead (sampler.rs:137-145 for DIR > 0, stop at
// s >= thr; sampler.rs:156-161 for DIR < 0, stop at s <= 0).  Returns the stop position or
// -1; s: the value after it (or after the run).  Same values for every thread.
template <int DIR>
__device__ __forceinline__ float big_step(float c, float v) {
    if constexpr (DIR > 0) return __fadd_rn(c, v); else return __fsub_rn(c, v);
}
template <int DIR>
__device__ __forceinline__ bool big_hit(float c, float thr) {
    if constexpr (DIR > 0) return c >= thr; else return c <= 0.0f;
}
__device__ __forceinline__ float big_p(const unsigned long long* keys, uint32_t i, uint32_t cnt) {
    return i < cnt ? __uint_as_float(~(uint32_t)(keys[i] >> 32)) : 0.0f;
}
template <int DIR>
__device__ __forceinline__ int big_serial(const unsigned long long* keys, uint32_t cnt, float& s, float thr,
                                          RowShared& sh) {
    if (threadIdx.x == 0) {
        float cur = s;
        int stop = -1;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = big_p(keys, (uint32_t)j, cnt);
        for (uint32_t i = 0; i < cnt; i += 8) {
            float nx[8], c[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) nx[j] = big_p(keys, i + 8u + (uint32_t)j, cnt);
            // (positions past cnt add 0: they neither move s nor stop it)
            c[0] = big_step<DIR>(cur, v[0]);
#pragma unroll
            for (int j = 1; j < 8; ++j) c[j] = big_step<DIR>(c[j - 1], v[j]);
            if (big_hit<DIR>(c[7], thr)) {
                int f = 7;
#pragma unroll
                for (int j = 6; j >= 0; --j) f = big_hit<DIR>(c[j], thr) ? j : f;
                float cf = c[7];
#pragma unroll
                for (int j = 6; j >= 0; --j) cf = f == j ? c[j] : cf;
                stop = (int)i + f;
                cur = cf;
                break;
            }
            cur = c[7];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = nx[j];
        }
        sh.fstate = cur;
        sh.stop = stop;
    }
    csync();
    s = sh.fstate;
    const int st = sh.stop;
    csync();
    return st;
}

// Sequential f32 run over sorted probabilities keys[0..cnt) (sampler.rs:137-139 / 148-151 /
// 156-158): dir > 0 adds until s >= thr, dir < 0 subtracts until s <= 0.  The first 512
// positions go one by one on thread 0, the rest chunk by chunk with the block's exact
// emulation (acc_tile).
// Returns the stop position or -1; every thread gets the same s.
__device__ __noinline__ int sorted_run(const SortedKeys keys, uint32_t cnt, int dir, float& s, float thr,
                                       RowShared& sh, uint32_t head_max = 512u) {
    // (the head of a sorted run holds its largest elements, nearly every one an ordered step
    // of the emulation: it goes one by one; the emulation takes the rest)
    const uint32_t head = cnt < head_max ? cnt : head_max;
    if (!keys.perm) {  // (keys in order: the scalar walker)
        const int st = dir > 0 ? big_serial<+1>(keys.keys, head, s, thr, sh) : big_serial<-1>(keys.keys, head, s, 0.0f, sh);
        if (st >= 0 || head == cnt) return st;
    } else {
        if (threadIdx.x == 0) {
            // Groups of eight: the sum steps through a group with no branch, and the stop test
            // runs once per group (the run is monotone: p >= 0), then finds the first position
            // inside it.  Positions past the head add 0, which neither moves s nor stops it.
            auto p_at = [&](uint32_t i) -> float {
                return i < head ? keys.p(i) : 0.0f;
            };
            float cur = s;
            int stop = -1;
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = p_at((uint32_t)j);
            for (uint32_t i0 = 0; i0 < head; i0 += 8) {
                float nv[8], c[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) nv[j] = p_at(i0 + 8u + (uint32_t)j);  // (the next group)
                if (dir > 0) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) c[j] = cur = __fadd_rn(cur, v[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) c[j] = cur = __fsub_rn(cur, v[j]);
                }
                if (dir > 0 ? cur >= thr : cur <= 0.0f) {
                    int j = 7;
#pragma unroll
                    for (int q = 6; q >= 0; --q)
                        if (dir > 0 ? c[q] >= thr : c[q] <= 0.0f) j = q;
                    stop = (int)i0 + j;
                    cur = c[j];
                    break;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = nv[j];
            }
            sh.fstate = cur;
            sh.stop = stop;
        }
        csync();
        s = sh.fstate;
        const int st = sh.stop;
        csync();
        if (st >= 0 || head == cnt) return st;
    }
    for (uint32_t b = head; b < cnt; b += kChunk) {
        const uint32_t tc = cnt - b < (uint32_t)kChunk ? cnt - b : (uint32_t)kChunk;
        float v[kVpt];
#pragma unroll
        for (int i = 0; i < kVpt; ++i) {  // (load_sorted_tile's layout, through the order)
            const int li = li_of(i);
            v[i] = (uint32_t)li < tc ? keys.p(b + (uint32_t)li) : 0.0f;
        }
        uint32_t ex = 0xFFFFFFFFu;
        const int st = acc_tile(v, ex, (int)tc, dir, s, thr, NoExact(), sh);
        if (st >= 0) return (int)b + st;
    }
    return -1;
}

// One CTA per row: the candidates' exact probabilities p = fl(libm expf(d) * (1 / S))
// (sampler.rs:129-131, ops.rs:409-416), sorted (p desc, index asc), then top-k, the top-p
// cut, the survivor sum and the draw (sampler.rs:122-162).
__global__ void __maxnreg__(144) lrs_stage_finish(const StageArgs S) {  // (2 CTAs of kThreads per SM)
    extern __shared__ __align__(16) unsigned long long keys[];  // kStageListCap, then the sort's permutations
    uint16_t* perm = reinterpret_cast<uint16_t*>(keys + kStageListCap);  // 2 x kStageListCap
    __shared__ RowShared sh;
    const lrs_kernel_args_t& a = S.a;
    const uint32_t r = blockIdx.x;
    const int tid = threadIdx.x;
    const RowPrep rp = S.rprep[r];
    if (rp.flags & (kRowDone | kRowFallback | kRowBig)) return;
    const long long t_start = clock64();
    const uint32_t nk = S.list_n[r];
    if (nk > kStageListCap && (rp.flags & kRowPathK)) {  // a top-k list overflow (ties): lrs_sample_rows
        if (tid == 0) stage_fallback(S, r);
        return;
    }
    const float kInf = __int_as_float(0x7F800000);
    const ExpTable exptab{a.exp_index, a.exp_entries, a.exp_near};
    const lrs_params P = a.params[r];
    const float M = rp.M;
    const float Ssum = __uint_as_float(rp.pad[0]);
    const float inv = __fdiv_rn(1.0f, Ssum);  // ops.rs:413
    const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;
    if (tid == 0) {
        sh.misc[7] = 0u;
        sh.events = 0u;
    }
    uint32_t n_keys = nk;
    float cand = rp.cand;
    float cum = 0.0f;
    int stp = -1;
    uint32_t kk = 0, cut = 0;
    long long c_regather = 0, c_sort = 0, c_runs = 0, tm = 0;  // (diagnostics: cycles by phase)
    SortedKeys sk{keys, nullptr};
    int split = 0;       // (the regather's levels: the coarse bucket that overflows the list ...)
    uint32_t above = 0;  // (... and the count above it)
    // attempt 0: the list; 1: the regather at a coarse edge; 2: at a fine edge
    for (int attempt = nk > kStageListCap ? 1 : 0; attempt < 3; ++attempt) {
        if (attempt == 0) {
            const uint2* lst = S.lists + (uint64_t)r * kStageListCap;
            // (four entries a thread side by side: the exps' chains overlap)
            for (uint32_t i0 = tid; i0 < nk; i0 += 4u * kThreads) {
                uint2 en[4];
                float d[4], ev[4];
                bool ok[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t i = i0 + (uint32_t)u * kThreads;
                    en[u] = i < nk ? lst[i] : make_uint2(__float_as_uint(M), 0u);
                    d[u] = __fsub_rn(__uint_as_float(en[u].x), M);
                    ok[u] = expf_rounded(d[u], exptab, ev[u]);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t i = i0 + (uint32_t)u * kThreads;
                    if (i < nk) {
                        const float e = ok[u] ? ev[u] : exact_expf_table(d[u], exptab, ev[u]);
                        const float p = __fmul_rn(e, inv);
                        keys[i] = ((unsigned long long)(~__float_as_uint(p)) << 32) | en[u].y;
                    }
                }
            }
        } else {
            // The nucleus reaches deeper than the list: gather it from the row down to a bucket
            // edge whose elements fit in the list's capacity.
            csync();
            tm = clock64();
            n_keys = regather_nucleus(S, r, P, M, inv, exptab, keys, sh, cand, attempt - 1, split, above);
            c_regather += clock64() - tm;
            if (n_keys == 0xFFFFFFFFu) {  // (deeper than the list's capacity)
                if (tid == 0) stage_big_or_fallback(S, r, a.n);
                return;
            }
        }
        // pass 0 of a long top-p list sorts only the head the prefilter keeps; pass 1 the
        // whole list again (from its copy in the row's list area) if the cut is not inside it
        bool inside = false;
        float short_by = 0.0f;  // (the whole list sorted short of top_p: the mass still missing / p_lim)
        for (int pass = 0; pass < 2 && !inside; ++pass) {
            uint32_t m_keys = n_keys;
            float p_left = 0.0f;
            unsigned long long* backup = reinterpret_cast<unsigned long long*>(S.lists + (uint64_t)r * kStageListCap);
            csync();
            if (pass == 0 && (rp.flags & kRowPathN) && topp_on && n_keys >= kPrefilterMin) {
                for (uint32_t i = tid; i < n_keys; i += kThreads) __stcg(backup + i, keys[i]);
                m_keys = nucleus_prefilter(keys, n_keys, P.top_p, inv, reinterpret_cast<float*>(perm), sh, p_left);
            } else if (pass == 1) {
                for (uint32_t i = tid; i < n_keys; i += kThreads) keys[i] = __ldcg(backup + i);
            }
            csync();
            tm = clock64();
            sk = stage_sort_u64(keys, m_keys, perm, perm + kStageListCap);  // (p desc, index asc): the reference's order
            c_sort += clock64() - tm;
            kk = rp.k < m_keys ? rp.k : m_keys;  // (path K: the list holds the top k; path N: the nucleus)
            // top-p over the first kk (sampler.rs:135-146); the survivor sum is the same sequence
            // up to the cutoff (sampler.rs:148-151)
            cum = 0.0f;
            tm = clock64();
            stp = sorted_run(sk, kk, +1, cum, topp_on ? P.top_p : kInf, sh);
            c_runs += clock64() - tm;
            cut = stp >= 0 ? (uint32_t)stp + 1 : kk;
            if (rp.flags & kRowPathK) {
                inside = true;
                break;
            }
            // path N: the list holds every element with d >= cand (every element, when it is the
            // whole row), so its sorted order is the row's as far as its probabilities exceed the
            // largest one an element outside can have (p_out), and the largest one the prefilter
            // left out; the cut (top_p reached, or k reached) must lie there
            const bool whole = n_keys >= a.n;
            const float p_out = whole ? 0.0f : __fmul_rn(exact_expf(cand, exptab), inv);
            const float p_lim = fmaxf(p_out, p_left);
            const bool complete = whole && m_keys == n_keys;
            inside = complete || ((stp >= 0 || kk == rp.k) && cut > 0 && sk.p(cut - 1) > p_lim);
            if (!inside && stp < 0 && m_keys == n_keys && kk < rp.k && p_lim > 0.0f)
                short_by = (float)(((double)P.top_p - (double)cum * 1.001) / (double)p_lim);
            if (m_keys == n_keys) break;  // (no second pass without a prefilter)
        }
        if (inside) break;
        // Every element outside the list has a probability of at most p_lim, so the nucleus holds
        // at least short_by more elements than the list: when no list can hold it, lrs_stage_big
        // takes the row now (a regather would fail).
        if (topp_on && (double)n_keys + (double)short_by > (double)kStageListCap) {
            if (tid == 0) stage_big_or_fallback(S, r, a.n);
            return;
        }
        if (attempt == 2) {
            if (tid == 0) stage_big_or_fallback(S, r, a.n);
            return;
        }
    }
    unsigned long long st = a.state[r];
    uint32_t ps = 0;
    float r0 = 0.0f;
    if (cum > 0.0f) {
        r0 = __fmul_rn(next_f32(&st), cum);  // sampler.rs:155
        float rv = r0;
        tm = clock64();
        const int w = sorted_run(sk, cut, -1, rv, 0.0f, sh);
        c_runs += clock64() - tm;
        ps = w >= 0 ? (uint32_t)w : cut - 1;  // sampler.rs:156-162
    }
    if (tid != 0) return;
    if (sh.misc[7]) {  // (an internal bound of the exact emulation failed: should not happen)
        stage_fallback(S, r);
        return;
    }
    const unsigned long long chosen = sk[ps];
    lrs_row_info inf = blank_info(2u, rp.k);
    inf.token = (uint32_t)(chosen & 0xFFFFFFFFu);
    inf.prob = __uint_as_float(~(uint32_t)(chosen >> 32));
    inf.cutoff = cut;
    inf.pos = ps;
    inf.max = M;
    inf.sum_exp = Ssum;
    inf.surv_sum = cum;
    inf.r0 = r0;
    inf.n_cand = n_keys;
    inf.events = rp.pad[1];
    inf.cycles[0] = rp.cyc_prep;  // (implementation detail: the stages' SM cycles and walked blocks)
    inf.cycles[1] = rp.cyc_sum;
    const long long dt = clock64() - t_start;
    inf.cycles[2] = dt > 0xFFFFFFFFll ? 0xFFFFFFFFu : (uint32_t)dt;
    inf.cycles[4] = 1u;  // (finished by the staged pipeline)
    inf.cycles[5] = rp.walks;
    auto sat = [](long long v) -> uint32_t { return v > 0xFFFFFFFFll ? 0xFFFFFFFFu : (uint32_t)v; };
    inf.cycles[3] = sat(c_regather);
    inf.cycles[6] = sat(c_sort);
    inf.cycles[7] = sat(c_runs);
    write_row(a, r, LRS_OK, inf.token, inf.prob, true, st, inf);
}

// ------------------------------------------------------------- big nuclei ----
// A top-p row whose nucleus cannot fit in a list (flat rows: nuclei of 10^5 tokens,
// sampler.rs:132-146) is sampled by lrs_stage_big, one CTA per row, after the sum stage
// has given its exact denominator S:
//   1. every element's exact p = fl(libm expf(d) * fl(1/S)) (ops.rs:409-416) is counted in
//      a bucket of its bits below those of the largest p (fl(1/S)): 2^kBigShift float steps
//      (1/256 binade) a bucket, kBigBuckets - 1 of them (32 binades), the last taking every
//      smaller p;
//      CUDA's expf decides the bucket where it cannot differ from libm's value;
//   2. the keys (p desc, index asc as an ascending 64-bit key) are scattered bucket by bucket
//      into the CTA's scratch (a counting sort: the buckets are in key order);
//   3. the top-p sum (sampler.rs:137-145) runs over chunks of whole buckets: a chunk's buckets
//      are sorted in shared memory (a warp a bucket), written back, and summed by the exact
//      emulation of the sequential f32 sum (acc_tile);
//   4. the draw (sampler.rs:155-162) runs over the sorted survivors the same way.
// A row whose walk reaches the last bucket, or whose bucket is larger than a chunk, goes to
// lrs_sample_rows (same inputs, same results).
constexpr int kBigShift = 15;
constexpr uint32_t kBigBuckets = 8192;
constexpr uint32_t kBigBitWords = kStageMaxTiles * (uint32_t)kTile / 32u + 8u;  // window bitmap (+ edges)
constexpr uint32_t kBigMargin = 12u;  // float steps between CUDA's expf-based p and the exact p (at most 7)

struct BigChunk {
    unsigned long long keys[kChunk];
    uint16_t perm[2 * kChunk];
};
struct BigShared {
    uint32_t end[kBigBuckets];  // counts, then bucket starts, then (after the scatter) bucket ends
    uint32_t sorted[kBigBuckets / 32];  // bucket b is sorted in the scratch
    union {
        uint32_t bits[kBigBitWords];  // steps 1-2: the window (sampler.rs:82-102)
        BigChunk ck;                  // steps 3-4
    } u;
};
constexpr size_t kBigSmem = sizeof(BigShared);

// Bucket of p (bits pb) below the largest p (bits top); kBigBuckets - 1: every smaller p.
__device__ __forceinline__ uint32_t big_bucket(uint32_t top, uint32_t pb) {
    const uint32_t diff = pb >= top ? 0u : top - pb;
    const uint32_t b = diff >> kBigShift;
    return b < kBigBuckets - 1u ? b : kBigBuckets - 1u;
}

// The scaled logit's d = fl(fl(pen(x) * inv_t) - M) of element i (sampler.rs:96-100, 115-118;
// ops.rs:409), with the window in `bits`.
__device__ __forceinline__ float big_d(float x, uint32_t i, const uint32_t* bits, bool pen, float penalty,
                                       float inv_t, float M) {
    if (pen && ((bits[i >> 5] >> (i & 31u)) & 1u)) x = penalise(x, penalty);
    return d_of(x, inv_t, M);
}

// The largest bucket end at most lim (pos + kChunk: the end of the chunk that starts at pos),
// or 0 when there is none past pos (the bucket at pos alone is longer, or pos has reached the
// last bucket).
__device__ __forceinline__ uint32_t big_chunk_end(const uint32_t* end, uint32_t pos, uint32_t nsorted,
                                                  uint32_t lim = 0xFFFFFFFFu) {
    if (pos >= nsorted) return 0u;
    if (lim == 0xFFFFFFFFu) lim = pos + (uint32_t)kChunk;
    // largest b <= kBigBuckets - 2 with end[b] <= lim (end is non-decreasing)
    int lo = -1, hi = (int)kBigBuckets - 2;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (end[mid] <= lim) lo = mid; else hi = mid - 1;
    }
    const uint32_t c1 = lo >= 0 ? end[lo] : 0u;
    return c1 > pos ? c1 : 0u;
}

// keys[0, cnt) = src[0, cnt), cnt <= kChunk: every load of the thread issued before its stores.
__device__ __forceinline__ void big_load_chunk(const unsigned long long* src, uint32_t cnt, unsigned long long* keys) {
    unsigned long long v[kVpt];
#pragma unroll
    for (int j = 0; j < kVpt; ++j) {
        const uint32_t i = threadIdx.x + (uint32_t)j * kThreads;
        v[j] = i < cnt ? __ldcg(src + i) : 0ull;
    }
#pragma unroll
    for (int j = 0; j < kVpt; ++j) {
        const uint32_t i = threadIdx.x + (uint32_t)j * kThreads;
        if (i < cnt) keys[i] = v[j];
    }
}

// First and last bucket of the chunk [pos, c1) (pos and c1 bucket boundaries, c1 > pos).
__device__ __forceinline__ void big_chunk_buckets(const uint32_t* end, uint32_t pos, uint32_t c1, uint32_t& b0,
                                                  uint32_t& b1) {
    int lo = 0, hi = (int)kBigBuckets - 2;  // smallest b with end[b] > pos
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (end[mid] > pos) hi = mid; else lo = mid + 1;
    }
    b0 = (uint32_t)lo;
    lo = (int)b0;
    hi = (int)kBigBuckets - 2;  // largest b with end[b] <= c1
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (end[mid] <= c1) lo = mid; else hi = mid - 1;
    }
    b1 = (uint32_t)lo;
}

// The chunk [pos, pos + cnt) of B, loaded in shared memory: each of its buckets sorted (a
// warp a bucket; a bucket of more than 512 keys: the whole chunk by the block), and the sorted
// chunk written back to B.
__device__ __noinline__ void big_sort_chunk(unsigned long long* B, uint32_t pos, uint32_t cnt, uint32_t b0,
                                            uint32_t b1, BigShared& bs, RowShared& sh) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long* keys = bs.u.ck.keys;
    if (tid == 0) sh.misc[3] = 0u;
    csync();
    for (uint32_t b = b0 + (uint32_t)warp; b <= b1; b += kWarps) {
        const uint32_t lo = (b == 0u ? 0u : bs.end[b - 1u]) - pos, hi = bs.end[b] - pos;
        const uint32_t c = hi - lo;
        if (c <= 1u || ((bs.sorted[b >> 5] >> (b & 31u)) & 1u)) continue;
        if (lane == 0 && c <= 512u) atomicOr(&bs.sorted[b >> 5], 1u << (b & 31u));
        if (c <= 512u)
            warp_sort_smem(keys + lo, c);
        else if (lane == 0)
            sh.misc[3] = 1u;
    }
    csync();
    if (sh.misc[3]) {
        (void)stage_sort_u64(keys, cnt, bs.u.ck.perm, bs.u.ck.perm + kChunk);
        for (uint32_t b = b0 + (uint32_t)tid; b <= b1; b += kThreads) atomicOr(&bs.sorted[b >> 5], 1u << (b & 31u));
    }
#pragma unroll
    for (int j = 0; j < kVpt; ++j) {
        const uint32_t i = (uint32_t)tid + (uint32_t)j * kThreads;
        if (i < cnt) __stcg(B + pos + i, keys[i]);
    }
    csync();
}

// A run of whole buckets of the walk, in any order (src: shared or global memory): its
// increments on the grid of s (unit 2^uu), summed over the block.  When no element is an
// ordered step (a tie or an element of half a binade on that grid) and the total keeps s inside
// its binade (and, for the top-p sum, below thr), every order of the run gives the same exact
// result: s is advanced and the run needs no order.  Same values for every thread.
template <int DIR>
__device__ __noinline__ bool big_fast_range(const unsigned long long* src, uint32_t cnt, float& s, float thr,
                                            RowShared& sh, bool apply = true) {
    const float kInf = __int_as_float(0x7F800000);
    const int uu = unit_exp(s);
    const uint32_t A = grid_count(s, uu);
    const uint32_t lower = grid_lower(uu);
    const float tq = (DIR > 0 && thr < kInf) ? ldexpf(thr, -uu) : kInf;
    uint32_t tot = 0, ev = 0;
    for (uint32_t base = 0; base < cnt; base += (uint32_t)kChunk) {
        unsigned long long k[kVpt];
#pragma unroll
        for (int j = 0; j < kVpt; ++j) {
            const uint32_t i = base + threadIdx.x + (uint32_t)j * kThreads;
            k[j] = i < cnt ? src[i] : ~0ull;  // (generic load: src may be shared or global; ~0: p = 0)
        }
#pragma unroll
        for (int j = 0; j < kVpt; ++j) {
            const Cls c = classify(~(uint32_t)(k[j] >> 32), uu);
            tot = sat_add(tot, c.inc);
            ev |= (c.tie || c.big) ? 1u : 0u;
        }
    }
    const uint32_t total = block_reduce_u32(tot, SatAdd(), sh.red);
    const uint32_t any = block_reduce_u32(ev, OrOp(), sh.red2);
    const bool fast = !any && (DIR > 0 ? (A + total <= kTwo24 - 1u && (float)(A + total) < tq) : total < A - lower);
    if (fast && apply) s = grid_value(uu, DIR > 0 ? A + total : A - total);
    return fast;
}

// The sequential run over positions [0, lim) of the bucketed keys (sampler.rs:137-145 for
// DIR > 0, sampler.rs:156-161 for DIR < 0).  A window of whole buckets (up to kBigWindow
// chunks, doubling while the windows need no order) is tried in one step straight from the
// scratch; otherwise one chunk: in one step if it needs no order, else its buckets sorted
// and the run taken one element after another.  Returns the stop position or -1 (fail: a
// bucket longer than a chunk, or the last bucket reached); s: the value after it.
constexpr uint32_t kBigWindow = 16;
template <int DIR>
__device__ __noinline__ int big_walk(unsigned long long* B, uint32_t lim, uint32_t nsorted, float& s, float thr,
                                     BigShared& bs, RowShared& sh, bool& fail, long long& c_sort) {
    const int tid = threadIdx.x;
    uint32_t win = 2;
    for (uint32_t pos = 0; pos < lim;) {
        if (DIR < 0 || pos > 0u) {  // (the top-p sum's first chunk holds its first, ordered steps)
            if (tid == 0) {
                const uint32_t far = pos + win * (uint32_t)kChunk;
                sh.misc[0] = big_chunk_end(bs.end, pos, nsorted, far < lim ? far : lim);
            }
            csync();
            const uint32_t wend = sh.misc[0];
            csync();
            if (wend > pos + (uint32_t)kChunk) {
                if (big_fast_range<DIR>(B + pos, wend - pos, s, thr, sh)) {
                    pos = wend;
                    win = win * 2u < kBigWindow ? win * 2u : kBigWindow;
                    continue;
                }
                win = 2;
            }
        }
        if (tid == 0) {
            const uint32_t c1 = big_chunk_end(bs.end, pos, nsorted);
            uint32_t b0 = 0, b1 = 0;
            if (c1) big_chunk_buckets(bs.end, pos, c1, b0, b1);
            sh.misc[0] = c1;
            sh.misc[1] = b0;
            sh.misc[2] = b1;
        }
        csync();
        const uint32_t c1 = sh.misc[0], b1 = sh.misc[2];
        uint32_t b0 = sh.misc[1];
        csync();
        if (!c1) {
            fail = true;
            return -1;
        }
        big_load_chunk(B + pos, c1 - pos, bs.u.ck.keys);
        csync();
        const uint32_t wc = (c1 < lim ? c1 : lim) - pos;
        bool sorted = false;
        if (c1 > lim) {  // (cut by lim: the first wc positions need their order)
            big_sort_chunk(B, pos, c1 - pos, b0, b1, bs, sh);
            sorted = true;
        }
        if ((DIR < 0 || pos > 0u) && big_fast_range<DIR>(bs.u.ck.keys, wc, s, thr, sh)) {
            pos = c1;
            continue;
        }
        uint32_t from = 0;  // (chunk-relative start of the part still to walk)
        if (!sorted && (DIR < 0 || pos > 0u) && b1 > b0) {
            // The first bucket holding an ordered step: the longest run of whole buckets from b0
            // that needs no order (bisection), added in one step; that bucket sorted and walked
            // one element after another; the rest of the chunk in one step if it needs no order.
            uint32_t good = b0, bad = b1 + 1u;  // [b0, good) needs no order; [b0, bad) does
            while (bad - good > 1u) {
                const uint32_t mid = (good + bad) >> 1;
                const uint32_t e = bs.end[mid - 1u] - pos;
                if (big_fast_range<DIR>(bs.u.ck.keys, e, s, thr, sh, false)) good = mid; else bad = mid;
            }
            const uint32_t e0 = good > b0 ? bs.end[good - 1u] - pos : 0u;  // (the event bucket: good)
            if (e0) (void)big_fast_range<DIR>(bs.u.ck.keys, e0, s, thr, sh);
            const uint32_t e1 = bs.end[good] - pos;
            const long long t0 = clock64();
            big_sort_chunk(B, pos, c1 - pos, good, good, bs, sh);
            c_sort += clock64() - t0;
            const uint32_t hi = e1 < wc ? e1 : wc;
            if (hi > e0) {
                const int st = big_serial<DIR>(bs.u.ck.keys + e0, hi - e0, s, thr, sh);
                if (st >= 0) return (int)(pos + e0) + st;
            }
            if (e1 >= wc) {
                pos = c1;
                continue;
            }
            if (big_fast_range<DIR>(bs.u.ck.keys + e1, wc - e1, s, thr, sh)) {
                pos = c1;
                continue;
            }
            from = e1;
            b0 = good + 1u;
        }
        if (!sorted) {
            const long long t0 = clock64();
            big_sort_chunk(B, pos, c1 - pos, b0, b1, bs, sh);
            c_sort += clock64() - t0;
        }
        const int st = big_serial<DIR>(bs.u.ck.keys + from, wc - from, s, thr, sh);
        if (st >= 0) return (int)(pos + from) + st;
        pos = c1;
    }
    return -1;
}

// One big-nucleus row by the CTA (steps 1-4 above); B: the CTA's scratch (n keys).
__device__ __noinline__ void big_row(const StageArgs& S, uint32_t r, unsigned long long* B, BigShared& bs,
                                     RowShared& sh) {
    const lrs_kernel_args_t& a = S.a;
    const int tid = threadIdx.x;
    const long long t_start = clock64();
    const RowPrep rp = S.rprep[r];
    if ((rp.flags & (kRowDone | kRowFallback)) || !(rp.flags & kRowBig)) return;  // (the sum may have left it)
    const lrs_params P = a.params[r];
    const Geo g = row_geometry(a, r);
    const uint32_t n = g.n;
    const float M = rp.M, inv_t = rp.inv_t;
    const float Ssum = __uint_as_float(rp.pad[0]);
    const float inv = __fdiv_rn(1.0f, Ssum);    // ops.rs:413
    const uint32_t top = __float_as_uint(inv);  // the largest p (e = 1)
    const ExpTable exptab{a.exp_index, a.exp_entries, a.exp_near};
    const bool pen = P.repetition_penalty != 1.0f;
    const float penalty = P.repetition_penalty;
    const uint32_t hlen = (pen && a.hist_len) ? a.hist_len[r] : 0u;
    const uint32_t* hrow = a.hist ? a.hist + (uint64_t)r * a.hist_ld : nullptr;
    const uint32_t hstart = window_start(P, hlen);
    const uint32_t words = (n + 31u) / 32u;
    if (words > kBigBitWords) {  // (prep sends no such row)
        if (tid == 0) stage_fallback(S, r);
        return;
    }
    uint32_t* bits = bs.u.bits;
    // ---- 1. the window's bits; the bucket counts ----
    for (uint32_t w = tid; w < words; w += kThreads) bits[w] = 0u;
    for (uint32_t b = tid; b < kBigBuckets; b += kThreads) bs.end[b] = 0u;
    if (tid == 0) {
        sh.misc[7] = 0u;
        sh.events = 0u;
    }
    csync();
    for (uint32_t j = hstart + tid; j < hlen; j += kThreads) {
        const uint32_t id = hrow[j];
        if (id < n) atomicOr(&bits[id >> 5], 1u << (id & 31u));
    }
    csync();
    // (kVpt elements a thread per batch, the next batch's loads issued before this one's work)
    constexpr uint32_t kBatch = (uint32_t)kVpt * kThreads;
    auto load_batch = [&](uint32_t i0, float (&x)[kVpt]) {
#pragma unroll
        for (int u = 0; u < kVpt; ++u) {
            const uint32_t i = i0 + (uint32_t)u * kThreads;
            x[u] = i < n ? __ldg(g.row + i) : 0.0f;
        }
    };
    float xa[kVpt];
    load_batch((uint32_t)tid, xa);
    for (uint32_t i0 = tid; i0 < n; i0 += kBatch) {
        float xb[kVpt];
        load_batch(i0 + kBatch, xb);
#pragma unroll
        for (int u = 0; u < kVpt; ++u) {
            const uint32_t i = i0 + (uint32_t)u * kThreads;
            if (i < n) {
                const float d = big_d(xa[u], i, bits, pen, penalty, inv_t, M);
                const uint32_t pb = __float_as_uint(__fmul_rn(expf(d), inv));
                uint32_t b = big_bucket(top, pb);
                if (big_bucket(top, pb + kBigMargin) != big_bucket(top, pb > kBigMargin ? pb - kBigMargin : 0u))
                    b = big_bucket(top, __float_as_uint(__fmul_rn(exact_expf(d, exptab), inv)));
                atomicAdd(&bs.end[b], 1u);
            }
        }
#pragma unroll
        for (int u = 0; u < kVpt; ++u) xa[u] = xb[u];
    }
    csync();
    {  // bucket starts (exclusive prefix over the buckets, a contiguous run of them a thread)
        constexpr uint32_t per = (kBigBuckets + kThreads - 1) / kThreads;
        const uint32_t b0 = (uint32_t)tid * per;
        uint32_t c = 0;
        for (uint32_t j = 0; j < per; ++j)
            if (b0 + j < kBigBuckets) c += bs.end[b0 + j];
        uint32_t total;
        uint32_t run = block_excl_scan(c, sh.red, total);
        for (uint32_t j = 0; j < per; ++j) {
            if (b0 + j < kBigBuckets) {
                const uint32_t x = bs.end[b0 + j];
                bs.end[b0 + j] = run;
                run += x;
            }
        }
    }
    csync();
    const uint32_t nsorted = bs.end[kBigBuckets - 1];  // keys scattered (the last bucket is not)
    // ---- 2. the keys, bucket by bucket (exact p: p desc, index asc) ----
    load_batch((uint32_t)tid, xa);
    for (uint32_t i0 = tid; i0 < n; i0 += kBatch) {
        float xb[kVpt];
        load_batch(i0 + kBatch, xb);
#pragma unroll
        for (int q = 0; q < kVpt; q += 4) {  // (four exps side by side)
            float d[4], ev[4];
            bool ok[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t i = i0 + (uint32_t)(q + u) * kThreads;
                d[u] = i < n ? big_d(xa[q + u], i, bits, pen, penalty, inv_t, M) : 0.0f;
                ok[u] = expf_rounded(d[u], exptab, ev[u]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t i = i0 + (uint32_t)(q + u) * kThreads;
                if (i < n) {
                    const float e = ok[u] ? ev[u] : exact_expf_table(d[u], exptab, ev[u]);
                    const uint32_t pb = __float_as_uint(__fmul_rn(e, inv));
                    const uint32_t b = big_bucket(top, pb);
                    if (b < kBigBuckets - 1u) {
                        const uint32_t slot = atomicAdd(&bs.end[b], 1u);
                        __stcg(B + slot, ((unsigned long long)(~pb) << 32) | i);
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kVpt; ++u) xa[u] = xb[u];
    }
    csync();
    const long long t_scatter = clock64();
    long long c_sort = 0;  // (diagnostics: cycles sorting chunks)
    // ---- 3. the top-p cut over the first k (sampler.rs:122-146), chunk by chunk ----
    const uint32_t kk = rp.k < n ? rp.k : n;
    float cum = 0.0f;
    int stop = -1;
    bool fail = false;
    for (uint32_t w = tid; w < kBigBuckets / 32u; w += kThreads) bs.sorted[w] = 0u;
    csync();
    stop = big_walk<+1>(B, kk, nsorted, cum, P.top_p, bs, sh, fail, c_sort);
    if (fail) {
        if (tid == 0) stage_fallback(S, r);
        return;
    }
    // the cutoff (sampler.rs:137-146); the survivor sum is the same sequence (sampler.rs:148-151)
    const uint32_t cut = stop >= 0 ? (uint32_t)stop + 1u : kk;
    // ---- 4. the draw over the sorted survivors (sampler.rs:152-162) ----
    unsigned long long st = a.state[r];
    uint32_t ps = 0;
    float r0 = 0.0f;
    if (cum > 0.0f) {
        r0 = __fmul_rn(next_f32(&st), cum);  // sampler.rs:155
        float rv = r0;
        ps = cut - 1u;
        bool dfail = false;
        const int w = big_walk<-1>(B, cut, nsorted, rv, 0.0f, bs, sh, dfail, c_sort);
        if (w >= 0) ps = (uint32_t)w;
        if (dfail && tid == 0) sh.misc[7] = 1u;  // (the top-p walk covered [0, cut): should not happen)
    }
    if (tid != 0) return;
    if (sh.misc[7]) {  // (an internal bound of the exact emulation failed: should not happen)
        stage_fallback(S, r);
        return;
    }
    const unsigned long long chosen = __ldcg(B + ps);
    lrs_row_info inf = blank_info(2u, rp.k);
    inf.token = (uint32_t)(chosen & 0xFFFFFFFFu);
    inf.prob = __uint_as_float(~(uint32_t)(chosen >> 32));
    inf.cutoff = cut;
    inf.pos = ps;
    inf.max = M;
    inf.sum_exp = Ssum;
    inf.surv_sum = cum;
    inf.r0 = r0;
    inf.n_cand = nsorted;
    inf.events = rp.pad[1];
    const long long dt = clock64() - t_start;
    inf.cycles[2] = dt > 0xFFFFFFFFll ? 0xFFFFFFFFu : (uint32_t)dt;
    inf.cycles[4] = 1u;  // (finished by the staged pipeline)
    inf.cycles[5] = rp.walks;
    auto sat = [](long long v) -> uint32_t { return v > 0xFFFFFFFFll ? 0xFFFFFFFFu : (v < 0 ? 0u : (uint32_t)v); };
    // (diagnostics: 0 and 1 the prep and sum stages; 3 the counting and scattering; 6 the two
    // walks; 7 the sorts within 6)
    inf.cycles[0] = rp.cyc_prep;
    inf.cycles[1] = rp.cyc_sum;
    inf.cycles[3] = sat(t_scatter - t_start);
    inf.cycles[6] = sat(clock64() - t_scatter);
    inf.cycles[7] = sat(c_sort);
    write_row(a, r, LRS_OK, inf.token, inf.prob, true, st, inf);
}

// Persistent: each CTA takes the next row of big_rows and samples it in its own scratch
// (the first n words of lrs_sample_rows' per-CTA scratch, which that kernel, launched after
// this one, overwrites before it reads).
__global__ void __launch_bounds__(kThreads, 2) lrs_stage_big(const StageArgs S) {
    extern __shared__ __align__(16) unsigned char big_smem[];
    BigShared& bs = *reinterpret_cast<BigShared*>(big_smem);
    __shared__ RowShared sh;
    __shared__ uint32_t claim;
    if (*(volatile const uint32_t*)S.big_count == 0u) return;
    unsigned long long* B = S.a.scratch + (uint64_t)blockIdx.x * S.a.scratch_stride;
    for (;;) {
        if (threadIdx.x == 0) {
            const uint32_t i = atomicAdd(S.big_claim, 1u);
            claim = i < *(volatile const uint32_t*)S.big_count ? S.big_rows[i] : 0xFFFFFFFFu;
        }
        csync();
        const uint32_t r = claim;
        csync();
        if (r == 0xFFFFFFFFu) return;
        big_row(S, r, B, bs, sh);
    }
}
