// oracle/sampler_ref.cpp — CPU restatement of rust-llama's token sampler.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
// baseline ("port" of the reference).  Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py load it; the product library never
// links or calls it.
//
// Reference restated (paths inside the rust-llama crate):
//   src/sampler.rs:40-48   next_u64 (xorshift64*, shifts 12/25/27, multiplier 0x2545F4914F6CDD1D)
//   src/sampler.rs:51-54   next_f32 = (next_u64() >> 40) as f32 / 2^24
//   src/sampler.rs:56-163  Sampler::sample
//   src/ops.rs:397-419     softmax_inplace
//
// Pinning.  The reference's own tests pin only the greedy repetition-penalty path
// (sampler.rs:181-206); tests/test_oracle.py replays those three tests against this
// file.  The stochastic path (softmax, top-k, top-p, draw) has no reference test and
// the Rust toolchain is absent here, so for that path parity is pinned by this
// restatement alone ("parity unpinned" by the reference's tests).
//
// Arithmetic.  Build with -O2 -fno-fast-math -ffp-contract=off: every f32 operation
// is one IEEE-754 binary32 operation in the reference's order, sums are sequential,
// exp is glibc expf (what Rust's f32::exp calls on x86_64-linux-gnu).
//
// Ordering.  Rust's `select_nth_unstable_by` (sampler.rs:129) leaves equal
// probabilities in an order that depends on std internals that are not available
// here.  This oracle orders by (probability desc, index asc), which is exactly the
// reference's order when top_k is off (stable sort of 0..n, sampler.rs:127,132), and
// flags rows whose result could depend on the unpinned order when top_k < n.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "../include/llamars_sampler.h"

namespace {

// sampler.rs:40-48
inline uint64_t next_u64(uint64_t* state) {
    uint64_t x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    return x * 0x2545F4914F6CDD1DULL;
}

// sampler.rs:51-54
inline float next_f32(uint64_t* state) {
    return (float)(next_u64(state) >> 40) / (float)(1ULL << 24);
}

// ops.rs:397-419
void softmax_inplace(float* x, size_t n, float* out_max, float* out_sum) {
    if (n == 0) return;
    float mx = x[0];
    for (size_t i = 1; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    if (sum > 0.0f) {
        float inv = 1.0f / sum;
        for (size_t i = 0; i < n; ++i) x[i] *= inv;
    }
    *out_max = mx;
    *out_sum = sum;
}

}  // namespace

// Flags set in lrs_ref_info::flags for rows whose token could depend on how Rust's
// select_nth_unstable orders equal probabilities (only possible when k < n).
#define LRS_REF_FLAG_KTIE    1u  // a tie group straddles the top-k boundary
#define LRS_REF_FLAG_DRAWTIE 2u  // the drawn position lies in a tie group of size > 1
#define LRS_REF_FLAG_CUTTIE  4u  // a tie group straddles the top-p cutoff

extern "C" {

typedef struct lrs_ref_info {
    lrs_row_info row;   // same fields as the GPU diagnostics
    uint32_t flags;     // LRS_REF_FLAG_*
    uint32_t pad;
} lrs_ref_info;

// One call of Sampler::sample (sampler.rs:56-163).  Returns the token; writes the
// status (LRS_OK or LRS_E_NAN where the reference panics) and the intermediates.
uint32_t lrs_ref_sample(const float* logits, size_t n, const lrs_params* params,
                        const uint32_t* recent, size_t recent_len, uint64_t* state,
                        lrs_ref_info* info) {
    lrs_ref_info local;
    if (!info) info = &local;
    std::memset(info, 0, sizeof(*info));
    info->row.status = LRS_OK;
    // sampler.rs:57-60
    if (n == 0) {
        info->row.token = 0;
        return 0;
    }
    const float temperature = params->temperature;
    const float penalty = params->repetition_penalty;
    // sampler.rs:62-70: greedy without penalty
    if (temperature <= 0.0f && penalty == 1.0f) {
        size_t best = 0;
        for (size_t i = 1; i < n; ++i)
            if (logits[i] > logits[best]) best = i;
        info->row.path = 0;
        info->row.token = (uint32_t)best;
        info->row.prob = 1.0f;
        return (uint32_t)best;
    }
    // sampler.rs:72
    std::vector<float> probs(logits, logits + n);
    // sampler.rs:82-102: windowed, once-per-distinct-token penalty
    if (penalty != 1.0f) {
        size_t start = 0;
        if (params->repeat_last_n != 0)
            start = recent_len > params->repeat_last_n ? recent_len - params->repeat_last_n : 0;
        std::vector<uint32_t> seen;
        seen.reserve(recent_len - start);
        for (size_t j = start; j < recent_len; ++j) {
            uint32_t t = recent[j];
            size_t i = t;
            if (i >= n || std::find(seen.begin(), seen.end(), t) != seen.end()) continue;
            seen.push_back(t);
            if (probs[i] > 0.0f)
                probs[i] /= penalty;
            else
                probs[i] *= penalty;
        }
    }
    // sampler.rs:104-113: greedy after penalty
    if (temperature <= 0.0f) {
        size_t best = 0;
        for (size_t i = 1; i < n; ++i)
            if (probs[i] > probs[best]) best = i;
        info->row.path = 1;
        info->row.token = (uint32_t)best;
        info->row.prob = 1.0f;
        return (uint32_t)best;
    }
    // sampler.rs:115-119
    const float inv_t = 1.0f / temperature;
    for (size_t i = 0; i < n; ++i) probs[i] *= inv_t;
    float mx = 0.0f, sum_exp = 0.0f;
    softmax_inplace(probs.data(), n, &mx, &sum_exp);
    info->row.max = mx;
    info->row.sum_exp = sum_exp;
    info->row.path = (n == 1) ? 3 : 2;
    // The reference panics (partial_cmp().unwrap(), sampler.rs:129/132) as soon as a
    // comparison sees a NaN; with n >= 2 every element is compared at least once.
    if (n >= 2) {
        for (size_t i = 0; i < n; ++i) {
            if (std::isnan(probs[i])) {
                info->row.status = LRS_E_NAN;
                info->row.token = LRS_TOKEN_NONE;
                return LRS_TOKEN_NONE;
            }
        }
    }
    // sampler.rs:122-132: top-k then sort by probability (descending)
    const size_t k = (params->top_k == 0 || params->top_k > n) ? n : params->top_k;
    info->row.k = (uint32_t)k;
    const float* pr = probs.data();
    auto cmp = [pr](size_t a, size_t b) {
        if (pr[a] != pr[b]) return pr[a] > pr[b];
        return a < b;
    };
    std::vector<size_t> idx(n);
    for (size_t i = 0; i < n; ++i) idx[i] = i;
    uint32_t flags = 0;
    if (k < n) {
        std::nth_element(idx.begin(), idx.begin() + (k - 1), idx.end(), cmp);
        // the best excluded element decides whether a tie straddles the boundary
        float best_excluded = -1.0f;
        for (size_t j = k; j < n; ++j) best_excluded = std::max(best_excluded, pr[idx[j]]);
        idx.resize(k);
        std::sort(idx.begin(), idx.end(), cmp);
        if (pr[idx[k - 1]] == best_excluded) flags |= LRS_REF_FLAG_KTIE;
    } else {
        std::sort(idx.begin(), idx.end(), cmp);
    }
    // sampler.rs:135-146: top-p on the sorted list (full-vocab probabilities)
    size_t cutoff = idx.size();
    if (params->top_p > 0.0f && params->top_p < 1.0f) {
        float cum = 0.0f;
        for (size_t pos = 0; pos < idx.size(); ++pos) {
            cum += pr[idx[pos]];
            if (cum >= params->top_p) {
                cutoff = pos + 1;
                break;
            }
        }
    }
    if (k < n && cutoff < idx.size() && pr[idx[cutoff - 1]] == pr[idx[cutoff]])
        flags |= LRS_REF_FLAG_CUTTIE;
    info->row.cutoff = (uint32_t)cutoff;
    // sampler.rs:148-154
    float sum = 0.0f;
    for (size_t pos = 0; pos < cutoff; ++pos) sum += pr[idx[pos]];
    info->row.surv_sum = sum;
    size_t chosen = cutoff - 1;
    if (sum <= 0.0f) {
        chosen = 0;
    } else {
        // sampler.rs:155-162
        float r = next_f32(state) * sum;
        info->row.r0 = r;
        for (size_t pos = 0; pos < cutoff; ++pos) {
            r -= pr[idx[pos]];
            if (r <= 0.0f) {
                chosen = pos;
                break;
            }
        }
    }
    if (k < n) {
        const float pc = pr[idx[chosen]];
        if ((chosen > 0 && pr[idx[chosen - 1]] == pc) || (chosen + 1 < k && pr[idx[chosen + 1]] == pc))
            flags |= LRS_REF_FLAG_DRAWTIE;
    }
    info->flags = flags;
    info->row.pos = (uint32_t)chosen;
    info->row.token = (uint32_t)idx[chosen];
    info->row.prob = pr[idx[chosen]];
    return (uint32_t)idx[chosen];
}

uint64_t lrs_ref_seed_state(uint64_t seed) { return seed | 1; }

uint64_t lrs_ref_next_u64(uint64_t* state) { return next_u64(state); }
float lrs_ref_next_f32(uint64_t* state) { return next_f32(state); }

// ops.rs:397-419 on its own (used to check the softmax sum and probability bits).
void lrs_ref_softmax(float* x, size_t n, float* out_max, float* out_sum) {
    float m = 0, s = 0;
    softmax_inplace(x, n, &m, &s);
    if (out_max) *out_max = m;
    if (out_sum) *out_sum = s;
}

// Full probability vector after penalty, temperature and softmax, for rows on the
// stochastic path (sampler.rs:72-119).  Used to check probability bits.
void lrs_ref_probs(const float* logits, size_t n, const lrs_params* params,
                   const uint32_t* recent, size_t recent_len, float* out) {
    std::memcpy(out, logits, n * sizeof(float));
    const float penalty = params->repetition_penalty;
    if (penalty != 1.0f) {
        size_t start = 0;
        if (params->repeat_last_n != 0)
            start = recent_len > params->repeat_last_n ? recent_len - params->repeat_last_n : 0;
        std::vector<uint32_t> seen;
        for (size_t j = start; j < recent_len; ++j) {
            uint32_t t = recent[j];
            if (t >= n || std::find(seen.begin(), seen.end(), t) != seen.end()) continue;
            seen.push_back(t);
            if (out[t] > 0.0f) out[t] /= penalty; else out[t] *= penalty;
        }
    }
    const float inv_t = 1.0f / params->temperature;
    for (size_t i = 0; i < n; ++i) out[i] *= inv_t;
    float m, s;
    softmax_inplace(out, n, &m, &s);
}

// Many independent samplers, one per row, rows spread over `threads` host threads
// (threads <= 1: the calling thread only, as the reference's single-threaded sampler).
// logits row r at logits + r*ld; history row r at hist + r*hist_ld, hist_len[r] ids.
void lrs_ref_sample_batch(const float* logits, uint32_t rows, uint32_t n, uint64_t ld,
                          const uint32_t* hist, uint64_t hist_ld, const uint32_t* hist_len,
                          const lrs_params* params, uint64_t* state, uint32_t* tokens,
                          lrs_ref_info* infos, int threads) {
    auto work = [&](uint32_t r0, uint32_t r1) {
        for (uint32_t r = r0; r < r1; ++r) {
            tokens[r] = lrs_ref_sample(logits + (size_t)r * ld, n, &params[r],
                                       hist ? hist + (size_t)r * hist_ld : nullptr,
                                       hist_len ? hist_len[r] : 0, &state[r],
                                       infos ? &infos[r] : nullptr);
        }
    };
    if (threads <= 1 || rows <= 1) {
        work(0, rows);
        return;
    }
    std::vector<std::thread> pool;
    uint32_t per = (rows + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        uint32_t a = t * per, b = std::min<uint32_t>(rows, a + per);
        if (a >= b) break;
        pool.emplace_back(work, a, b);
    }
    for (auto& th : pool) th.join();
}

// Sizes so the Python side can check the struct layout.
size_t lrs_ref_sizeof_info(void) { return sizeof(lrs_ref_info); }
size_t lrs_ref_sizeof_params(void) { return sizeof(lrs_params); }

}  // extern "C"
