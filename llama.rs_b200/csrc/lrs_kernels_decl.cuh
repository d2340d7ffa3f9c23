// lrs_kernels_decl.cuh — interface between the C-ABI host code (lrs_api.cu) and the
// sampling kernel (lrs_kernels.cu).
#pragma once
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/llamars_sampler.h"

constexpr int kLrsRowCounters = 8;  // row claim classes of the sampling kernel

struct lrs_kernel_args_t {
    const float* logits;      // row r at logits + r * ld
    uint64_t ld;
    uint32_t n;               // vocabulary entries per row
    uint32_t rows;
    const uint32_t* hist;     // row r's history at hist + r * hist_ld, hist_len[r] ids
    uint64_t hist_ld;
    const uint32_t* hist_len;
    const lrs_params* params;
    unsigned long long* state;
    uint32_t* tokens;
    float* probs;             // nullable
    int32_t* status;          // nullable
    lrs_row_info* info;       // nullable
    const unsigned long long* exp_index;  // libm expf exception table (see lrs_device.cuh)
    const uint2* exp_entries;
    float exp_near;           // every table entry lies within this many float ulps of a rounding midpoint
    unsigned long long* scratch;          // per CTA: scratch_stride 8-byte words
    uint64_t scratch_stride;              // laid out by lrs_kernel_scratch_layout
    uint64_t bitmap_off;                  // window bitmap (zero between rows)
    uint64_t tiles_off;                   // tile records of rows longer than the shared table
    uint64_t lanes_off;                   // per-tile lane sums
    uint64_t lists_off;                   // candidate lists of sparse tiles
    uint32_t* row_counter;    // kLrsRowCounters row counters (one per claim class), zeroed before each launch
    uint32_t* order;          // nullable: rows in claim order, written by the launch's ordering pass
                              // (rows entries; then row_counter[0] alone indexes it)
    const uint32_t* claim_count;  // nullable: `order` is given (no ordering pass) and holds this many rows
    int32_t* err_flag;        // sticky error word
};

// Working memory of the staged pipeline (lrs_stage_launch) for up to `rows` rows of up to
// `vocab` entries: byte offsets into one device buffer of `bytes` bytes (256-byte aligned).
struct lrs_stage_layout_t {
    uint32_t rows, nt;        // rows and tile slots per row
    uint64_t tstat, lmax, tprep, tres, rprep, lists, list_n, fb_rows, fb_count, live_count, big_rows, big_count,
        big_claim, bytes;
};
void lrs_stage_layout(uint32_t rows, uint32_t vocab, lrs_stage_layout_t* L);
// The staged pipeline on args->rows rows, then lrs_sample_rows on the rows it leaves
// (fallback_grid CTAs with `smem` bytes; args->row_counter is zeroed here).  Top-p rows whose
// nucleus is larger than a list are sampled by lrs_stage_big on fallback_grid CTAs, each in
// the first n words of its lrs_sample_rows scratch (args->scratch, at most fallback_grid
// CTAs' worth).
cudaError_t lrs_stage_launch(const lrs_kernel_args_t* args, void* mem, const lrs_stage_layout_t* L,
                             uint32_t fallback_grid, size_t smem, cudaStream_t s);

// Largest distance (in float ulps, plus a margin for the difference between two
// double-precision exps) of a libm-expf table entry from the rounding midpoint next to
// its exact value: an input farther than this from every midpoint has no entry, so
// libm's value there is the correctly rounded one.  Computed by the loaders from the
// entries with this machine's double exp.
inline float lrs_exp_near(const uint2* ent, size_t n) {
    double m = 0x1p-16;  // (the generator's near-midpoint entries lie within 2^-16)
    for (size_t i = 0; i < n; ++i) {
        float x;
        memcpy(&x, &ent[i].x, 4);
        const double d = exp((double)x);
        const float c = (float)d;
        if (!(c >= 0x1p-126f)) continue;  // (subnormal results always take the table)
        float nb = d >= (double)c ? nextafterf(c, INFINITY) : nextafterf(c, 0.0f);
        const double u = fabs((double)nb - (double)c);
        const double dist = 0.5 - fabs(d - (double)c) / u;
        if (dist > m) m = dist;
    }
    return (float)(m + 0x1p-20);
}

size_t lrs_kernel_smem_bytes();   // dynamic shared memory of a CTA (independent of n)
int lrs_kernel_block_threads();
// Per-CTA scratch for rows of up to n entries: stride and the offsets of the window
// bitmap, the tile records, the lane sums and the candidate lists (8-byte words).  The bitmap words must be
// zero before the first launch; every row clears the bits it sets.
void lrs_kernel_scratch_layout(uint32_t n, uint64_t* stride, uint64_t* bitmap_off, uint64_t* tiles_off,
                               uint64_t* lanes_off, uint64_t* lists_off);
cudaError_t lrs_kernel_set_smem(size_t bytes);
cudaError_t lrs_kernel_occupancy(int* ctas_per_sm, size_t smem);
cudaError_t lrs_kernel_launch(const lrs_kernel_args_t* args, uint32_t grid, size_t smem, cudaStream_t s);
// Test of the bounded wait (lrs_test_wait_timeout): a wait of `bound` cycles on a barrier
// nothing completes, which sets *err to LRS_E_TIMEOUT.
cudaError_t lrs_wait_probe_launch(int32_t* err, long long bound, cudaStream_t s);
