// lrs_kernels_decl.cuh — interface between the C-ABI host code (lrs_api.cu) and the
// sampling kernel (lrs_kernels.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/llamars_sampler.h"

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
    unsigned long long* scratch;          // per CTA: scratch_stride entries
    uint64_t scratch_stride;
    uint32_t* row_counter;    // zeroed before each launch
    int32_t* err_flag;        // sticky error word
    uint32_t bitmap_words;    // ceil(n / 32)
};

size_t lrs_kernel_ring_bytes();
size_t lrs_kernel_area_bytes();
cudaError_t lrs_kernel_set_smem(size_t bytes);
cudaError_t lrs_kernel_occupancy(int* ctas_per_sm, size_t smem);
cudaError_t lrs_kernel_launch(const lrs_kernel_args_t* args, uint32_t grid, size_t smem, cudaStream_t s);
