// lrs_generate.cu — state of a batched generation loop kept on the device (sm_100a).
//
// rust-llama's generation loops keep, per sequence, a `recent` Vec of ids that the sampler's
// repetition penalty reads (model.rs:756-770, server.rs:180-190: prompt ids, then every
// sampled id pushed after its draw) and, with a pruned vocabulary, sample in the pruned id
// space (prune.rs:187-195 renumbers the kept ids in order).  Here both live on the device next
// to the batched sampler, so a step of a batched loop uploads nothing:
//   lrs_history_append  recent.push(next) for every row of the batch, in place
//   lrs_remap_tokens    pruned ids back to the full vocabulary through a device table
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/llamars_sampler.h"

namespace {

// One warp per row.  A row whose history is full keeps its last `keep` ids (moved to the
// front: keep <= hist_ld / 2, so source and destination do not overlap), then takes the token.
__global__ void history_append_kernel(const uint32_t* __restrict__ tokens, const int32_t* __restrict__ status,
                                      uint32_t rows, uint32_t eos, uint32_t* __restrict__ hist, uint64_t hist_ld,
                                      uint32_t* __restrict__ hist_len, uint32_t keep) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const uint32_t tok = tokens[r];
    // (a row that failed, or drew the end of its sequence, is not extended: the reference's
    // loops stop before the push, model.rs:761-763, server.rs:184-186)
    if ((status && status[r] != LRS_OK) || tok == eos || tok == LRS_TOKEN_NONE) return;
    uint32_t* h = hist + (uint64_t)r * hist_ld;
    uint64_t len = hist_len[r];
    if (len > hist_ld) len = hist_ld;
    if (len == hist_ld) {
        const uint64_t from = hist_ld - keep;
        for (uint64_t i = lane; i < keep; i += 32u) h[i] = h[from + i];
        __syncwarp();
        len = keep;
    }
    if (lane == 0) {
        h[len] = tok;
        hist_len[r] = (uint32_t)(len + 1u);
    }
}

__global__ void remap_kernel(const uint32_t* __restrict__ tokens, const int32_t* __restrict__ status, uint32_t rows,
                             const uint32_t* __restrict__ map, uint32_t map_n, uint32_t* __restrict__ out) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint32_t tok = tokens[r];
    const bool ok = (!status || status[r] == LRS_OK) && tok < map_n;
    out[r] = ok ? map[tok] : tok;
}

}  // namespace

extern "C" int lrs_history_append(const uint32_t* d_tokens, const int32_t* d_status, uint32_t rows, uint32_t eos,
                                  uint32_t* d_hist, uint64_t hist_ld, uint32_t* d_hist_len, uint32_t keep,
                                  void* stream) {
    if (rows == 0) return LRS_OK;
    if (!d_tokens || !d_hist || !d_hist_len || hist_ld < 2 || keep == 0 || keep > hist_ld / 2) return LRS_E_INVALID;
    const uint32_t threads = 256, rows_per_block = threads / 32u;
    history_append_kernel<<<(rows + rows_per_block - 1) / rows_per_block, threads, 0, (cudaStream_t)stream>>>(
        d_tokens, d_status, rows, eos, d_hist, hist_ld, d_hist_len, keep);
    return cudaGetLastError() == cudaSuccess ? LRS_OK : LRS_E_CUDA;
}

extern "C" int lrs_remap_tokens(const uint32_t* d_tokens, const int32_t* d_status, uint32_t rows,
                                const uint32_t* d_map, uint32_t map_n, uint32_t* d_out, void* stream) {
    if (rows == 0) return LRS_OK;
    if (!d_tokens || !d_map || !d_out || map_n == 0) return LRS_E_INVALID;
    remap_kernel<<<(rows + 255u) / 256u, 256, 0, (cudaStream_t)stream>>>(d_tokens, d_status, rows, d_map, map_n, d_out);
    return cudaGetLastError() == cudaSuccess ? LRS_OK : LRS_E_CUDA;
}
