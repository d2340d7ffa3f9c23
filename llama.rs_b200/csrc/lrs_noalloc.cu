// lrs_noalloc.cu — batched sampling without any allocation by the library.
//
// Some callers cannot let a library call cudaMalloc: a serving process that hands all of
// its GPU memory to its own pool at start-up and must not see allocations (or their
// implicit device synchronisation) in the decode loop, or a plug-in host that forbids
// device allocations after initialisation.  lrs_sample_device_noalloc serves them: it runs
// the same sampling kernel as lrs_sample_device, but the kernel's working memory (the
// per-CTA candidate scratch of the large-candidate path, the row counters, the error word
// and the libm-expf exception table) lives in file-scope __device__ arrays of fixed size,
// held on each GPU where this library's device code is loaded until the process exits.
//
// The caller owns and passes every input and output buffer (device pointers).  The first
// call on a device performs a one-time set-up on that device (looks up the arrays'
// device addresses and copies the exception table into its array); make that first call
// outside any stream capture.  All calls on a device share the arrays, so calls whose
// kernels may overlap on the GPU (different streams, different host threads) race on
// them: serialise such calls on one stream.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/llamars_sampler.h"
#include "lrs_device.cuh"
#include "lrs_kernels_decl.cuh"

namespace {

constexpr size_t kScratchBytes = (size_t)LRS_NOALLOC_SCRATCH_BYTES;
constexpr uint32_t kMaxTableEntries = 131072;  // libm exceptions (about 103,000 on glibc 2.39)
constexpr int kMaxDevices = 64;

// The kernel's working memory, one copy per device.
static __device__ __align__(256) unsigned long long g_scratch[kScratchBytes / 8];
static __device__ __align__(256) unsigned long long g_exp_index[lrs::kExpIndexWords];
static __device__ __align__(256) uint2 g_exp_entries[kMaxTableEntries + 1];
static __device__ __align__(256) uint32_t g_counter[kLrsRowCounters + 1];  // row counters, then the error word

struct DeviceSetup {
    bool done = false;     // set-up finished (successfully, or with a permanent failure)
    int status = LRS_OK;
    unsigned long long* scratch = nullptr;
    unsigned long long* index = nullptr;
    uint2* entries = nullptr;
    uint32_t* counter = nullptr;
    int ctas = 0;          // CTAs that fit on the device at once (SMs x resident CTAs per SM)
    uint32_t layout_n = 0; // vocabulary the scratch's window bitmaps are laid out for (0: none yet)
    uint32_t layout_grid = 0;  // ... and the CTAs whose bitmaps were cleared for it
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_lock;

// Host copies of the table, filled once from the file (no heap allocation).
uint2 h_entries[kMaxTableEntries];
unsigned long long h_index[lrs::kExpIndexWords];
uint32_t h_count = 0;
float h_near = 0.5f;  // lrs_exp_near of the table
bool h_loaded = false;

int load_table_once() {
    if (h_loaded) return LRS_OK;
    Dl_info info;
    char path[4096];
    const char* env = getenv("LRS_EXPF_TABLE");
    if (env && *env) {
        snprintf(path, sizeof path, "%s", env);
    } else {
        if (!dladdr((void*)&lrs_sample_device_noalloc, &info) || !info.dli_fname) return LRS_E_INVALID;
        snprintf(path, sizeof path, "%s", info.dli_fname);
        char* slash = strrchr(path, '/');
        if (slash)
            snprintf(slash + 1, sizeof path - (size_t)(slash + 1 - path), "data/expf_glibc.bin");
        else
            snprintf(path, sizeof path, "data/expf_glibc.bin");
    }
    FILE* f = fopen(path, "rb");
    if (!f) return LRS_E_INVALID;
    char magic[8];
    uint32_t hdr[3];
    const bool ok = fread(magic, 1, 8, f) == 8 && memcmp(magic, "LRSEXPF1", 8) == 0 && fread(hdr, 4, 3, f) == 3 &&
                    hdr[0] <= kMaxTableEntries && hdr[1] == lrs::kExpDomainLo && hdr[2] == lrs::kExpDomainHi &&
                    fread(h_entries, sizeof(uint2), hdr[0], f) == hdr[0];
    fclose(f);
    if (!ok) return LRS_E_INVALID;
    // the table must describe this machine's libm (spot check)
    for (uint32_t i = 0; i < hdr[0]; i += 97) {
        float x, y;
        memcpy(&x, &h_entries[i].x, 4);
        memcpy(&y, &h_entries[i].y, 4);
        if (!(expf(x) == y)) return LRS_E_INVALID;
    }
    uint32_t j = 0;
    memset(h_index, 0, sizeof h_index);
    for (uint32_t b = 0; b < lrs::kExpBlocks; ++b) {
        const uint32_t start = j;
        while (j < hdr[0] && ((h_entries[j].x - 0x80000000u) >> lrs::kExpBlockShift) == b) ++j;
        h_index[lrs::kExpBitWords + b] = ((unsigned long long)start << 32) | (unsigned long long)(j - start);
        if (j > start) h_index[b >> 6] |= 1ull << (b & 63);
    }
    if (j != hdr[0]) return LRS_E_INVALID;
    h_count = hdr[0];
    h_near = lrs_exp_near(h_entries, h_count);
    h_loaded = true;
    return LRS_OK;
}

// One-time set-up of `device` (current): device addresses of the arrays, table upload,
// occupancy.  A missing or mismatching table is permanent (latched); a failed CUDA call
// is not, so a later call retries the set-up.
int setup_device(int device) {
    DeviceSetup& s = g_setup[device];
    if (s.done) return s.status;
    int rc = load_table_once();
    if (rc != LRS_OK) {
        s.status = rc;
        s.done = true;
        return rc;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LRS_E_CUDA;
    if (prop.major < 10) {  // the kernel is built for sm_100a only
        s.status = LRS_E_INVALID;
        s.done = true;
        return s.status;
    }
    if (cudaGetSymbolAddress((void**)&s.scratch, g_scratch) != cudaSuccess) return LRS_E_CUDA;
    if (cudaGetSymbolAddress((void**)&s.index, g_exp_index) != cudaSuccess) return LRS_E_CUDA;
    if (cudaGetSymbolAddress((void**)&s.entries, g_exp_entries) != cudaSuccess) return LRS_E_CUDA;
    if (cudaGetSymbolAddress((void**)&s.counter, g_counter) != cudaSuccess) return LRS_E_CUDA;
    if (cudaMemcpy(s.index, h_index, sizeof h_index, cudaMemcpyHostToDevice) != cudaSuccess) return LRS_E_CUDA;
    if (cudaMemcpy(s.entries, h_entries, (size_t)h_count * sizeof(uint2), cudaMemcpyHostToDevice) != cudaSuccess)
        return LRS_E_CUDA;
    const size_t smem = lrs_kernel_smem_bytes();
    if (lrs_kernel_set_smem(smem) != cudaSuccess) return LRS_E_CUDA;
    int occ = 0;
    if (lrs_kernel_occupancy(&occ, smem) != cudaSuccess) return LRS_E_CUDA;
    if (occ < 1) {
        s.status = LRS_E_INVALID;
        s.done = true;
        return s.status;
    }
    s.ctas = prop.multiProcessorCount * (occ > 2 ? 2 : occ);
    s.layout_n = 0;
    s.status = LRS_OK;
    s.done = true;
    return LRS_OK;
}

}  // namespace

extern "C" int lrs_sample_device_noalloc(int device, const float* d_logits, uint32_t rows, uint32_t n, uint64_t ld,
                                         const uint32_t* d_hist, uint64_t hist_ld, const uint32_t* d_hist_len,
                                         const lrs_params* d_params, uint64_t* d_state, uint32_t* d_tokens,
                                         float* d_probs, int32_t* d_status, void* stream) {
    if (device < 0 || device >= kMaxDevices) return LRS_E_INVALID;
    if (rows == 0) return LRS_OK;
    // The per-CTA scratch (n candidate keys, the window bitmap, tile records) of at least
    // one CTA must fit in the static array.
    if (n == 0 || n > LRS_NOALLOC_MAX_VOCAB) return LRS_E_INVALID;
    if (!d_logits || !d_params || !d_state || !d_tokens) return LRS_E_INVALID;
    if (rows > 1 && ld != 0 && ld < n) return LRS_E_INVALID;
    if ((uintptr_t)d_logits % 4) return LRS_E_INVALID;
    if (d_hist_len && !d_hist) return LRS_E_INVALID;
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return LRS_E_CUDA;
    if (cur != device && cudaSetDevice(device) != cudaSuccess) return LRS_E_CUDA;
    int rc;
    {
        std::lock_guard<std::mutex> lock(g_setup_lock);
        rc = setup_device(device);
    }
    DeviceSetup& s = g_setup[device];
    if (rc == LRS_OK) {
        const size_t smem = lrs_kernel_smem_bytes();
        uint64_t per_cta = 0, bitmap_off = 0, tiles_off = 0, lanes_off = 0, lists_off = 0;  // scratch words per CTA and its layout
        lrs_kernel_scratch_layout(n, &per_cta, &bitmap_off, &tiles_off, &lanes_off, &lists_off);
        // as many CTAs as the fixed scratch holds at this n (for example 84 at n = 151,936,
        // of the 296 that the context entry point runs), at most one per row
        uint32_t grid = (uint32_t)(kScratchBytes / 8 / per_cta);
        if (grid > (uint32_t)s.ctas) grid = (uint32_t)s.ctas;
        if (grid > rows) grid = rows;
        // (a change of the grid at the same n leaves bitmaps of CTAs beyond the last
        // cleared grid untouched: clear again whenever this call reaches further)
        if (grid > s.layout_grid) s.layout_n = 0;
        lrs_kernel_args_t args;
        memset(&args, 0, sizeof args);
        args.logits = d_logits;
        args.ld = ld;
        args.n = n;
        args.rows = rows;
        args.hist = d_hist;
        args.hist_ld = hist_ld;
        args.hist_len = d_hist_len;
        args.params = d_params;
        args.state = reinterpret_cast<unsigned long long*>(d_state);
        args.tokens = d_tokens;
        args.probs = d_probs;
        args.status = d_status;
        args.info = nullptr;
        args.exp_index = s.index;
        args.exp_entries = s.entries;
        args.exp_near = h_near;
        args.scratch = s.scratch;
        args.scratch_stride = per_cta;
        args.bitmap_off = bitmap_off;
        args.tiles_off = tiles_off;
        args.lanes_off = lanes_off;
        args.lists_off = lists_off;
        args.row_counter = s.counter;
        args.err_flag = reinterpret_cast<int32_t*>(s.counter + kLrsRowCounters);
        cudaStream_t st = (cudaStream_t)stream;
        // The kernel needs every CTA's window bitmap to be zero on entry (each row clears
        // the bits it sets).  The scratch is laid out for this call's n, so a call with
        // another n than the last one finds other data (an earlier call's candidate keys)
        // where its bitmaps lie: clear them first.
        if (s.layout_n != n) {
            if (cudaMemset2DAsync(s.scratch + bitmap_off, per_cta * 8, 0, (tiles_off - bitmap_off) * 8, grid,
                                  st) != cudaSuccess)
                rc = LRS_E_CUDA;
            else {
                s.layout_n = n;
                s.layout_grid = grid;
            }
        }
        // the row counters start at zero on every call; the error word is read back (and
        // cleared) by lrs_noalloc_poll_error
        if (rc == LRS_OK && cudaMemsetAsync(s.counter, 0, kLrsRowCounters * sizeof(uint32_t), st) != cudaSuccess)
            rc = LRS_E_CUDA;
        if (rc == LRS_OK && lrs_kernel_launch(&args, grid, smem, st) != cudaSuccess) rc = LRS_E_CUDA;
    }
    if (cur != device) cudaSetDevice(cur);
    return rc;
}

extern "C" int lrs_noalloc_poll_error(int device, void* stream) {
    if (device < 0 || device >= kMaxDevices) return LRS_E_INVALID;
    DeviceSetup& s = g_setup[device];
    if (!s.done || s.status != LRS_OK) return s.done ? s.status : LRS_OK;
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return LRS_E_CUDA;
    if (cur != device && cudaSetDevice(device) != cudaSuccess) return LRS_E_CUDA;
    int32_t err = 0;
    int rc = LRS_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyAsync(&err, s.counter + kLrsRowCounters, sizeof err, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        rc = LRS_E_CUDA;
    else if (err != 0) {
        rc = err;
        if (cudaMemsetAsync(s.counter + kLrsRowCounters, 0, sizeof err, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            rc = LRS_E_CUDA;
    }
    if (cur != device) cudaSetDevice(cur);
    return rc;
}
