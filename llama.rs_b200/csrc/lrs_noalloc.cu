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
    bool done = false;
    int status = LRS_OK;
    unsigned long long* scratch = nullptr;
    unsigned long long* index = nullptr;
    uint2* entries = nullptr;
    uint32_t* counter = nullptr;
    int ctas = 0;  // CTAs that fit on the device at the largest shared-memory size
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

// One-time set-up of `device` (current): device addresses of the arrays, table upload.
int setup_device(int device) {
    DeviceSetup& s = g_setup[device];
    if (s.done) return s.status;
    s.done = true;
    s.status = LRS_E_CUDA;
    int rc = load_table_once();
    if (rc != LRS_OK) {
        s.status = rc;
        return rc;
    }
    if (cudaGetSymbolAddress((void**)&s.scratch, g_scratch) != cudaSuccess) return s.status;
    if (cudaGetSymbolAddress((void**)&s.index, g_exp_index) != cudaSuccess) return s.status;
    if (cudaGetSymbolAddress((void**)&s.entries, g_exp_entries) != cudaSuccess) return s.status;
    if (cudaGetSymbolAddress((void**)&s.counter, g_counter) != cudaSuccess) return s.status;
    if (cudaMemcpy(s.index, h_index, sizeof h_index, cudaMemcpyHostToDevice) != cudaSuccess) return s.status;
    if (cudaMemcpy(s.entries, h_entries, (size_t)h_count * sizeof(uint2), cudaMemcpyHostToDevice) != cudaSuccess)
        return s.status;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return s.status;
    s.ctas = prop.multiProcessorCount * 2;
    s.status = LRS_OK;
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
    const DeviceSetup& s = g_setup[device];
    if (rc == LRS_OK) {
        const size_t smem = lrs_kernel_smem_bytes();
        uint64_t per_cta = 0, bitmap_off = 0, tiles_off = 0, lanes_off = 0, lists_off = 0;  // scratch words per CTA and its layout
        lrs_kernel_scratch_layout(n, &per_cta, &bitmap_off, &tiles_off, &lanes_off, &lists_off);
        uint32_t grid = (uint32_t)(kScratchBytes / 8 / per_cta);
        if (grid > (uint32_t)s.ctas) grid = (uint32_t)s.ctas;
        if (grid > rows) grid = rows;
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
        // the row counters and the error word must start at zero on every call
        if (cudaMemsetAsync(s.counter, 0, (kLrsRowCounters + 1) * sizeof(uint32_t), st) != cudaSuccess)
            rc = LRS_E_CUDA;
        else if (lrs_kernel_launch(&args, grid, smem, st) != cudaSuccess)
            rc = LRS_E_CUDA;
    }
    if (cur != device) cudaSetDevice(cur);
    return rc;
}
