// lrs_api.cu — host side of the C ABI declared in include/llamars_sampler.h.
//
// A context owns, on one device: per-row parameter/state/output buffers, device
// staging for logits and history, pinned host staging for the synchronous entry
// point, the libm-expf exception table, the per-CTA scratch of the large-candidate
// path, and a stream.  Every entry point validates its arguments and returns a
// status; none aborts.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/llamars_sampler.h"
#include "lrs_device.cuh"

#include "lrs_kernels_decl.cuh"

namespace {
thread_local std::string g_create_error;
}  // namespace

// lrs_sample with pinned host rows: copies overlapped with sampling in this many pieces
// (batches of at least kPipeMinRows rows)
constexpr uint32_t kPipeChunks = 4;
constexpr uint32_t kPipeMinRows = 512;

struct lrs_ctx {
    int device = 0;
    uint32_t max_rows = 0, max_vocab = 0, max_hist = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;          // host rows: copies overlapped with sampling
    cudaEvent_t copied[kPipeChunks] = {};
    int num_sms = 0;
    int ctas_per_sm = 0;
    // device buffers
    lrs_params* d_params = nullptr;
    unsigned long long* d_state = nullptr;
    uint32_t* d_tokens = nullptr;
    float* d_probs = nullptr;
    int32_t* d_status = nullptr;
    float* d_logits = nullptr;
    uint32_t* d_hist = nullptr;
    uint32_t* d_hist_len = nullptr;
    unsigned long long* d_exp_index = nullptr;
    uint2* d_exp_entries = nullptr;
    float exp_near = 0.5f;
    unsigned long long* d_scratch = nullptr;
    uint64_t scratch_stride = 0, bitmap_off = 0, tiles_off = 0, lanes_off = 0, lists_off = 0;
    uint32_t scratch_ctas = 0;
    uint32_t* d_counter = nullptr;
    uint32_t* d_order = nullptr;  // claim order of a launch (max_rows entries)
    void* d_stage = nullptr;      // working memory of the staged pipeline
    lrs_stage_layout_t stage{};
    bool staged = true;           // the staged pipeline (false: lrs_sample_rows alone, LRS_STAGED=0)
    int32_t* d_err = nullptr;
    // the sticky error word as of the last launch: copied to pinned memory after every
    // launch (err_ev marks the copy), reported by the next call or lrs_poll_error
    int32_t* h_err = nullptr;
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;     // err_ev recorded and not yet looked at
    // pinned host staging
    float* h_logits = nullptr;
    uint32_t* h_hist = nullptr;
    uint32_t* h_hist_len = nullptr;
    uint32_t* h_tokens = nullptr;
    float* h_probs = nullptr;
    int32_t* h_status = nullptr;
    std::string err;
};

static int set_err(lrs_ctx* c, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c)
        c->err = buf;
    else
        g_create_error = buf;
    return code;
}

#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess)                                                                \
            return set_err(ctx, e_ == cudaErrorMemoryAllocation ? LRS_E_NOMEM : LRS_E_CUDA,   \
                           "%s failed: %s", #call, cudaGetErrorString(e_));                   \
    } while (0)

// ------------------------------------------------------------- expf exceptions ----
static std::string library_dir() {
    Dl_info info;
    if (dladdr((void*)&lrs_seed_state, &info) && info.dli_fname) {
        std::string p(info.dli_fname);
        size_t s = p.find_last_of('/');
        if (s != std::string::npos) return p.substr(0, s);
    }
    return ".";
}

static std::string table_path() {
    const char* env = getenv("LRS_EXPF_TABLE");
    if (env && *env) return env;
    return library_dir() + "/data/expf_glibc.bin";
}

static int load_exp_table(lrs_ctx* ctx) {
    const std::string path = table_path();
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return set_err(ctx, LRS_E_INVALID, "libm expf table %s not found (run the build)", path.c_str());
    char magic[8];
    uint32_t hdr[3];
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "LRSEXPF1", 8) != 0 || fread(hdr, 4, 3, f) != 3 ||
        hdr[1] != lrs::kExpDomainLo || hdr[2] != lrs::kExpDomainHi) {
        fclose(f);
        return set_err(ctx, LRS_E_INVALID, "libm expf table %s: bad header", path.c_str());
    }
    std::vector<uint2> ent(hdr[0]);
    if (fread(ent.data(), sizeof(uint2), ent.size(), f) != ent.size()) {
        fclose(f);
        return set_err(ctx, LRS_E_INVALID, "libm expf table %s: truncated", path.c_str());
    }
    fclose(f);
    // The table must describe this machine's libm: spot-check it (every 97th entry
    // and the domain ends).  A mismatch means the table was built against another
    // libm and the probabilities would not be the reference's.
    for (size_t i = 0; i < ent.size(); i += 97) {
        float x, y;
        memcpy(&x, &ent[i].x, 4);
        const float e = expf(x);
        memcpy(&y, &ent[i].y, 4);
        if (!(e == y)) return set_err(ctx, LRS_E_INVALID, "libm expf table %s does not match this libm", path.c_str());
        if (i && ent[i].x <= ent[i - 1].x) return set_err(ctx, LRS_E_INVALID, "libm expf table unsorted");
    }
    const uint32_t nblocks = lrs::kExpBlocks;
    std::vector<unsigned long long> index(lrs::kExpIndexWords, 0ull);
    size_t j = 0;
    for (uint32_t b = 0; b < nblocks; ++b) {
        const size_t start = j;
        while (j < ent.size() && ((ent[j].x - 0x80000000u) >> lrs::kExpBlockShift) == b) ++j;
        index[lrs::kExpBitWords + b] = ((unsigned long long)start << 32) | (unsigned long long)(j - start);
        if (j > start) index[b >> 6] |= 1ull << (b & 63);
    }
    if (j != ent.size()) return set_err(ctx, LRS_E_INVALID, "libm expf table has entries outside its domain");
    CK(cudaMalloc(&ctx->d_exp_index, index.size() * sizeof(unsigned long long)));
    CK(cudaMalloc(&ctx->d_exp_entries, ent.size() * sizeof(uint2) + sizeof(uint2)));
    CK(cudaMemcpy(ctx->d_exp_index, index.data(), index.size() * sizeof(unsigned long long),
                  cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ctx->d_exp_entries, ent.data(), ent.size() * sizeof(uint2), cudaMemcpyHostToDevice));
    ctx->exp_near = lrs_exp_near(ent.data(), ent.size());
    return LRS_OK;
}

static size_t dyn_smem_bytes(uint32_t) { return lrs_kernel_smem_bytes(); }

// Rows of vocabulary shards: out[row][g * shard_n + col] = in[g][row][col].  One thread
// per 4 floats when the widths allow 16-byte accesses, else one per float.
__global__ void lrs_assemble_kernel(const float* __restrict__ in, uint32_t shards, uint32_t rows, uint32_t shard_n,
                                    float* __restrict__ out, uint64_t ld_out, bool vec4) {
    const uint64_t per_row = (uint64_t)shards * shard_n;
    const uint64_t total = (uint64_t)rows * per_row;
    const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
    if (vec4) {
        for (uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < total; i += step * 4) {
            const uint64_t row = i / per_row, c = i % per_row;
            const uint64_t g = c / shard_n, col = c % shard_n;
            const float4 v = *reinterpret_cast<const float4*>(in + (g * rows + row) * shard_n + col);
            *reinterpret_cast<float4*>(out + row * ld_out + c) = v;
        }
    } else {
        for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
            const uint64_t row = i / per_row, c = i % per_row;
            const uint64_t g = c / shard_n, col = c % shard_n;
            out[row * ld_out + c] = in[(g * rows + row) * shard_n + col];
        }
    }
}

extern "C" {

uint64_t lrs_seed_state(uint64_t seed) { return seed | 1ull; }  // sampler.rs:33-37

int lrs_assemble_shards(const float* d_gathered, uint32_t shards, uint32_t rows, uint32_t shard_n, float* d_out,
                        uint64_t ld_out, void* stream) {
    if (!d_gathered || !d_out || shards == 0 || rows == 0 || shard_n == 0) return LRS_E_INVALID;
    if (ld_out < (uint64_t)shards * shard_n) return LRS_E_INVALID;
    const bool vec4 = shard_n % 4 == 0 && ld_out % 4 == 0 && (uintptr_t)d_gathered % 16 == 0 && (uintptr_t)d_out % 16 == 0;
    const uint64_t work = (uint64_t)rows * shards * shard_n / (vec4 ? 4 : 1);
    uint64_t blocks = (work + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    lrs_assemble_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(d_gathered, shards, rows, shard_n, d_out,
                                                                          ld_out, vec4);
    return cudaGetLastError() == cudaSuccess ? LRS_OK : LRS_E_CUDA;
}

const char* lrs_last_error(const lrs_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_create_error.c_str();
}

int lrs_destroy(lrs_ctx* ctx) {
    if (!ctx) return LRS_E_INVALID;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    void* dev[] = {ctx->d_params, ctx->d_state, ctx->d_tokens, ctx->d_probs, ctx->d_status, ctx->d_logits,
                   ctx->d_hist, ctx->d_hist_len, ctx->d_exp_index, ctx->d_exp_entries, ctx->d_scratch,
                   ctx->d_counter, ctx->d_order, ctx->d_err, ctx->d_stage};
    for (void* p : dev)
        if (p) cudaFree(p);
    void* host[] = {ctx->h_logits, ctx->h_hist, ctx->h_hist_len, ctx->h_tokens, ctx->h_probs, ctx->h_status,
                    ctx->h_err};
    for (void* p : host)
        if (p) cudaFreeHost(p);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
    for (cudaEvent_t e : ctx->copied)
        if (e) cudaEventDestroy(e);
    if (ctx->err_ev) cudaEventDestroy(ctx->err_ev);
    delete ctx;
    return LRS_OK;
}

int lrs_create(int device, uint32_t max_rows, uint32_t max_vocab, uint32_t max_hist, lrs_ctx** out) {
    if (!out) return set_err(nullptr, LRS_E_INVALID, "lrs_create: out is NULL");
    *out = nullptr;
    if (max_rows == 0 || max_vocab == 0 || max_vocab > (1u << 22))
        return set_err(nullptr, LRS_E_INVALID, "lrs_create: max_rows must be > 0 and 0 < max_vocab <= 2^22");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return set_err(nullptr, LRS_E_CUDA, "lrs_create: no CUDA device");
    if (device < 0 || device >= ndev) return set_err(nullptr, LRS_E_INVALID, "lrs_create: bad device %d", device);
    lrs_ctx* ctx = new lrs_ctx();
    ctx->device = device;
    ctx->max_rows = max_rows;
    ctx->max_vocab = max_vocab;
    ctx->max_hist = max_hist;
    auto fail = [&](int code) {
        std::string msg = ctx->err;
        lrs_destroy(ctx);
        g_create_error = msg;
        return code;
    };
#define CKF(call)                                                                          \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess) {                                                           \
            set_err(ctx, e_ == cudaErrorMemoryAllocation ? LRS_E_NOMEM : LRS_E_CUDA,       \
                    "%s failed: %s", #call, cudaGetErrorString(e_));                       \
            return fail(e_ == cudaErrorMemoryAllocation ? LRS_E_NOMEM : LRS_E_CUDA);       \
        }                                                                                  \
    } while (0)
    CKF(cudaSetDevice(device));
    cudaDeviceProp prop;
    CKF(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) {
        set_err(ctx, LRS_E_INVALID, "lrs_create: device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
        return fail(LRS_E_INVALID);
    }
    ctx->num_sms = prop.multiProcessorCount;
    CKF(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
    const size_t smem = dyn_smem_bytes(max_vocab);
    if (smem > (size_t)prop.sharedMemPerBlockOptin) {
        set_err(ctx, LRS_E_INVALID, "lrs_create: vocab %u needs %zu B of shared memory (> %zu)", max_vocab, smem,
                (size_t)prop.sharedMemPerBlockOptin);
        return fail(LRS_E_INVALID);
    }
    CKF(lrs_kernel_set_smem(smem));
    int occ = 0;
    CKF(lrs_kernel_occupancy(&occ, smem));
    if (occ < 1) {
        set_err(ctx, LRS_E_INVALID, "lrs_create: kernel does not fit on an SM");
        return fail(LRS_E_INVALID);
    }
    ctx->ctas_per_sm = occ > 2 ? 2 : occ;
    ctx->scratch_ctas = (uint32_t)(ctx->num_sms * ctx->ctas_per_sm);
    lrs_kernel_scratch_layout(max_vocab, &ctx->scratch_stride, &ctx->bitmap_off, &ctx->tiles_off, &ctx->lanes_off,
                              &ctx->lists_off);
    const size_t R = max_rows;
    CKF(cudaMalloc(&ctx->d_params, R * sizeof(lrs_params)));
    CKF(cudaMalloc(&ctx->d_state, R * sizeof(unsigned long long)));
    CKF(cudaMalloc(&ctx->d_tokens, R * sizeof(uint32_t)));
    CKF(cudaMalloc(&ctx->d_probs, R * sizeof(float)));
    CKF(cudaMalloc(&ctx->d_status, R * sizeof(int32_t)));
    CKF(cudaMalloc(&ctx->d_hist, R * (size_t)(max_hist ? max_hist : 1) * sizeof(uint32_t)));
    CKF(cudaMalloc(&ctx->d_hist_len, R * sizeof(uint32_t)));
    CKF(cudaMalloc(&ctx->d_scratch, (size_t)ctx->scratch_ctas * ctx->scratch_stride * sizeof(unsigned long long)));
    CKF(cudaMemset(ctx->d_scratch, 0, (size_t)ctx->scratch_ctas * ctx->scratch_stride * sizeof(unsigned long long)));
    CKF(cudaMalloc(&ctx->d_counter, kLrsRowCounters * sizeof(uint32_t)));
    CKF(cudaMalloc(&ctx->d_order, R * sizeof(uint32_t)));
    {
        const char* st = getenv("LRS_STAGED");
        ctx->staged = !(st && st[0] == '0');
    }
    lrs_stage_layout(max_rows, max_vocab, &ctx->stage);
    CKF(cudaMalloc(&ctx->d_stage, ctx->stage.bytes));
    CKF(cudaMalloc(&ctx->d_err, sizeof(int32_t)));
    CKF(cudaMemset(ctx->d_err, 0, sizeof(int32_t)));
    CKF(cudaMemset(ctx->d_state, 0, R * sizeof(unsigned long long)));
    CKF(cudaMemset(ctx->d_params, 0, R * sizeof(lrs_params)));
    CKF(cudaMallocHost(&ctx->h_hist, R * (size_t)(max_hist ? max_hist : 1) * sizeof(uint32_t)));
    CKF(cudaMallocHost(&ctx->h_hist_len, R * sizeof(uint32_t)));
    CKF(cudaMallocHost(&ctx->h_tokens, R * sizeof(uint32_t)));
    CKF(cudaMallocHost(&ctx->h_probs, R * sizeof(float)));
    CKF(cudaMallocHost(&ctx->h_status, R * sizeof(int32_t)));
    CKF(cudaMallocHost(&ctx->h_err, sizeof(int32_t)));
    *ctx->h_err = 0;
    CKF(cudaEventCreateWithFlags(&ctx->err_ev, cudaEventDisableTiming));
    int rc = load_exp_table(ctx);
    if (rc != LRS_OK) return fail(rc);
#undef CKF
    *out = ctx;
    return LRS_OK;
}

int lrs_set_state(lrs_ctx* ctx, const uint64_t* state, uint32_t rows) {
    if (!ctx || !state || rows > ctx->max_rows) return set_err(ctx, LRS_E_INVALID, "lrs_set_state: bad argument");
    CK(cudaSetDevice(ctx->device));
    CK(cudaMemcpyAsync(ctx->d_state, state, rows * sizeof(uint64_t), cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    return LRS_OK;
}

int lrs_get_state(lrs_ctx* ctx, uint64_t* state, uint32_t rows) {
    if (!ctx || !state || rows > ctx->max_rows) return set_err(ctx, LRS_E_INVALID, "lrs_get_state: bad argument");
    CK(cudaSetDevice(ctx->device));
    CK(cudaMemcpyAsync(state, ctx->d_state, rows * sizeof(uint64_t), cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    return LRS_OK;
}

int lrs_set_params(lrs_ctx* ctx, const lrs_params* params, uint32_t rows) {
    if (!ctx || !params || rows > ctx->max_rows) return set_err(ctx, LRS_E_INVALID, "lrs_set_params: bad argument");
    for (uint32_t r = 0; r < rows; ++r)
        if (params[r].reserved != 0) return set_err(ctx, LRS_E_INVALID, "lrs_set_params: reserved field must be 0");
    CK(cudaSetDevice(ctx->device));
    CK(cudaMemcpyAsync(ctx->d_params, params, rows * sizeof(lrs_params), cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    return LRS_OK;
}

// The sticky error word of earlier launches, if the copy made after the last launch has
// landed (wait: block until it has).  A non-zero word is returned once and cleared.
static int take_pending_error(lrs_ctx* ctx, bool wait) {
    if (!ctx->err_pending) return LRS_OK;
    if (wait) {
        CK(cudaEventSynchronize(ctx->err_ev));
    } else {
        const cudaError_t q = cudaEventQuery(ctx->err_ev);
        if (q == cudaErrorNotReady) return LRS_OK;
        if (q != cudaSuccess) return set_err(ctx, LRS_E_CUDA, "error-word copy failed: %s", cudaGetErrorString(q));
    }
    ctx->err_pending = false;
    const int32_t err = *ctx->h_err;
    if (err == 0) return LRS_OK;
    *ctx->h_err = 0;
    CK(cudaMemset(ctx->d_err, 0, sizeof(int32_t)));
    return set_err(ctx, err, "an earlier launch on this context reported error %d (%s)", err,
                   err == LRS_E_TIMEOUT ? "a bounded wait ran out" : "an internal check failed");
}

int lrs_poll_error(lrs_ctx* ctx) {
    if (!ctx) return set_err(nullptr, LRS_E_INVALID, "lrs_poll_error: ctx is NULL");
    CK(cudaSetDevice(ctx->device));
    return take_pending_error(ctx, true);
}

int lrs_sample_device(lrs_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t n, uint64_t ld,
                      const uint32_t* d_hist, uint64_t hist_ld, const uint32_t* d_hist_len,
                      const lrs_params* d_params, uint64_t* d_state, uint32_t* d_tokens, float* d_probs,
                      int32_t* d_status, lrs_row_info* d_info, void* stream) {
    if (!ctx) return set_err(nullptr, LRS_E_INVALID, "lrs_sample_device: ctx is NULL");
    if (rows == 0) return LRS_OK;
    if (rows > ctx->max_rows || n > ctx->max_vocab)
        return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: rows %u / n %u exceed the context (%u / %u)", rows, n,
                       ctx->max_rows, ctx->max_vocab);
    if (!d_logits && n > 0) return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: logits is NULL");
    if (ld < n && rows > 1 && ld != 0) return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: ld < n");
    if ((uintptr_t)d_logits % 4) return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: logits not 4-byte aligned");
    if (!d_params || !d_state || !d_tokens) return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: NULL buffer");
    if (d_hist_len && !d_hist) return set_err(ctx, LRS_E_INVALID, "lrs_sample_device: hist_len without hist");
    CK(cudaSetDevice(ctx->device));
    {
        const int perr = take_pending_error(ctx, false);
        if (perr != LRS_OK) return perr;  // (this call is not enqueued)
    }
    cudaStream_t s = (cudaStream_t)stream;
    const size_t smem = dyn_smem_bytes(n);
    lrs_kernel_args_t args;
    memset(&args, 0, sizeof(args));
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
    args.info = d_info;
    args.exp_index = ctx->d_exp_index;
    args.exp_entries = ctx->d_exp_entries;
    args.exp_near = ctx->exp_near;
    args.scratch = ctx->d_scratch;
    args.scratch_stride = ctx->scratch_stride;
    args.bitmap_off = ctx->bitmap_off;
    args.tiles_off = ctx->tiles_off;
    args.lanes_off = ctx->lanes_off;
    args.lists_off = ctx->lists_off;
    args.row_counter = ctx->d_counter;
    args.err_flag = ctx->d_err;
    uint32_t grid = ctx->scratch_ctas;
    if (grid > rows) grid = rows;
    if (ctx->staged) {
        // the staged pipeline; the rows it leaves go to lrs_sample_rows on `grid` CTAs
        CK(lrs_stage_launch(&args, ctx->d_stage, &ctx->stage, grid, smem, s));
    } else {
        // the claim order matters only when some CTA takes more than one row: smaller batches
        // skip the ordering pass (and its launch) and claim by the class sweeps
        args.order = rows > grid ? ctx->d_order : nullptr;
        CK(cudaMemsetAsync(ctx->d_counter, 0, kLrsRowCounters * sizeof(uint32_t), s));
        CK(lrs_kernel_launch(&args, grid, smem, s));
    }
    // the error word after this launch, for the next call (no host synchronisation)
    CK(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(ctx->err_ev, s));
    ctx->err_pending = true;
    return LRS_OK;
}

int lrs_test_wait_timeout(lrs_ctx* ctx, uint32_t bound_cycles, void* stream) {
    if (!ctx) return set_err(nullptr, LRS_E_INVALID, "lrs_test_wait_timeout: ctx is NULL");
    if (bound_cycles == 0) return set_err(ctx, LRS_E_INVALID, "lrs_test_wait_timeout: bound is 0");
    CK(cudaSetDevice(ctx->device));
    {
        const int perr = take_pending_error(ctx, false);
        if (perr != LRS_OK) return perr;
    }
    cudaStream_t s = (cudaStream_t)stream;
    CK(lrs_wait_probe_launch(ctx->d_err, (long long)bound_cycles, s));
    // the error word after this launch, read back as after a sampling launch
    CK(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(ctx->err_ev, s));
    ctx->err_pending = true;
    return LRS_OK;
}

int lrs_sample(lrs_ctx* ctx, const float* logits, int logits_on_device, uint32_t rows, uint32_t n, uint64_t ld,
               const uint32_t* hist, uint64_t hist_ld, const uint32_t* hist_len, uint32_t* out_tokens,
               float* out_probs) {
    if (!ctx) return set_err(nullptr, LRS_E_INVALID, "lrs_sample: ctx is NULL");
    if (rows == 0) return LRS_OK;
    if (!out_tokens || (!logits && n > 0)) return set_err(ctx, LRS_E_INVALID, "lrs_sample: NULL buffer");
    if (rows > ctx->max_rows || n > ctx->max_vocab)
        return set_err(ctx, LRS_E_INVALID, "lrs_sample: rows %u / n %u exceed the context", rows, n);
    if (ld < n && ld != 0) return set_err(ctx, LRS_E_INVALID, "lrs_sample: ld < n");
    if (hist_len && !hist) return set_err(ctx, LRS_E_INVALID, "lrs_sample: hist_len without hist");
    uint32_t hmax = 0;
    if (hist_len)
        for (uint32_t r = 0; r < rows; ++r) hmax = hist_len[r] > hmax ? hist_len[r] : hmax;
    if (hmax > ctx->max_hist) return set_err(ctx, LRS_E_INVALID, "lrs_sample: history %u > max_hist %u", hmax, ctx->max_hist);
    CK(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const float* d_logits = logits;
    uint64_t dld = ld;
    bool pipelined = false;
    if (!logits_on_device && n > 0) {
        // One H2D copy of the rows (all rows share one when ld == 0).  Caller memory
        // that is already pinned is copied from directly; pageable memory goes through
        // the context's pinned staging buffer.
        const uint32_t rcopy = (ld == 0) ? 1 : rows;
        if (!ctx->d_logits) {
            CK(cudaMalloc(&ctx->d_logits, (size_t)ctx->max_rows * ctx->max_vocab * sizeof(float)));
        }
        cudaPointerAttributes pa;
        const bool pinned = cudaPointerGetAttributes(&pa, logits) == cudaSuccess && pa.type == cudaMemoryTypeHost;
        cudaGetLastError();
        if (pinned && ld != 0 && rows >= kPipeMinRows) {
            pipelined = true;  // copied chunk by chunk below, each sampled as soon as it lands
        } else if (pinned) {
            CK(cudaMemcpy2DAsync(ctx->d_logits, (size_t)n * 4, logits, (size_t)(ld ? ld : n) * 4, (size_t)n * 4,
                                 rcopy, cudaMemcpyHostToDevice, s));
        } else {
            if (!ctx->h_logits) {
                CK(cudaMallocHost(&ctx->h_logits, (size_t)ctx->max_rows * ctx->max_vocab * sizeof(float)));
            }
            for (uint32_t r = 0; r < rcopy; ++r)
                memcpy(ctx->h_logits + (size_t)r * n, logits + (size_t)r * ld, (size_t)n * 4);
            CK(cudaMemcpyAsync(ctx->d_logits, ctx->h_logits, (size_t)rcopy * n * 4, cudaMemcpyHostToDevice, s));
        }
        d_logits = ctx->d_logits;
        dld = (ld == 0) ? 0 : n;
    }
    const uint32_t* d_hist = nullptr;
    const uint32_t* d_hlen = nullptr;
    uint64_t dhld = 0;
    if (hist_len && hmax > 0) {
        for (uint32_t r = 0; r < rows; ++r) {
            memcpy(ctx->h_hist + (size_t)r * hmax, hist + (size_t)r * hist_ld, hist_len[r] * 4);
            ctx->h_hist_len[r] = hist_len[r];
        }
        CK(cudaMemcpyAsync(ctx->d_hist, ctx->h_hist, (size_t)rows * hmax * 4, cudaMemcpyHostToDevice, s));
        CK(cudaMemcpyAsync(ctx->d_hist_len, ctx->h_hist_len, rows * 4, cudaMemcpyHostToDevice, s));
        d_hist = ctx->d_hist;
        d_hlen = ctx->d_hist_len;
        dhld = hmax;
    }
    int rc = LRS_OK;
    if (pipelined) {
        // Pinned host rows in kPipeChunks pieces: the copy of piece c + 1 (copy stream,
        // copy engine) runs while piece c is sampled (sampling stream); the launches stay
        // in order on one stream, so they never share the per-CTA scratch at once.
        if (!ctx->copy_stream) {
            CK(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
            for (cudaEvent_t& e : ctx->copied) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        }
        // the copies may not overwrite rows an earlier call is still sampling
        CK(cudaEventRecord(ctx->copied[0], s));
        CK(cudaStreamWaitEvent(ctx->copy_stream, ctx->copied[0], 0));
        const uint32_t per = (rows + kPipeChunks - 1) / kPipeChunks;
        for (uint32_t c = 0, r0 = 0; r0 < rows; ++c, r0 += per) {
            const uint32_t nr = rows - r0 < per ? rows - r0 : per;
            float* dst = ctx->d_logits + (size_t)r0 * n;
            CK(cudaMemcpy2DAsync(dst, (size_t)n * 4, logits + (size_t)r0 * ld, (size_t)ld * 4, (size_t)n * 4, nr,
                                 cudaMemcpyHostToDevice, ctx->copy_stream));
            CK(cudaEventRecord(ctx->copied[c], ctx->copy_stream));
            CK(cudaStreamWaitEvent(s, ctx->copied[c], 0));
            rc = lrs_sample_device(ctx, dst, nr, n, n, d_hist ? d_hist + (size_t)r0 * dhld : nullptr, dhld,
                                   d_hlen ? d_hlen + r0 : nullptr, ctx->d_params + r0,
                                   reinterpret_cast<uint64_t*>(ctx->d_state) + r0, ctx->d_tokens + r0,
                                   ctx->d_probs + r0, ctx->d_status + r0, nullptr, s);
            if (rc != LRS_OK) return rc;
        }
    } else {
        rc = lrs_sample_device(ctx, d_logits, rows, n, dld, d_hist, dhld, d_hlen, ctx->d_params,
                               reinterpret_cast<uint64_t*>(ctx->d_state), ctx->d_tokens, ctx->d_probs,
                               ctx->d_status, nullptr, s);
        if (rc != LRS_OK) return rc;
    }
    CK(cudaMemcpyAsync(ctx->h_tokens, ctx->d_tokens, rows * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(ctx->h_status, ctx->d_status, rows * 4, cudaMemcpyDeviceToHost, s));
    if (out_probs) CK(cudaMemcpyAsync(ctx->h_probs, ctx->d_probs, rows * 4, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    memcpy(out_tokens, ctx->h_tokens, rows * 4);
    if (out_probs) memcpy(out_probs, ctx->h_probs, rows * 4);
    {
        const int perr = take_pending_error(ctx, true);  // (the stream is idle: the copy has landed)
        if (perr != LRS_OK) return perr;
    }
    for (uint32_t r = 0; r < rows; ++r)
        if (ctx->h_status[r] != LRS_OK)
            return set_err(ctx, ctx->h_status[r], "lrs_sample: row %u status %d (NaN probabilities: the reference "
                                                  "sampler would panic)", r, ctx->h_status[r]);
    return LRS_OK;
}

// ------------------------------------------------------------ single-row drop-in ----
// One synchronous round trip a draw: the row's state, parameters and history go up in one
// copy from a pinned block (with the logits), the sampling launch reads them in place, and
// the token, status and advanced state come back in one copy of the block's head.
namespace {
constexpr size_t kOneState = 0, kOneParams = 8, kOneHistLen = 32, kOneToken = 36, kOneStatus = 40, kOneHist = 48;
static_assert(kOneParams + sizeof(lrs_params) <= kOneHistLen, "single-row block layout");
}  // namespace

struct lrs_sampler {
    uint64_t state;
    int device;
    lrs_ctx* ctx;
    unsigned char* h_blk;  // pinned: the block's host copy
    unsigned char* d_blk;  // the block on the device
    size_t blk_cap;        // bytes of both
};

lrs_sampler* lrs_sampler_new(uint64_t seed, int device) {
    lrs_sampler* s = new lrs_sampler();
    s->state = seed | 1ull;  // Sampler::new (sampler.rs:33-37)
    s->device = device;
    s->ctx = nullptr;
    s->h_blk = nullptr;
    s->d_blk = nullptr;
    s->blk_cap = 0;
    return s;
}

void lrs_sampler_free(lrs_sampler* s) {
    if (!s) return;
    if (s->ctx) {
        cudaSetDevice(s->ctx->device);
        if (s->d_blk) cudaFree(s->d_blk);
        if (s->h_blk) cudaFreeHost(s->h_blk);
        lrs_destroy(s->ctx);
    }
    delete s;
}

uint64_t lrs_sampler_state(const lrs_sampler* s) { return s ? s->state : 0; }

uint32_t lrs_sampler_sample(lrs_sampler* s, const float* logits, size_t n, const lrs_params* params,
                            const uint32_t* recent, size_t recent_len, int* status) {
    int dummy;
    if (!status) status = &dummy;
    *status = LRS_OK;
    if (!s || !params || (!logits && n) || (!recent && recent_len) || n > (1u << 22) || recent_len > 0xFFFFFFFFu ||
        params->reserved != 0) {
        *status = LRS_E_INVALID;
        return LRS_TOKEN_NONE;
    }
    if (n == 0) return 0;  // sampler.rs:57-60
    if (!s->ctx || s->ctx->max_vocab < n || s->ctx->max_hist < recent_len) {
        if (s->ctx) {
            cudaSetDevice(s->ctx->device);
            if (s->d_blk) cudaFree(s->d_blk);
            if (s->h_blk) cudaFreeHost(s->h_blk);
            s->d_blk = nullptr;
            s->h_blk = nullptr;
            s->blk_cap = 0;
            lrs_destroy(s->ctx);
        }
        s->ctx = nullptr;
        uint32_t hcap = 64;
        while (hcap < recent_len) hcap *= 2;
        int rc = lrs_create(s->device, 1, (uint32_t)n, hcap, &s->ctx);
        if (rc != LRS_OK) {
            *status = rc;
            return LRS_TOKEN_NONE;
        }
    }
    lrs_ctx* ctx = s->ctx;
    const size_t need = kOneHist + (size_t)ctx->max_hist * sizeof(uint32_t);
    auto fail = [&](int rc) -> uint32_t {
        *status = rc;
        return LRS_TOKEN_NONE;
    };
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(set_err(ctx, LRS_E_CUDA, "cudaSetDevice failed"));
    if (s->blk_cap < need) {
        if (s->d_blk) cudaFree(s->d_blk);
        if (s->h_blk) cudaFreeHost(s->h_blk);
        s->d_blk = nullptr;
        s->h_blk = nullptr;
        s->blk_cap = 0;
        if (cudaMalloc(&s->d_blk, need) != cudaSuccess || cudaMallocHost(&s->h_blk, need) != cudaSuccess)
            return fail(set_err(ctx, LRS_E_NOMEM, "lrs_sampler_sample: staging allocation failed"));
        s->blk_cap = need;
    }
    const uint32_t hl = (uint32_t)recent_len;
    memcpy(s->h_blk + kOneState, &s->state, sizeof(uint64_t));
    memcpy(s->h_blk + kOneParams, params, sizeof(lrs_params));
    memcpy(s->h_blk + kOneHistLen, &hl, sizeof(uint32_t));
    if (hl) memcpy(s->h_blk + kOneHist, recent, (size_t)hl * sizeof(uint32_t));
    cudaStream_t st = ctx->stream;
    // the logits: from caller memory that is pinned, else through the context's pinned staging
    cudaPointerAttributes pa;
    const bool pinned = cudaPointerGetAttributes(&pa, logits) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();
    if (!ctx->d_logits && cudaMalloc(&ctx->d_logits, (size_t)ctx->max_rows * ctx->max_vocab * sizeof(float)) != cudaSuccess)
        return fail(set_err(ctx, LRS_E_NOMEM, "lrs_sampler_sample: logits allocation failed"));
    const float* src = logits;
    if (!pinned) {
        if (!ctx->h_logits &&
            cudaMallocHost(&ctx->h_logits, (size_t)ctx->max_rows * ctx->max_vocab * sizeof(float)) != cudaSuccess)
            return fail(set_err(ctx, LRS_E_NOMEM, "lrs_sampler_sample: staging allocation failed"));
        memcpy(ctx->h_logits, logits, n * sizeof(float));
        src = ctx->h_logits;
    }
    if (cudaMemcpyAsync(ctx->d_logits, src, n * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(s->d_blk, s->h_blk, kOneHist + (size_t)hl * sizeof(uint32_t), cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
        return fail(set_err(ctx, LRS_E_CUDA, "lrs_sampler_sample: copy failed"));
    int rc = lrs_sample_device(ctx, ctx->d_logits, 1, (uint32_t)n, n,
                               hl ? reinterpret_cast<const uint32_t*>(s->d_blk + kOneHist) : nullptr, hl,
                               hl ? reinterpret_cast<const uint32_t*>(s->d_blk + kOneHistLen) : nullptr,
                               reinterpret_cast<const lrs_params*>(s->d_blk + kOneParams),
                               reinterpret_cast<uint64_t*>(s->d_blk + kOneState),
                               reinterpret_cast<uint32_t*>(s->d_blk + kOneToken), nullptr,
                               reinterpret_cast<int32_t*>(s->d_blk + kOneStatus), nullptr, st);
    if (rc != LRS_OK) return fail(rc);
    if (cudaMemcpyAsync(s->h_blk, s->d_blk, kOneHist, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(set_err(ctx, LRS_E_CUDA, "lrs_sampler_sample: copy back failed"));
    rc = take_pending_error(ctx, true);  // (the launch's error word has landed with the stream)
    if (rc != LRS_OK) return fail(rc);
    int32_t row_status;
    uint32_t tok;
    memcpy(&row_status, s->h_blk + kOneStatus, sizeof(int32_t));
    memcpy(&tok, s->h_blk + kOneToken, sizeof(uint32_t));
    if (row_status != LRS_OK)
        return fail(set_err(ctx, row_status, "lrs_sampler_sample: status %d (NaN probabilities: the reference "
                                             "sampler would panic)", row_status));
    memcpy(&s->state, s->h_blk + kOneState, sizeof(uint64_t));
    return tok;
}

}  // extern "C"
