/* rust_abi.c — the ABI that the Rust crate (rust/src/ffi.rs) declares, checked against the
 * C header and the built library.  No GPU needed.
 *
 * Every `extern "C"` function of rust/src/ffi.rs appears below as a function-pointer type
 * written from the Rust signature (c_int -> int, u32 -> uint32_t, u64 -> uint64_t, usize ->
 * size_t, f32 -> float, *const T -> const T *, *mut T -> T *, *mut c_void -> void *).
 *   compile time: each type is initialised from the header's prototype, so a signature the
 *                 Rust side gets wrong is an incompatible-pointer error (-Werror);
 *                 the #[repr(C)] struct layouts of ffi.rs are asserted field by field;
 *   run time:     the library is opened and every symbol is looked up; the calls that need
 *                 no GPU are made.
 * tests/test_rust_binding.py checks that this list and ffi.rs name the same functions.   */
#include <dlfcn.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/llamars_sampler.h"

/* ---- #[repr(C)] layouts of ffi.rs ---- */
_Static_assert(sizeof(lrs_params) == 24, "lrs_params size");
_Static_assert(offsetof(lrs_params, temperature) == 0, "temperature");
_Static_assert(offsetof(lrs_params, top_k) == 4, "top_k");
_Static_assert(offsetof(lrs_params, top_p) == 8, "top_p");
_Static_assert(offsetof(lrs_params, repetition_penalty) == 12, "repetition_penalty");
_Static_assert(offsetof(lrs_params, repeat_last_n) == 16, "repeat_last_n");
_Static_assert(offsetof(lrs_params, reserved) == 20, "reserved");
_Static_assert(sizeof(lrs_row_info) == 88, "lrs_row_info size");
_Static_assert(offsetof(lrs_row_info, status) == 0, "status");
_Static_assert(offsetof(lrs_row_info, token) == 4, "token");
_Static_assert(offsetof(lrs_row_info, path) == 8, "path");
_Static_assert(offsetof(lrs_row_info, k) == 12, "k");
_Static_assert(offsetof(lrs_row_info, cutoff) == 16, "cutoff");
_Static_assert(offsetof(lrs_row_info, pos) == 20, "pos");
_Static_assert(offsetof(lrs_row_info, max) == 24, "max");
_Static_assert(offsetof(lrs_row_info, sum_exp) == 28, "sum_exp");
_Static_assert(offsetof(lrs_row_info, surv_sum) == 32, "surv_sum");
_Static_assert(offsetof(lrs_row_info, r0) == 36, "r0");
_Static_assert(offsetof(lrs_row_info, prob) == 40, "prob");
_Static_assert(offsetof(lrs_row_info, n_cand) == 44, "n_cand");
_Static_assert(offsetof(lrs_row_info, events) == 48, "events");
_Static_assert(offsetof(lrs_row_info, cycles) == 52, "cycles");
_Static_assert(offsetof(lrs_row_info, reserved) == 84, "reserved");
_Static_assert(LRS_OK == 0 && LRS_E_INVALID == -1 && LRS_E_NAN == -2 && LRS_E_CUDA == -3 && LRS_E_NOMEM == -4 &&
               LRS_E_TIMEOUT == -5 && LRS_E_NCCL == -6 && LRS_E_INTERNAL == -7, "status codes");
_Static_assert(LRS_TOKEN_NONE == 0xFFFFFFFFu, "token none");

/* ---- the extern "C" block of ffi.rs ---- */
typedef int (*rs_lrs_create)(int, uint32_t, uint32_t, uint32_t, lrs_ctx **);
typedef int (*rs_lrs_destroy)(lrs_ctx *);
typedef const char *(*rs_lrs_last_error)(const lrs_ctx *);
typedef uint64_t (*rs_lrs_seed_state)(uint64_t);
typedef int (*rs_lrs_set_state)(lrs_ctx *, const uint64_t *, uint32_t);
typedef int (*rs_lrs_get_state)(lrs_ctx *, uint64_t *, uint32_t);
typedef int (*rs_lrs_set_params)(lrs_ctx *, const lrs_params *, uint32_t);
typedef int (*rs_lrs_sample)(lrs_ctx *, const float *, int, uint32_t, uint32_t, uint64_t, const uint32_t *, uint64_t,
                             const uint32_t *, uint32_t *, float *);
typedef int (*rs_lrs_sample_device)(lrs_ctx *, const float *, uint32_t, uint32_t, uint64_t, const uint32_t *, uint64_t,
                                    const uint32_t *, const lrs_params *, uint64_t *, uint32_t *, float *, int32_t *,
                                    lrs_row_info *, void *);
typedef int (*rs_lrs_poll_error)(lrs_ctx *);
typedef int (*rs_lrs_sample_device_noalloc)(int, const float *, uint32_t, uint32_t, uint64_t, const uint32_t *,
                                            uint64_t, const uint32_t *, const lrs_params *, uint64_t *, uint32_t *,
                                            float *, int32_t *, void *);
typedef int (*rs_lrs_noalloc_poll_error)(int, void *);
typedef int (*rs_lrs_history_append)(const uint32_t *, const int32_t *, uint32_t, uint32_t, uint32_t *, uint64_t,
                                     uint32_t *, uint32_t, void *);
typedef int (*rs_lrs_remap_tokens)(const uint32_t *, const int32_t *, uint32_t, const uint32_t *, uint32_t, uint32_t *,
                                   void *);
typedef lrs_sampler *(*rs_lrs_sampler_new)(uint64_t, int);
typedef void (*rs_lrs_sampler_free)(lrs_sampler *);
typedef uint64_t (*rs_lrs_sampler_state)(const lrs_sampler *);
typedef uint32_t (*rs_lrs_sampler_sample)(lrs_sampler *, const float *, size_t, const lrs_params *, const uint32_t *,
                                          size_t, int *);

/* compile-time: the header's prototypes must have exactly these types */
#define SAME(f) _Static_assert(__builtin_types_compatible_p(__typeof__(&f), rs_##f), #f " differs from ffi.rs")
SAME(lrs_create);
SAME(lrs_destroy);
SAME(lrs_last_error);
SAME(lrs_seed_state);
SAME(lrs_set_state);
SAME(lrs_get_state);
SAME(lrs_set_params);
SAME(lrs_sample);
SAME(lrs_sample_device);
SAME(lrs_poll_error);
SAME(lrs_sample_device_noalloc);
SAME(lrs_noalloc_poll_error);
SAME(lrs_history_append);
SAME(lrs_remap_tokens);
SAME(lrs_sampler_new);
SAME(lrs_sampler_free);
SAME(lrs_sampler_state);
SAME(lrs_sampler_sample);

static const char *const kSymbols[] = {
    "lrs_create", "lrs_destroy", "lrs_last_error", "lrs_seed_state", "lrs_set_state", "lrs_get_state",
    "lrs_set_params", "lrs_sample", "lrs_sample_device", "lrs_poll_error", "lrs_sample_device_noalloc",
    "lrs_noalloc_poll_error", "lrs_history_append", "lrs_remap_tokens", "lrs_sampler_new", "lrs_sampler_free",
    "lrs_sampler_state", "lrs_sampler_sample",
};

int main(int argc, char **argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s <libllamars_sampler.so>\n", argv[0]);
        return 2;
    }
    void *h = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        fprintf(stderr, "dlopen: %s\n", dlerror());
        return 1;
    }
    int missing = 0;
    for (size_t i = 0; i < sizeof kSymbols / sizeof kSymbols[0]; ++i)
        if (!dlsym(h, kSymbols[i])) {
            fprintf(stderr, "missing symbol %s\n", kSymbols[i]);
            ++missing;
        }
    if (missing) return 1;
    /* calls that need no GPU, through the types the Rust side assumes */
    const rs_lrs_seed_state seed = (rs_lrs_seed_state)dlsym(h, "lrs_seed_state");
    if (seed(42) != 43 || seed(0) != 1) return 1;
    const rs_lrs_poll_error poll = (rs_lrs_poll_error)dlsym(h, "lrs_poll_error");
    if (poll(NULL) != LRS_E_INVALID) return 1;
    const rs_lrs_sampler_sample samp = (rs_lrs_sampler_sample)dlsym(h, "lrs_sampler_sample");
    int status = 0;
    if (samp(NULL, NULL, 0, NULL, NULL, 0, &status) != LRS_TOKEN_NONE || status != LRS_E_INVALID) return 1;
    /* argument checks that reject before any device work */
    const rs_lrs_history_append app = (rs_lrs_history_append)dlsym(h, "lrs_history_append");
    if (app(NULL, NULL, 0, 0, NULL, 0, NULL, 0, NULL) != LRS_OK) return 1;            /* no rows: nothing to do */
    if (app(NULL, NULL, 4, 0, NULL, 64, NULL, 32, NULL) != LRS_E_INVALID) return 1;    /* null buffers */
    const rs_lrs_remap_tokens rmp = (rs_lrs_remap_tokens)dlsym(h, "lrs_remap_tokens");
    if (rmp(NULL, NULL, 4, NULL, 0, NULL, NULL) != LRS_E_INVALID) return 1;
    printf("rust ABI ok: %zu symbols\n", sizeof kSymbols / sizeof kSymbols[0]);
    dlclose(h);
    return 0;
}
