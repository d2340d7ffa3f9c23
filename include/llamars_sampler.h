/*
 * llamars_sampler.h — C ABI of the B200 batched token sampler.
 *
 * Drop-in replacement for rust-llama's token sampler:
 *   src/sampler.rs:3-13    pub struct SamplingParams { temperature, top_k, top_p,
 *                                                      repetition_penalty, repeat_last_n, seed }
 *   src/sampler.rs:28-37   pub struct Sampler { state }, Sampler::new(seed) -> state = seed | 1
 *   src/sampler.rs:56-163  Sampler::sample(&mut self, logits: &[f32], params, recent: &[u32]) -> u32
 *   src/ops.rs:397-419     ops::softmax_inplace (called by sample, fused into the kernels here)
 *
 * Results are those of sampler.rs on the same inputs: the same token, the same
 * probability bits and the same PRNG state after the call (the sequential f32
 * accumulations and libm expf of the reference are reproduced exactly on the GPU).
 *
 * Error behaviour.  Sampler::sample is infallible except that a NaN probability makes
 * the `partial_cmp().unwrap()` at sampler.rs:129/132 panic, which aborts the process
 * (Cargo.toml:25 sets panic = "abort").  Here such a row gets status LRS_E_NAN, its
 * token is LRS_TOKEN_NONE and its PRNG state is left unchanged; the call returns
 * LRS_E_NAN after finishing every other row.  No entry point aborts the process.
 *
 * Threading.  A context is bound to one CUDA device and is not reentrant: drive it
 * from one host thread (or serialise calls).  Several contexts (one per GPU) may be
 * driven from several threads at once.
 */
#ifndef LLAMARS_SAMPLER_H
#define LLAMARS_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define LRS_OK            0
#define LRS_E_INVALID    -1  /* bad argument (null pointer, size out of range, ...) */
#define LRS_E_NAN        -2  /* a row's probabilities contain NaN: the reference would panic */
#define LRS_E_CUDA       -3  /* a CUDA runtime call failed; see lrs_last_error */
#define LRS_E_NOMEM      -4  /* device or pinned-host allocation failed */
#define LRS_E_TIMEOUT    -5  /* a bounded wait (multi-GPU exchange) ran out */
#define LRS_E_NCCL       -6  /* an NCCL call failed */
#define LRS_E_INTERNAL   -7  /* an internal consistency check failed (a bug; please report) */

#define LRS_TOKEN_NONE   0xFFFFFFFFu

/* ---- per-row parameters ----------------------------------------------------
 * One row's SamplingParams (sampler.rs:3-13) without the seed: the seed only
 * initialises the PRNG state (Sampler::new, sampler.rs:33-37), which the batched
 * API carries separately as uint64_t state[rows].
 * top_k == 0 means "off" exactly as in the reference (sampler.rs:122).
 * repeat_last_n == 0 means "the whole history" (sampler.rs:84-88).           */
typedef struct lrs_params {
    float    temperature;
    uint32_t top_k;
    float    top_p;
    float    repetition_penalty;
    uint32_t repeat_last_n;
    uint32_t reserved;          /* must be 0 */
} lrs_params;

/* Defaults of SamplingParams::default() (sampler.rs:15-26). */
#define LRS_DEFAULT_TEMPERATURE   0.7f
#define LRS_DEFAULT_TOP_K         40u
#define LRS_DEFAULT_TOP_P         0.95f
#define LRS_DEFAULT_PENALTY       1.1f
#define LRS_DEFAULT_LAST_N        64u
#define LRS_DEFAULT_SEED          0x123456789abcdef0ull

/* Optional per-row diagnostics written by the kernels (tests and tools use them to
 * check every intermediate of sampler.rs against a CPU restatement).            */
typedef struct lrs_row_info {
    int32_t  status;     /* LRS_OK or LRS_E_NAN */
    uint32_t token;
    uint32_t path;       /* 0 greedy fast path (sampler.rs:62-70), 1 greedy after penalty
                            (sampler.rs:104-113), 2 stochastic, 3 stochastic with n == 1 */
    uint32_t k;          /* effective top-k (sampler.rs:122-126) */
    uint32_t cutoff;     /* survivors after top-p (sampler.rs:135-146) */
    uint32_t pos;        /* position of the drawn token in the sorted survivor list */
    float    max;        /* softmax max over the scaled logits (ops.rs:401-406) */
    float    sum_exp;    /* softmax sequential f32 sum (ops.rs:408-411) */
    float    surv_sum;   /* survivor sum (sampler.rs:148-151) */
    float    r0;         /* next_f32() * sum (sampler.rs:155) */
    float    prob;       /* probability of the returned token */
    uint32_t n_cand;     /* candidates examined after the streaming pass (implementation detail) */
    uint32_t events;     /* ordered (exact) steps taken by the sum emulation (implementation detail) */
    uint32_t cycles[8];  /* rows of the persistent kernel: SM clock cycles (saturating) by phase: 0
                            max/filter pass, 1 estimates and thresholds, 2 softmax-sum pass, 3
                            top-k/top-p/draw, 7 sorting within 3; rows finished by the staged
                            pipeline: 4 is 1, 0-2 the cycles of its prep, sum and finish stages,
                            3, 6 and 7 those of the finish's regather, sorts and sequential runs,
                            5 the blocks its sum walked; rows of a nucleus larger than a list
                            (sampled by the big-nucleus stage, n_cand the keys it bucketed): 2 its
                            cycles, 3 those of counting and scattering the keys, 6 of the two
                            walks and 7 of the sorts within them (implementation detail) */
    uint32_t reserved;
} lrs_row_info;

typedef struct lrs_ctx lrs_ctx;

/* ---- context ---------------------------------------------------------------
 * Replaces: nothing in the reference holds device state; a context owns the GPU
 * resources that a sequence of Sampler::sample calls (model.rs:752-771,
 * server.rs:182-187, main.rs:552-577) would otherwise re-create per call.
 * max_rows rows of up to max_vocab logits and max_hist history ids per call.     */
int  lrs_create(int device, uint32_t max_rows, uint32_t max_vocab, uint32_t max_hist, lrs_ctx** out);
int  lrs_destroy(lrs_ctx* ctx);
const char* lrs_last_error(const lrs_ctx* ctx);

/* ---- PRNG state ----------------------------------------------------------------
 * Replaces Sampler::new(seed) (sampler.rs:33-37): lrs_seed_state returns seed | 1.
 * State arrays are host memory, `rows` entries, copied to/from the context.      */
uint64_t lrs_seed_state(uint64_t seed);
int  lrs_set_state(lrs_ctx* ctx, const uint64_t* state, uint32_t rows);
int  lrs_get_state(lrs_ctx* ctx, uint64_t* state, uint32_t rows);
int  lrs_set_params(lrs_ctx* ctx, const lrs_params* params, uint32_t rows);

/* ---- batched sampling from host buffers ---------------------------------------
 * Replaces `rows` calls of Sampler::sample (sampler.rs:56) on independent samplers.
 *   logits   host (or device if logits_on_device) f32[rows][ld], row r = logits + r*ld,
 *            n = vocab entries used per row (n <= ld, n <= max_vocab)
 *   hist     host u32[rows][hist_ld]; row r's history is hist[r*hist_ld .. + hist_len[r]]
 *            (the `recent` slice: prompt ids + generated ids, oldest first)
 *   out_tokens host u32[rows]; out_probs (nullable) host f32[rows]: probability of the
 *            returned token (1.0f for greedy rows)
 * Parameters and PRNG state come from lrs_set_params / lrs_set_state; the state is
 * advanced exactly as sampler.rs advances it (one next_u64 per stochastic row).
 * Synchronous: returns after the results are in host memory.                       */
int  lrs_sample(lrs_ctx* ctx, const float* logits, int logits_on_device, uint32_t rows,
                uint32_t n, uint64_t ld, const uint32_t* hist, uint64_t hist_ld,
                const uint32_t* hist_len, uint32_t* out_tokens, float* out_probs);

/* ---- batched sampling on device buffers (the hot path) -------------------------
 * Same computation, every pointer a device pointer, enqueued on `stream`
 * (a cudaStream_t, NULL = legacy default stream), no host synchronisation.
 * d_params[rows], d_state[rows] (read and advanced in place), d_tokens[rows],
 * d_probs[rows] (nullable), d_status[rows] (nullable, int32), d_info[rows] (nullable).
 * Returns LRS_OK once enqueued; row errors are reported through d_status.
 * Errors of the launch as a whole (a bounded wait that ran out, LRS_E_TIMEOUT, or a
 * failed internal check, LRS_E_INTERNAL) are also kept in the context's sticky error
 * word, so that they are seen when d_status is NULL: the next call on the context
 * returns such an error of an earlier launch once it is known on the host (that call
 * is then not enqueued), and lrs_poll_error waits for the last launch and returns it.  */
int  lrs_sample_device(lrs_ctx* ctx, const float* d_logits, uint32_t rows, uint32_t n, uint64_t ld,
                       const uint32_t* d_hist, uint64_t hist_ld, const uint32_t* d_hist_len,
                       const lrs_params* d_params, uint64_t* d_state,
                       uint32_t* d_tokens, float* d_probs, int32_t* d_status,
                       lrs_row_info* d_info, void* stream);
/* Replaces: nothing (the reference's sampler cannot fail this way).  Waits for the
 * context's last launch and returns (and clears) the error it reported: LRS_OK,
 * LRS_E_TIMEOUT or LRS_E_INTERNAL; LRS_E_CUDA if the wait itself failed.          */
int  lrs_poll_error(lrs_ctx* ctx);

/* Test of the bounded waits (no counterpart in the reference): enqueues one block that
 * waits `bound_cycles` SM cycles for an mbarrier phase that nothing completes, with the
 * wait primitive every wait of the sampling kernel uses.  The wait runs out and sets the
 * context's sticky error word to LRS_E_TIMEOUT, which the next call or lrs_poll_error
 * returns; the context stays usable.  Returns LRS_OK once enqueued.                  */
int  lrs_test_wait_timeout(lrs_ctx* ctx, uint32_t bound_cycles, void* stream);

/* ---- batched sampling without allocation ----------------------------------------
 * No counterpart in the reference (rust-llama has no GPU path); an addition for callers
 * that cannot let a library allocate device memory, e.g. a server whose GPU memory is
 * handed to its own pool at start-up, or a plug-in host that forbids allocations after
 * initialisation.  Same computation and arguments as lrs_sample_device, without a
 * context: the kernel's working memory is a fixed set of file-scope device arrays
 * (LRS_NOALLOC_SCRATCH_BYTES of candidate scratch plus the libm-expf table), held on
 * each GPU where the library's device code is loaded until the process exits.  Nothing
 * is allocated by this call, and no per-row diagnostics are written.
 *   device   the GPU that owns every buffer; the calling thread's current device is
 *            restored before returning
 *   n        1 <= n <= LRS_NOALLOC_MAX_VOCAB, otherwise LRS_E_INVALID
 * The first call on a device sets that device up once (array addresses, table copy):
 * make it outside any stream capture.  All calls on a device share the arrays, so calls
 * whose kernels can overlap on the GPU race with each other: issue them on one stream.
 * Returns LRS_OK once enqueued, LRS_E_INVALID for bad arguments (or a missing or
 * mismatching libm-expf table), LRS_E_CUDA if a CUDA call failed; row errors go to
 * d_status as with lrs_sample_device, and an error of the launch as a whole (a bounded
 * wait that ran out, a failed internal check) stays in the device's sticky error word
 * until lrs_noalloc_poll_error reads it: pass d_status, or poll, to see such errors.
 * Parallelism: the kernel runs as many CTAs as the fixed scratch holds at this n, at
 * most one per row: 84 at n = 151,936 (the context entry point runs 296 on a B200), 49
 * at the largest n.  Throughput on large batches is lower than lrs_sample_device's by
 * about that ratio; small batches (up to 84 rows at n = 151,936) are not affected.   */
#define LRS_NOALLOC_SCRATCH_BYTES (128u << 20)
#define LRS_NOALLOC_MAX_VOCAB     262144u
int  lrs_sample_device_noalloc(int device, const float* d_logits, uint32_t rows, uint32_t n, uint64_t ld,
                               const uint32_t* d_hist, uint64_t hist_ld, const uint32_t* d_hist_len,
                               const lrs_params* d_params, uint64_t* d_state,
                               uint32_t* d_tokens, float* d_probs, int32_t* d_status, void* stream);
/* No counterpart in the reference.  Waits for the work enqueued on `stream` and returns
 * (and clears) the device's sticky error word of lrs_sample_device_noalloc launches:
 * LRS_OK, LRS_E_TIMEOUT or LRS_E_INTERNAL; the set-up's error if set-up failed for good. */
int  lrs_noalloc_poll_error(int device, void* stream);

/* ---- vocabulary-sharded rows (multi-GPU exchange) -------------------------------
 * lrs_assemble_shards  the exchange step of vocabulary sharding: G ranks each hold
 *                      columns [g*shard_n, (g+1)*shard_n) of `rows` rows; after one
 *                      all-gather (NCCL, rank-major: d_gathered[g][row][col]) this writes
 *                      the full rows d_out[row][g*shard_n + col] (leading dimension
 *                      ld_out >= G*shard_n), ready for lrs_sample_device.  It replaces the
 *                      per-rank logits slice a tensor-parallel LM head would hand to
 *                      Sampler::sample (model.rs:752-761 calls it with the full vocab).
 * Enqueued on `stream` (cudaStream_t); returns LRS_OK, LRS_E_INVALID or LRS_E_CUDA.   */
int  lrs_assemble_shards(const float* d_gathered, uint32_t shards, uint32_t rows, uint32_t shard_n,
                         float* d_out, uint64_t ld_out, void* stream);

/* ---- batched generation loop: its per-row state on the device ---------------------
 * lrs_history_append  replaces `recent.push(next)` after each draw of the generation loops
 *                     (model.rs:768, server.rs:187; `recent` starts as the prompt ids,
 *                     model.rs:758, server.rs:182): for every row r < rows whose d_status[r]
 *                     is LRS_OK (d_status NULL: every row) and whose token is neither `eos`
 *                     (the loops stop before the push, model.rs:761-763) nor LRS_TOKEN_NONE,
 *                     appends d_tokens[r] to row r's history d_hist[r*hist_ld ..] and
 *                     increments d_hist_len[r], the same history layout lrs_sample_device
 *                     reads.  A row whose history already holds hist_ld ids first keeps its
 *                     last `keep` (1 <= keep <= hist_ld / 2, LRS_E_INVALID otherwise): the
 *                     penalty window (sampler.rs:84-88) stays exact while repeat_last_n <= keep
 *                     (repeat_last_n == 0, the whole history, while a row has held at most
 *                     hist_ld ids).  A loop then uploads its prompts once and no history after.
 * lrs_remap_tokens    sampling on rows of a pruned vocabulary (prune.rs:187-195 renumbers the
 *                     kept ids in order): d_out[r] = d_map[d_tokens[r]] (the original id of
 *                     pruned id t is d_map[t], t < map_n) where d_status[r] is LRS_OK (or
 *                     d_status is NULL), otherwise d_out[r] = d_tokens[r]; d_out may be
 *                     d_tokens.  Keep the history in pruned ids (the logits' id space).
 * Both are enqueued on `stream` (cudaStream_t) with device pointers; they return LRS_OK,
 * LRS_E_INVALID or LRS_E_CUDA.                                                        */
int  lrs_history_append(const uint32_t* d_tokens, const int32_t* d_status, uint32_t rows, uint32_t eos,
                        uint32_t* d_hist, uint64_t hist_ld, uint32_t* d_hist_len, uint32_t keep, void* stream);
int  lrs_remap_tokens(const uint32_t* d_tokens, const int32_t* d_status, uint32_t rows,
                      const uint32_t* d_map, uint32_t map_n, uint32_t* d_out, void* stream);

/* ---- single-row drop-in (Sampler API) -------------------------------------------
 * lrs_sampler_new    replaces Sampler::new(seed)               (sampler.rs:33-37)
 * lrs_sampler_sample replaces Sampler::sample(logits, params, recent) (sampler.rs:56)
 *                    host slices in, token out; *status (nullable) gets LRS_OK or an error;
 *                    on error the token is LRS_TOKEN_NONE.
 * A sampler lazily creates a one-row context on `device` sized to the first call.   */
typedef struct lrs_sampler lrs_sampler;
lrs_sampler* lrs_sampler_new(uint64_t seed, int device);
void         lrs_sampler_free(lrs_sampler* s);
uint64_t     lrs_sampler_state(const lrs_sampler* s);
uint32_t     lrs_sampler_sample(lrs_sampler* s, const float* logits, size_t n,
                                const lrs_params* params, const uint32_t* recent,
                                size_t recent_len, int* status);

#ifdef __cplusplus
}
#endif
#endif /* LLAMARS_SAMPLER_H */
