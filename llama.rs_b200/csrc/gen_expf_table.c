/*
 * gen_expf_table.c — build step: records where this machine's libm expf differs
 * from a correctly rounded exp, over the softmax input domain d = x - max <= 0.
 *
 * Why: rust-llama's softmax (src/ops.rs:408-410) calls f32::exp, which on
 * x86_64-linux-gnu is libm's expf.  The GPU kernels compute a correctly rounded
 * exp (double-precision exp rounded once to float) and then replace it by libm's
 * value wherever the two differ, so every probability bit matches the reference.
 *
 * For every negative float d in [-104, -0] (below -104 both are 0) an entry
 * (bits(d), bits(expf(d))) is written when
 *   (a) expf(d) != (float)exp((double)d), or
 *   (b) exp(d) lies within 2^-16 float ulp of a rounding midpoint, where a
 *       double exp with a 1-ulp error bound could round either way.
 * Output: "LRSEXPF1", u32 count, u32 domain_lo, u32 domain_hi, then count pairs of
 * (u32 input bits, u32 output bits) sorted by input bits.
 * Compile: gcc -O2 -fno-fast-math -ffp-contract=off gen_expf_table.c -lm -pthread
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define DOMAIN_LO 0x80000001u /* -tiny */
#define DOMAIN_HI 0xC2D00000u /* -104.0 */
#define NTHREADS 16

typedef struct { uint32_t key, val; } entry_t;
typedef struct {
    uint32_t lo, hi;
    entry_t* out;
    size_t n, cap;
    int bad;
} job_t;

static float asf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t asu(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static void push(job_t* j, uint32_t k, uint32_t v) {
    if (j->n == j->cap) {
        j->cap = j->cap ? 2 * j->cap : 4096;
        j->out = (entry_t*)realloc(j->out, j->cap * sizeof(entry_t));
        if (!j->out) { j->bad = 1; return; }
    }
    j->out[j->n].key = k;
    j->out[j->n].val = v;
    j->n++;
}

static void* run(void* arg) {
    job_t* j = (job_t*)arg;
    for (uint32_t u = j->lo;; u++) {
        float x = asf(u);
        float g = expf(x);
        double d = exp((double)x);
        float c = (float)d;
        int hard = 0;
        if ((double)c != d && c != 0.0f) {
            float nb = (d > (double)c) ? nextafterf(c, INFINITY) : nextafterf(c, 0.0f);
            double mid = ((double)c + (double)nb) * 0.5;
            double ulp = fabs((double)nb - (double)c);
            if (fabs(d - mid) < ulp * 0x1p-16) hard = 1;
        }
        if (c == 0.0f && d > 0.0) {
            /* result rounds to zero or the smallest subnormal: check the midpoint 2^-150 */
            if (fabs(d - 0x1p-150) < 0x1p-165) hard = 1;
        }
        if (g != c || hard) {
            int32_t diff = (int32_t)asu(g) - (int32_t)asu(c);
            if (diff > 1 || diff < -1) j->bad = 1; /* libm must be within one ulp */
            push(j, u, asu(g));
        }
        if (u == j->hi) break;
    }
    return NULL;
}

int main(int argc, char** argv) {
    if (argc != 2) { fprintf(stderr, "usage: %s out.bin\n", argv[0]); return 2; }
    job_t jobs[NTHREADS];
    pthread_t th[NTHREADS];
    uint64_t span = (uint64_t)DOMAIN_HI - DOMAIN_LO + 1;
    for (int t = 0; t < NTHREADS; t++) {
        memset(&jobs[t], 0, sizeof(job_t));
        jobs[t].lo = (uint32_t)(DOMAIN_LO + span * t / NTHREADS);
        jobs[t].hi = (uint32_t)(DOMAIN_LO + span * (t + 1) / NTHREADS - 1);
        pthread_create(&th[t], NULL, run, &jobs[t]);
    }
    size_t total = 0;
    int bad = 0;
    for (int t = 0; t < NTHREADS; t++) {
        pthread_join(th[t], NULL);
        total += jobs[t].n;
        bad |= jobs[t].bad;
    }
    /* below the domain both sides are zero; spot-check it */
    for (float x = -104.0f; x > -200.0f; x -= 0.37f)
        if (expf(x) != 0.0f || (float)exp((double)x) != 0.0f) bad = 1;
    if (expf(-0.0f) != 1.0f || expf(0.0f) != 1.0f || expf(-INFINITY) != 0.0f) bad = 1;
    if (bad) { fprintf(stderr, "gen_expf_table: libm expf outside the expected bounds\n"); return 1; }
    FILE* f = fopen(argv[1], "wb");
    if (!f) { perror("fopen"); return 1; }
    uint32_t hdr[3] = {(uint32_t)total, DOMAIN_LO, DOMAIN_HI};
    fwrite("LRSEXPF1", 1, 8, f);
    fwrite(hdr, 4, 3, f);
    for (int t = 0; t < NTHREADS; t++) fwrite(jobs[t].out, sizeof(entry_t), jobs[t].n, f);
    fclose(f);
    printf("gen_expf_table: %zu entries\n", total);
    return 0;
}
