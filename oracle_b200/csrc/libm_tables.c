/* libm_tables.c -- build-time generator of the float exp / log1p correction
 * tables that make the decoder's transcendentals equal to the C library the
 * reference runs on.
 *
 * Oracle's decoder computes sigmoid, SiLU, softplus, the recurrent decay and
 * the attention softmax with std::exp / std::log1p on floats
 * (qwen35_block.cpp:138-159, reference_kernels.cpp:296, cpu_backend.cpp:166),
 * i.e. with the host C library's expf / log1pf.  Those are not correctly
 * rounded everywhere (glibc 2.39: expf differs from the correctly rounded
 * value on ~7.6e-5 of inputs, log1pf on ~1.5 %), and the Q8_K contract makes
 * any last-bit difference visible: a one-ulp change of an activation can move
 * a quantized value or a block scale, and the difference grows along the
 * recurrence.  The GPU therefore evaluates
 *     exp(x) or log1p(x) in double precision, rounded once to float
 * (the correctly rounded value whenever the exact result is not within 2^-48,
 * relative, of a float rounding midpoint: CUDA's double exp / log1p are within
 * 1 ulp of double, 2^-52), and corrects it from these tables:
 *     expf:   every float x in [-104, 89] where this library's expf(x) differs
 *             from the correctly rounded value, or where the exact value lies
 *             within 2^-48 of a midpoint (value: the library's result);
 *     log1pf: the same over y = expf(v) for every float v in [-20, 20] -- the
 *             only arguments log1pf gets (softplus, whose other branches
 *             return v or expf(v)).
 * "Correctly rounded" is decided from long double evaluations (expl, log1pl:
 * 64-bit significands, errors far below the 2^-48 margin).
 *
 * Output (little-endian uint32 words):
 *   [0] magic 0x314D424C ("LBM1"), [1] expf entries, [2] log1pf entries, [3] 0,
 *   expf bucket offsets (2^20 + 1 words; bucket = key bits >> 12),
 *   log1pf bucket offsets (2^20 + 1 words),
 *   expf entries (key bits, value bits) sorted by key, then log1pf entries.
 *
 * Usage: libm_tables <out.bin>   (8 threads, a few minutes) */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define BUCKETS (1u << 20)
#define THREADS 8

typedef struct {
    uint32_t key, value;
} Entry;

typedef struct {
    Entry* e;
    size_t n, cap;
} Vec;

static void push(Vec* v, uint32_t key, uint32_t value) {
    if (v->n == v->cap) {
        v->cap = v->cap ? 2 * v->cap : 4096;
        v->e = realloc(v->e, v->cap * sizeof(Entry));
        if (!v->e) {
            fprintf(stderr, "libm_tables: out of memory\n");
            exit(1);
        }
    }
    v->e[v->n].key = key;
    v->e[v->n].value = value;
    ++v->n;
}

static float from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static uint32_t to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

/* Distance of v to the nearest float rounding midpoint, relative to |v|. */
static long double midpoint_distance(long double v) {
    const float f = (float)v;
    const long double a = f, up = nextafterf(f, INFINITY), dn = nextafterf(f, -INFINITY);
    const long double d1 = fabsl(v - (a + up) / 2), d2 = fabsl(v - (a + dn) / 2);
    return (d1 < d2 ? d1 : d2) / fabsl(v);
}

/* Does the GPU's double-then-round evaluation need the library's value? */
static int needs_entry(float lib, long double exact, long double margin) {
    if (!isfinite(exact) || exact == 0.0L) return to_bits(lib) != to_bits((float)exact);
    return to_bits(lib) != to_bits((float)exact) || midpoint_distance(exact) < margin;
}

typedef struct {
    uint64_t lo, hi; /* bit patterns [lo, hi) */
    Vec exp_v, l1p_v;
} Job;

static void* work(void* arg) {
    Job* j = (Job*)arg;
    const long double margin = ldexpl(1.0L, -48);
    uint32_t last_y = 0xFFFFFFFFu;
    for (uint64_t u = j->lo; u < j->hi; ++u) {
        const float x = from_bits((uint32_t)u);
        if (x != x) continue;
        if (x >= -104.0f && x <= 89.0f) {
            const float lib = expf(x);
            if (needs_entry(lib, expl((long double)x), margin)) push(&j->exp_v, (uint32_t)u, to_bits(lib));
        }
        if (x >= -20.0f && x <= 20.0f) {
            const float y = expf(x);
            const uint32_t yb = to_bits(y);
            if (yb != last_y) { /* consecutive x give runs of equal y */
                last_y = yb;
                const float lib = log1pf(y);
                if (needs_entry(lib, log1pl((long double)y), margin)) push(&j->l1p_v, yb, to_bits(lib));
            }
        }
    }
    return NULL;
}

static int by_key(const void* a, const void* b) {
    const uint32_t x = ((const Entry*)a)->key, y = ((const Entry*)b)->key;
    return x < y ? -1 : x > y;
}

/* Merge the threads' lists, sort, drop duplicate keys, build bucket offsets. */
static Vec merge(Job* jobs, int which, uint32_t* offsets) {
    Vec out = {0};
    for (int t = 0; t < THREADS; ++t) {
        Vec* v = which ? &jobs[t].l1p_v : &jobs[t].exp_v;
        for (size_t i = 0; i < v->n; ++i) push(&out, v->e[i].key, v->e[i].value);
    }
    qsort(out.e, out.n, sizeof(Entry), by_key);
    size_t w = 0;
    for (size_t i = 0; i < out.n; ++i)
        if (w == 0 || out.e[w - 1].key != out.e[i].key) out.e[w++] = out.e[i];
    out.n = w;
    size_t i = 0;
    for (uint32_t b = 0; b <= BUCKETS; ++b) {
        while (i < out.n && (out.e[i].key >> 12) < b) ++i;
        offsets[b] = (uint32_t)i;
    }
    return out;
}

int main(int argc, char** argv) {
    if (argc != 2) {
        fprintf(stderr, "usage: libm_tables <out.bin>\n");
        return 2;
    }
    Job jobs[THREADS];
    pthread_t th[THREADS];
    const uint64_t total = 1ull << 32;
    for (int t = 0; t < THREADS; ++t) {
        memset(&jobs[t], 0, sizeof(Job));
        jobs[t].lo = total * t / THREADS;
        jobs[t].hi = total * (t + 1) / THREADS;
        pthread_create(&th[t], NULL, work, &jobs[t]);
    }
    for (int t = 0; t < THREADS; ++t) pthread_join(th[t], NULL);
    uint32_t* off_exp = malloc((BUCKETS + 1) * sizeof(uint32_t));
    uint32_t* off_l1p = malloc((BUCKETS + 1) * sizeof(uint32_t));
    Vec ve = merge(jobs, 0, off_exp), vl = merge(jobs, 1, off_l1p);
    char tmp[4096];
    snprintf(tmp, sizeof tmp, "%s.tmp", argv[1]);
    FILE* f = fopen(tmp, "wb");
    if (!f) {
        perror(tmp);
        return 1;
    }
    const uint32_t hdr[4] = {0x314D424Cu, (uint32_t)ve.n, (uint32_t)vl.n, 0u};
    fwrite(hdr, sizeof hdr, 1, f);
    fwrite(off_exp, sizeof(uint32_t), BUCKETS + 1, f);
    fwrite(off_l1p, sizeof(uint32_t), BUCKETS + 1, f);
    fwrite(ve.e, sizeof(Entry), ve.n, f);
    fwrite(vl.e, sizeof(Entry), vl.n, f);
    if (fclose(f) != 0 || rename(tmp, argv[1]) != 0) {
        perror(argv[1]);
        return 1;
    }
    printf("libm_tables: %zu expf and %zu log1pf entries -> %s\n", ve.n, vl.n, argv[1]);
    return 0;
}
