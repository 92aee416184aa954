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
 * recurrence.  The GPU evaluates exp(x) or log1p(x) in double precision and
 * rounds once to float -- the correctly rounded value whenever its double is
 * at least 2^-49 (relative) away from a float rounding midpoint, since CUDA's
 * double exp / log1p are within 1 ulp (2^-52) -- and corrects it from:
 *
 *   exceptions  every input of the domain where the library's result differs
 *               from the correctly rounded one.  The library is then always
 *               the other float neighbour of the exact value (checked here),
 *               so an entry is the input plus one direction bit; entries live
 *               in an open-addressing hash table of 128-byte lines (32 keys,
 *               load factor <= 0.6), so a lookup is one line read (two when
 *               its line is full);
 *   hard        every input whose exact value is within 2^-48 of a midpoint
 *               (the only ones where the GPU's rounding could differ from the
 *               correctly rounded value), with the library's result; sorted,
 *               searched only when the GPU's double lands within 2^-49.
 *
 * Domains: expf on [-104, 89]; log1pf on y = expf(v) for every float v in
 * [-20, 20] -- the only arguments log1pf gets (softplus, whose other branches
 * return v or expf(v)).  "Correctly rounded" and "near a midpoint" are decided
 * from long double evaluations (expl, log1pl: 64-bit significands).
 *
 * Output (little-endian uint32 words):
 *   [0] magic 0x324D424C ("LBM2"), [1] expf lines (power of 2),
 *   [2] log1pf lines (power of 2), [3] expf hard entries, [4] log1pf hard
 *   entries, [5..7] 0;
 *   expf key lines (32 words each; empty slot 0xFFFFFFFF);
 *   expf direction bits (one per slot: 1 = library is one float above);
 *   log1pf key lines (key | direction << 31; the keys are positive floats);
 *   expf hard (key, value) pairs sorted by key; log1pf hard pairs.
 * Line of a key: (key * 0x9E3779B1) >> (32 - log2(lines)); a full line
 * continues in the next one.
 *
 * Usage: libm_tables <out.bin>   (8 threads, about a minute) */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define THREADS 8
#define SLOTS 32u
#define EMPTY 0xFFFFFFFFu

typedef struct {
    uint32_t key, value, cr;
} Entry;

typedef struct {
    Entry* e;
    size_t n, cap;
} Vec;

static void push(Vec* v, uint32_t key, uint32_t value, uint32_t cr) {
    if (v->n == v->cap) {
        v->cap = v->cap ? 2 * v->cap : 4096;
        v->e = realloc(v->e, v->cap * sizeof(Entry));
        if (!v->e) {
            fprintf(stderr, "libm_tables: out of memory\n");
            exit(1);
        }
    }
    v->e[v->n++] = (Entry){key, value, cr};
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

typedef struct {
    uint64_t lo, hi; /* bit patterns [lo, hi) */
    Vec exc[2], hard[2];
} Job;

static void classify(Job* j, int fn, uint32_t key, float lib, long double exact) {
    const float cr = (float)exact;
    if (to_bits(lib) != to_bits(cr)) push(&j->exc[fn], key, to_bits(lib), to_bits(cr));
    if (isfinite(exact) && exact != 0.0L && midpoint_distance(exact) < ldexpl(1.0L, -48))
        push(&j->hard[fn], key, to_bits(lib), to_bits(cr));
}

static void* work(void* arg) {
    Job* j = (Job*)arg;
    uint32_t last_y = EMPTY;
    for (uint64_t u = j->lo; u < j->hi; ++u) {
        const float x = from_bits((uint32_t)u);
        if (x != x) continue;
        if (x >= -104.0f && x <= 89.0f) classify(j, 0, (uint32_t)u, expf(x), expl((long double)x));
        if (x >= -20.0f && x <= 20.0f) {
            const float y = expf(x);
            const uint32_t yb = to_bits(y);
            if (yb != last_y) { /* consecutive x give runs of equal y */
                last_y = yb;
                classify(j, 1, yb, log1pf(y), log1pl((long double)y));
            }
        }
    }
    return NULL;
}

static int by_key(const void* a, const void* b) {
    const uint32_t x = ((const Entry*)a)->key, y = ((const Entry*)b)->key;
    return x < y ? -1 : x > y;
}

static Vec gather(Job* jobs, int fn, int hard) {
    Vec out = {0};
    for (int t = 0; t < THREADS; ++t) {
        Vec* v = hard ? &jobs[t].hard[fn] : &jobs[t].exc[fn];
        for (size_t i = 0; i < v->n; ++i) push(&out, v->e[i].key, v->e[i].value, v->e[i].cr);
    }
    qsort(out.e, out.n, sizeof(Entry), by_key);
    size_t w = 0;
    for (size_t i = 0; i < out.n; ++i)
        if (w == 0 || out.e[w - 1].key != out.e[i].key) out.e[w++] = out.e[i];
    out.n = w;
    return out;
}

static uint32_t line_of(uint32_t key, uint32_t log2_lines) {
    return (uint32_t)((key * 0x9E3779B1u) >> (32u - log2_lines));
}

/* Hash the exceptions into lines (load factor <= 0.6).  keys: lines * SLOTS
 * words; dir: one bit per slot (expf), or in bit 31 of the key (log1pf). */
static uint32_t* build_lines(const Vec* exc, int dir_in_key, uint32_t* log2_out, uint32_t** dir_out) {
    uint32_t lg = 4;
    while ((1ull << lg) * SLOTS * 3 < 5ull * exc->n) ++lg;
    const uint32_t lines = 1u << lg;
    uint32_t* keys = malloc((size_t)lines * SLOTS * sizeof(uint32_t));
    uint32_t* dir = calloc(lines, sizeof(uint32_t));
    uint32_t* fill = calloc(lines, sizeof(uint32_t));
    memset(keys, 0xFF, (size_t)lines * SLOTS * sizeof(uint32_t));
    for (size_t i = 0; i < exc->n; ++i) {
        const Entry* e = &exc->e[i];
        /* the library is the other neighbour of the exact value: one ulp away */
        const int64_t step = (int64_t)(int32_t)e->value - (int64_t)(int32_t)e->cr;
        if (step != 1 && step != -1) {
            fprintf(stderr, "libm_tables: %08x is %lld ulp from the correctly rounded value\n", e->key,
                    (long long)step);
            exit(1);
        }
        uint32_t key = e->key;
        if (dir_in_key) {
            if (key & 0x80000000u) {
                fprintf(stderr, "libm_tables: log1pf key %08x is not a positive float\n", key);
                exit(1);
            }
            key |= step > 0 ? 0x80000000u : 0u;
        }
        uint32_t l = line_of(e->key, lg);
        while (fill[l] == SLOTS) l = (l + 1) & (lines - 1);
        const uint32_t slot = l * SLOTS + fill[l]++;
        keys[slot] = key;
        if (step > 0) dir[slot / 32] |= 1u << (slot % 32);
    }
    free(fill);
    *log2_out = lg;
    *dir_out = dir;
    return keys;
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
    Vec exc_e = gather(jobs, 0, 0), exc_l = gather(jobs, 1, 0);
    Vec hard_e = gather(jobs, 0, 1), hard_l = gather(jobs, 1, 1);
    uint32_t lg_e, lg_l, *dir_e, *dir_l;
    uint32_t* keys_e = build_lines(&exc_e, 0, &lg_e, &dir_e);
    uint32_t* keys_l = build_lines(&exc_l, 1, &lg_l, &dir_l);
    const uint32_t lines_e = 1u << lg_e, lines_l = 1u << lg_l;
    char tmp[4096];
    snprintf(tmp, sizeof tmp, "%s.tmp", argv[1]);
    FILE* f = fopen(tmp, "wb");
    if (!f) {
        perror(tmp);
        return 1;
    }
    const uint32_t hdr[8] = {0x324D424Cu, lines_e, lines_l, (uint32_t)hard_e.n, (uint32_t)hard_l.n, 0, 0, 0};
    fwrite(hdr, sizeof hdr, 1, f);
    fwrite(keys_e, sizeof(uint32_t), (size_t)lines_e * SLOTS, f);
    fwrite(dir_e, sizeof(uint32_t), lines_e, f);
    fwrite(keys_l, sizeof(uint32_t), (size_t)lines_l * SLOTS, f);
    for (int k = 0; k < 2; ++k) {
        const Vec* h = k ? &hard_l : &hard_e;
        for (size_t i = 0; i < h->n; ++i) {
            const uint32_t kv[2] = {h->e[i].key, h->e[i].value};
            fwrite(kv, sizeof kv, 1, f);
        }
    }
    if (fclose(f) != 0 || rename(tmp, argv[1]) != 0) {
        perror(argv[1]);
        return 1;
    }
    printf("libm_tables: expf %zu exceptions (%u lines), %zu hard; log1pf %zu exceptions (%u lines), %zu hard -> %s\n",
           exc_e.n, lines_e, hard_e.n, exc_l.n, lines_l, hard_l.n, argv[1]);
    return 0;
}
