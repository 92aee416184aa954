/*
 * quant_oracle.c -- CPU restatement of Oracle's quantized-weight path.
 *
 * TEST INFRASTRUCTURE ONLY (see quant_oracle.h for provenance and scope).
 * Build with -ffp-contract=off: every f32 expression below must round after
 * each operation, exactly as Oracle's scalar C++ does.
 */
#include "quant_oracle.h"

#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- helpers */

static uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static uint32_t rd_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}

static float bits_to_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint32_t f32_to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static int8_t as_i8(uint8_t v) { return (int8_t)v; }

/* IEEE binary16 -> binary32, exact for every input (storage_decode.cpp:150-176):
 * subnormals are renormalised, inf/NaN keep their payload bits. */
float oq_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0x1Fu) return bits_to_f32(sign | 0x7F800000u | (man << 13));
    if (exp != 0) return bits_to_f32(sign | ((exp + 112u) << 23) | (man << 13));
    if (man == 0) return bits_to_f32(sign);
    /* subnormal: value = man * 2^-24; shift until the implicit bit appears */
    int e = -14;
    while (!(man & 0x400u)) {
        man <<= 1;
        e -= 1;
    }
    return bits_to_f32(sign | ((uint32_t)(e + 127) << 23) | ((man & 0x3FFu) << 13));
}

float oq_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

uint16_t oq_f32_to_bf16_rne(float value) {
    uint32_t u = f32_to_bits(value);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------------------- layout */

typedef struct {
    uint32_t type;
    uint32_t block_elems;
    uint32_t block_bytes;
} oq_layout;

/* The subset of the GGML layout table (ggml_type.cpp:12-56) this path uses. */
static const oq_layout k_layouts[] = {
    {OQ_TYPE_F32, 1, 4},     {OQ_TYPE_F16, 1, 2},     {OQ_TYPE_Q8_0, 32, 34},
    {OQ_TYPE_Q4_K, 256, 144}, {OQ_TYPE_Q5_K, 256, 176}, {OQ_TYPE_Q6_K, 256, 210},
    {OQ_TYPE_Q8_K, 256, 292}, {OQ_TYPE_BF16, 1, 2},
};

static const oq_layout* find_layout(uint32_t type) {
    for (size_t i = 0; i < sizeof(k_layouts) / sizeof(k_layouts[0]); ++i)
        if (k_layouts[i].type == type) return &k_layouts[i];
    return NULL;
}

uint64_t oq_row_bytes(uint32_t type, uint64_t k) {
    const oq_layout* l = find_layout(type);
    if (!l || k == 0 || k % l->block_elems) return 0;
    return (k / l->block_elems) * l->block_bytes;
}

/* ---------------------------------------------------------------- decode */

/* 6-bit (scale, min) of sub-block j from the 12 packed bytes
 * (storage_decode.cpp:44-61): bytes 0-3 hold scale j / top bits of scale j+4,
 * bytes 4-7 min j / top bits of min j+4, bytes 8-11 the low nibbles of
 * scale j+4 (low) and min j+4 (high). */
static void k4_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void decode_q8_0(const uint8_t* b, float* y) {
    float d = oq_f16_to_f32(rd_u16(b));
    for (int i = 0; i < 32; ++i) y[i] = d * (float)as_i8(b[2 + i]);
}

/* Element e of a 256-block sits in 64-wide group e/64; the first 32 take the
 * low nibble of qs[32*group + e%32], the next 32 the high nibble; its
 * sub-block is 2*group + (upper half).  value = (d*sc)*q - dmin*m. */
static void decode_q4_k(const uint8_t* b, float* y) {
    float d = oq_f16_to_f32(rd_u16(b));
    float dmin = oq_f16_to_f32(rd_u16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    for (int g = 0; g < 4; ++g) {
        for (int half = 0; half < 2; ++half) {
            int sc, mn;
            k4_scale_min(scales, 2 * g + half, &sc, &mn);
            for (int l = 0; l < 32; ++l) {
                uint8_t byte = qs[32 * g + l];
                int q = half ? (byte >> 4) : (byte & 0x0F);
                y[64 * g + 32 * half + l] = d * (float)sc * (float)q - dmin * (float)mn;
            }
        }
    }
}

/* Q5_K adds bit (2*group + half) of qh[l] as the fifth quant bit
 * (storage_decode.cpp:63-94). */
static void decode_q5_k(const uint8_t* b, float* y) {
    float d = oq_f16_to_f32(rd_u16(b));
    float dmin = oq_f16_to_f32(rd_u16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int g = 0; g < 4; ++g) {
        for (int half = 0; half < 2; ++half) {
            int sc, mn;
            k4_scale_min(scales, 2 * g + half, &sc, &mn);
            for (int l = 0; l < 32; ++l) {
                uint8_t byte = qs[32 * g + l];
                int q = half ? (byte >> 4) : (byte & 0x0F);
                if (qh[l] & (1u << (2 * g + half))) q += 16;
                y[64 * g + 32 * half + l] = d * (float)sc * (float)q - dmin * (float)mn;
            }
        }
    }
}

/* Q6_K: two halves of 128; in half h, segment s (32 wide) lane l reads
 * ql[64h + l + 32*(s&1)] (low nibble for s<2, high for s>=2) and bits
 * 2s..2s+1 of qh[32h + l]; quant = (low | high<<4) - 32; scale index
 * 8h + l/16 + 2s (storage_decode.cpp:96-125). */
static void decode_q6_k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const uint8_t* sc = b + 192;
    float d = oq_f16_to_f32(rd_u16(b + 208));
    for (int h = 0; h < 2; ++h) {
        for (int s = 0; s < 4; ++s) {
            for (int l = 0; l < 32; ++l) {
                uint8_t lo_byte = ql[64 * h + l + ((s & 1) ? 32 : 0)];
                int lo = (s >= 2) ? (lo_byte >> 4) : (lo_byte & 0x0F);
                int hi = (qh[32 * h + l] >> (2 * s)) & 3;
                int q = (lo | (hi << 4)) - 32;
                int scale = as_i8(sc[8 * h + l / 16 + 2 * s]);
                y[128 * h + 32 * s + l] = d * (float)scale * (float)q;
            }
        }
    }
}

int oq_decode_row(uint32_t type, uint64_t k, const uint8_t* row, float* out) {
    if (!oq_row_bytes(type, k)) return find_layout(type) ? OQ_EINVAL : OQ_EUNSUPPORTED;
    switch (type) {
        case OQ_TYPE_F32:
            for (uint64_t i = 0; i < k; ++i) out[i] = bits_to_f32(rd_u32(row + 4 * i));
            return OQ_OK;
        case OQ_TYPE_F16:
            for (uint64_t i = 0; i < k; ++i) out[i] = oq_f16_to_f32(rd_u16(row + 2 * i));
            return OQ_OK;
        case OQ_TYPE_BF16:
            for (uint64_t i = 0; i < k; ++i) out[i] = oq_bf16_to_f32(rd_u16(row + 2 * i));
            return OQ_OK;
        case OQ_TYPE_Q8_0:
            for (uint64_t b = 0; b < k / 32; ++b) decode_q8_0(row + 34 * b, out + 32 * b);
            return OQ_OK;
        case OQ_TYPE_Q4_K:
            for (uint64_t b = 0; b < k / 256; ++b) decode_q4_k(row + 144 * b, out + 256 * b);
            return OQ_OK;
        case OQ_TYPE_Q5_K:
            for (uint64_t b = 0; b < k / 256; ++b) decode_q5_k(row + 176 * b, out + 256 * b);
            return OQ_OK;
        case OQ_TYPE_Q6_K:
            for (uint64_t b = 0; b < k / 256; ++b) decode_q6_k(row + 210 * b, out + 256 * b);
            return OQ_OK;
        default:
            return OQ_EUNSUPPORTED;
    }
}

/* ---------------------------------------------------------------- Q8_K */

/* GGML quantize_row_q8_K_ref, restated.  Per 256-block: the element of
 * largest magnitude (first one on ties) gives max; iscale = -127/max;
 * q = round-half-even(iscale * x) clamped above at 127; bsums[i] = sum of
 * qs[16i..16i+15]; d = 1/iscale.  An all-zero block stores d = 0, qs = 0 and
 * bsums = 0 (GGML leaves bsums untouched there; zero is what they sum to). */
int oq_quantize_row_q8_k(const float* x, uint64_t k, uint8_t* out) {
    if (k == 0 || k % 256) return OQ_EINVAL;
    for (uint64_t b = 0; b < k / 256; ++b) {
        const float* xb = x + 256 * b;
        uint8_t* blk = out + 292 * b;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 256; ++j) {
            float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                vmax = xb[j];
            }
        }
        int8_t qs[256];
        int16_t bsums[16];
        float d = 0.0f;
        if (amax == 0.0f) {
            memset(qs, 0, sizeof qs);
            memset(bsums, 0, sizeof bsums);
        } else {
            float iscale = -127.0f / vmax;
            for (int j = 0; j < 256; ++j) {
                float v = iscale * xb[j];
                int q = (int)rintf(v); /* default rounding: nearest, ties to even */
                qs[j] = (int8_t)(q > 127 ? 127 : q);
            }
            for (int i = 0; i < 16; ++i) {
                int s = 0;
                for (int j = 0; j < 16; ++j) s += qs[16 * i + j];
                bsums[i] = (int16_t)s;
            }
            d = 1.0f / iscale;
        }
        uint32_t dbits = f32_to_bits(d);
        for (int i = 0; i < 4; ++i) blk[i] = (uint8_t)(dbits >> (8 * i));
        memcpy(blk + 4, qs, 256);
        for (int i = 0; i < 16; ++i) {
            blk[260 + 2 * i] = (uint8_t)((uint16_t)bsums[i] & 0xFF);
            blk[261 + 2 * i] = (uint8_t)((uint16_t)bsums[i] >> 8);
        }
    }
    return OQ_OK;
}

static float q8k_d(const uint8_t* blk) { return bits_to_f32(rd_u32(blk)); }
static int q8k_q(const uint8_t* blk, int i) { return as_i8(blk[4 + i]); }
static int q8k_bsum(const uint8_t* blk, int i) { return (int16_t)rd_u16(blk + 260 + 2 * i); }

/* ---------------------------------------------------------------- integer dots */

void oq_block_sums_q4_k(const uint8_t* w, const uint8_t* q8, int32_t* isum, int32_t* msum) {
    const uint8_t* scales = w + 4;
    const uint8_t* qs = w + 16;
    int32_t is = 0, ms = 0;
    for (int j = 0; j < 8; ++j) {
        int sc, mn;
        k4_scale_min(scales, j, &sc, &mn);
        int g = j / 2, half = j % 2;
        int32_t dot = 0;
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = qs[32 * g + l];
            int q = half ? (byte >> 4) : (byte & 0x0F);
            dot += q * q8k_q(q8, 32 * j + l);
        }
        is += sc * dot;
        ms += mn * (q8k_bsum(q8, 2 * j) + q8k_bsum(q8, 2 * j + 1));
    }
    *isum = is;
    *msum = ms;
}

void oq_block_sums_q6_k(const uint8_t* w, const uint8_t* q8, int32_t* isum, int32_t* msum) {
    const uint8_t* ql = w;
    const uint8_t* qh = w + 128;
    const uint8_t* sc = w + 192;
    int32_t dots[16] = {0};
    for (int h = 0; h < 2; ++h)
        for (int s = 0; s < 4; ++s)
            for (int l = 0; l < 32; ++l) {
                uint8_t lo_byte = ql[64 * h + l + ((s & 1) ? 32 : 0)];
                int lo = (s >= 2) ? (lo_byte >> 4) : (lo_byte & 0x0F);
                int hi = (qh[32 * h + l] >> (2 * s)) & 3;
                int e = 128 * h + 32 * s + l;
                dots[e / 16] += (lo | (hi << 4)) * q8k_q(q8, e);
            }
    int32_t is = 0;
    for (int i = 0; i < 16; ++i) is += as_i8(sc[i]) * (dots[i] - 32 * q8k_bsum(q8, i));
    *isum = is;
    *msum = 0;
}

static int kq_block_bytes(uint32_t type) {
    return type == OQ_TYPE_Q4_K ? 144 : type == OQ_TYPE_Q6_K ? 210 : 0;
}

/* f32 contribution of one super-block: (d_w*d_x)*isum - (dmin_w*d_x)*msum. */
static float kq_block_partial(uint32_t type, const uint8_t* w, const uint8_t* q8) {
    int32_t isum, msum;
    float dx = q8k_d(q8);
    if (type == OQ_TYPE_Q4_K) {
        oq_block_sums_q4_k(w, q8, &isum, &msum);
        float dd = oq_f16_to_f32(rd_u16(w)) * dx;
        float dm = oq_f16_to_f32(rd_u16(w + 2)) * dx;
        return dd * (float)isum - dm * (float)msum;
    }
    oq_block_sums_q6_k(w, q8, &isum, &msum);
    float dd = oq_f16_to_f32(rd_u16(w + 208)) * dx;
    return dd * (float)isum;
}

float oq_vec_dot_q8_k(uint32_t type, uint64_t k, const uint8_t* wrow, const uint8_t* q8row) {
    int bb = kq_block_bytes(type);
    if (!bb || k == 0 || k % 256) return NAN;
    const uint64_t nb = k / 256;
    float total = 0.0f;
    for (uint64_t g = 0; g * 16 < nb; ++g) {
        float leaf[16];
        for (int j = 0; j < 16; ++j) {
            const uint64_t i = 16 * g + (uint64_t)j;
            leaf[j] = 0.0f;
            if (i < nb) leaf[j] += kq_block_partial(type, wrow + (uint64_t)bb * i, q8row + 292 * i);
        }
        for (int stride = 8; stride >= 1; stride /= 2)
            for (int s = 0; s < stride; ++s) leaf[s] += leaf[s + stride];
        total += leaf[0];
    }
    return total;
}

/* GGML generic order: per super-block, 8 interleaved int32 partial sums of
 * scale*dot (lane l collects elements l, l+8, l+16, ...) are each scaled by
 * d_w*d_x into 8 running f32 sums; the min term is subtracted from one
 * running f32 total; the 8 sums are added to that total at the end. */
float oq_vec_dot_q8_k_ggml_order(uint32_t type, uint64_t k, const uint8_t* wrow,
                                 const uint8_t* q8row) {
    int bb = kq_block_bytes(type);
    if (!bb || k == 0 || k % 256) return NAN;
    float sums[8] = {0};
    float total = 0.0f;
    for (uint64_t i = 0; i < k / 256; ++i) {
        const uint8_t* w = wrow + (uint64_t)bb * i;
        const uint8_t* q8 = q8row + 292 * i;
        int32_t lanes[8] = {0};
        float dx = q8k_d(q8);
        if (type == OQ_TYPE_Q4_K) {
            const uint8_t* scales = w + 4;
            const uint8_t* qs = w + 16;
            int32_t msum = 0;
            for (int j = 0; j < 8; ++j) {
                int sc, mn;
                k4_scale_min(scales, j, &sc, &mn);
                for (int l = 0; l < 32; ++l) {
                    uint8_t byte = qs[32 * (j / 2) + l];
                    int q = (j % 2) ? (byte >> 4) : (byte & 0x0F);
                    lanes[l % 8] += sc * (q * q8k_q(q8, 32 * j + l));
                }
                msum += mn * (q8k_bsum(q8, 2 * j) + q8k_bsum(q8, 2 * j + 1));
            }
            float dd = oq_f16_to_f32(rd_u16(w)) * dx;
            for (int l = 0; l < 8; ++l) sums[l] += dd * (float)lanes[l];
            float dm = oq_f16_to_f32(rd_u16(w + 2)) * dx;
            total -= dm * (float)msum;
        } else {
            const uint8_t* ql = w;
            const uint8_t* qh = w + 128;
            const uint8_t* sc = w + 192;
            for (int e = 0; e < 256; ++e) {
                int h = e / 128, s = (e % 128) / 32, l = e % 32;
                uint8_t lo_byte = ql[64 * h + l + ((s & 1) ? 32 : 0)];
                int lo = (s >= 2) ? (lo_byte >> 4) : (lo_byte & 0x0F);
                int hi = (qh[32 * h + l] >> (2 * s)) & 3;
                int q = (lo | (hi << 4)) - 32;
                lanes[e % 8] += as_i8(sc[e / 16]) * (q * q8k_q(q8, e));
            }
            float dd = oq_f16_to_f32(rd_u16(w + 208)) * dx;
            for (int l = 0; l < 8; ++l) sums[l] += dd * (float)lanes[l];
        }
    }
    for (int l = 0; l < 8; ++l) total += sums[l];
    return total;
}

int oq_matvec_q8_k(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                   const uint8_t* q8k, uint64_t batch, float* y) {
    uint64_t rb = oq_row_bytes(type, k);
    if (!kq_block_bytes(type)) return OQ_EUNSUPPORTED;
    if (!rb || rows == 0 || batch == 0) return OQ_EINVAL;
    uint64_t xb = (k / 256) * 292;
    for (uint64_t b = 0; b < batch; ++b)
        for (uint64_t r = 0; r < rows; ++r)
            y[b * rows + r] = oq_vec_dot_q8_k(type, k, w + r * rb, q8k + b * xb);
    return OQ_OK;
}

/* ---------------------------------------------------------------- f32 contract */

/* Oracle's reference_storage_dot (quantized_reference.cpp:24-82): decode one
 * block at a time and add decoded*x into a single running f32 sum. */
float oq_storage_dot_f32(uint32_t type, uint64_t k, const uint8_t* row, const float* x) {
    const oq_layout* l = find_layout(type);
    if (!l || type == OQ_TYPE_Q8_K || !oq_row_bytes(type, k)) return NAN;
    uint32_t be = l->block_elems; /* 1, 32 or 256: the sum order is element order */
    float buf[256];
    float sum = 0.0f;
    for (uint64_t e = 0; e < k; e += be) {
        oq_decode_row(type, be, row + (e / l->block_elems) * l->block_bytes, buf);
        for (uint32_t i = 0; i < be; ++i) sum += buf[i] * x[e + i];
    }
    return sum;
}

int oq_storage_matvec_f32(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                          const float* x, uint64_t batch, float* y) {
    uint64_t rb = oq_row_bytes(type, k);
    if (!find_layout(type) || type == OQ_TYPE_Q8_K) return OQ_EUNSUPPORTED;
    if (!rb || rows == 0 || batch == 0) return OQ_EINVAL;
    for (uint64_t b = 0; b < batch; ++b)
        for (uint64_t r = 0; r < rows; ++r)
            y[b * rows + r] = oq_storage_dot_f32(type, k, w + r * rb, x + b * k);
    return OQ_OK;
}

int oq_storage_matvec_f64(uint32_t type, uint64_t rows, uint64_t k, const uint8_t* w,
                          const float* x, uint64_t batch, double* y) {
    uint64_t rb = oq_row_bytes(type, k);
    if (!find_layout(type) || type == OQ_TYPE_Q8_K) return OQ_EUNSUPPORTED;
    if (!rb || rows == 0 || batch == 0) return OQ_EINVAL;
    float* dec = (float*)malloc(sizeof(float) * k);
    if (!dec) return OQ_EINVAL;
    for (uint64_t r = 0; r < rows; ++r) {
        oq_decode_row(type, k, w + r * rb, dec);
        for (uint64_t b = 0; b < batch; ++b) {
            double s = 0.0;
            for (uint64_t i = 0; i < k; ++i) s += (double)dec[i] * (double)x[b * k + i];
            y[b * rows + r] = s;
        }
    }
    free(dec);
    return OQ_OK;
}

/* ---------------------------------------------------------------- prefill GEMM */

int oq_gemm_sampled(uint32_t type, uint64_t n, uint64_t k, const uint8_t* w, uint64_t m,
                    const float* x, uint64_t count, const uint64_t* mi, const uint64_t* ni,
                    int mode, double* y) {
    uint64_t rb = oq_row_bytes(type, k);
    if (!find_layout(type) || type == OQ_TYPE_Q8_K) return OQ_EUNSUPPORTED;
    if (!rb) return OQ_EINVAL;
    for (uint64_t c = 0; c < count; ++c)
        if (mi[c] >= m || ni[c] >= n) return OQ_EINVAL;
    float* dec = (float*)malloc(sizeof(float) * k);
    if (!dec) return OQ_EINVAL;
    uint64_t cached = (uint64_t)-1;
    for (uint64_t c = 0; c < count; ++c) {
        if (ni[c] != cached) {
            oq_decode_row(type, k, w + ni[c] * rb, dec);
            cached = ni[c];
        }
        const float* xr = x + mi[c] * k;
        double s = 0.0;
        for (uint64_t i = 0; i < k; ++i) {
            float a = xr[i], b = dec[i];
            if (mode == 1 || mode == 2) {
                a = oq_bf16_to_f32(oq_f32_to_bf16_rne(a));
                b = oq_bf16_to_f32(oq_f32_to_bf16_rne(b));
            }
            const double t = (double)a * (double)b;
            s += mode >= 2 ? fabs(t) : t;
        }
        y[c] = s;
    }
    free(dec);
    return OQ_OK;
}

/* qwen35_block.cpp:161-188 */
int oq_rms_norm_rows(const float* in, const float* weight, uint64_t rows, uint64_t width, float eps, float* out) {
    if (width == 0 || !(eps > 0.0f)) return OQ_EINVAL;
    for (uint64_t r = 0; r < rows; ++r) {
        const float* x = in + r * width;
        double sum = 0.0;
        for (uint64_t c = 0; c < width; ++c) {
            const double v = (double)x[c];
            sum += v * v;
        }
        const double mean = sum / (double)width;
        const float inv = (float)(1.0 / sqrt(mean + (double)eps));
        for (uint64_t c = 0; c < width; ++c) out[r * width + c] = x[c] * inv * weight[c];
    }
    return OQ_OK;
}

/* qwen35_block.cpp:138-145 */
static float oq_sigmoid(float v) {
    if (v >= 0.0f) {
        const float e = expf(-v);
        return 1.0f / (1.0f + e);
    }
    const float e = expf(v);
    return e / (1.0f + e);
}

/* qwen35_block.cpp:157-159, 315-318 */
void oq_swiglu(const float* gate, const float* up, uint64_t n, float* out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = gate[i] * oq_sigmoid(gate[i]) * up[i];
}
