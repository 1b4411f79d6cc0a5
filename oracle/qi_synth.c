/*
 * qi_synth.c -- seeded synthetic inputs and BF16/FP16 conversions for the
 * CPU oracle.  TEST INFRASTRUCTURE ONLY (see qi_oracle.c).
 *
 * Compiled with -ffp-contract=off: the generator's multiply and add must stay
 * two IEEE roundings so that the device generator (csrc/synth.cu, which uses
 * __fmul_rn/__fadd_rn) reproduces the same bits, and the RoPE table must round
 * like the reference's host build (no FMA contraction), bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------- */
/* Synthetic data.  The benchmark configurations specify seeded N(0, s^2)
 * weights and activations; the reference's own tests ship no fixtures, so the
 * inputs are generated.  The generator below is integer-only up to a single
 * int->float conversion and two IEEE multiplies, so the CUDA generator in the
 * product (csrc/synth.cu) produces the same bits on the device.
 * Distribution: Irwin-Hall sum of four 24-bit uniforms, centred and scaled to
 * unit variance (a bounded approximation of N(0,1), |z| <= 3.46).            */

static inline uint64_t sm64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* FNV-1a of a tensor name mixed with the base seed. */
uint64_t or_seed_for(uint64_t base, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (const unsigned char* p = (const unsigned char*)name; *p; ++p) {
        h ^= *p;
        h *= 0x100000001b3ull;
    }
    return sm64(base ^ h);
}

#define OR_UNIT_SCALE 0x1.bb67aep-24f /* sqrt(3) / 2^24 rounded to float: unit variance */

static inline float or_unit_normal(uint64_t seed_mixed, int64_t i) {
    uint64_t h1 = sm64(seed_mixed + 2ull * (uint64_t)i);
    uint64_t h2 = sm64(seed_mixed + 2ull * (uint64_t)i + 1ull);
    const uint64_t m24 = 0xFFFFFFull;
    int64_t s = (int64_t)(h1 & m24) + (int64_t)((h1 >> 24) & m24) +
                (int64_t)(h2 & m24) + (int64_t)((h2 >> 24) & m24);
    int32_t c = (int32_t)(s - 33554430); /* 4 * (2^24 - 1) / 2 */
    return (float)c * OR_UNIT_SCALE;
}

static inline uint16_t f32_to_bf16_rn(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* out[i] = z_i * scale + offset (offset added only when nonzero, as a separate
 * rounding step: the device generator does the same with __fmul_rn/__fadd_rn). */
void or_gen_f32(uint64_t seed, int64_t n, float scale, float offset, float* out) {
    uint64_t sm = sm64(seed);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float v = or_unit_normal(sm, i) * scale;
        if (offset != 0.0f) v = v + offset;
        out[i] = v;
    }
}

void or_gen_bf16(uint64_t seed, int64_t n, float scale, float offset, uint16_t* out) {
    uint64_t sm = sm64(seed);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float v = or_unit_normal(sm, i) * scale;
        if (offset != 0.0f) v = v + offset;
        out[i] = f32_to_bf16_rn(v);
    }
}

void or_bf16_to_f32(const uint16_t* in, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

void or_f32_to_bf16(const float* in, int64_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rn(in[i]);
}

/* ------------------------------------------------------------------------- */
/* FP16 helpers (IEEE binary16, round to nearest even).                      */

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);       /* NaN */
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);      /* overflow -> inf */
    if (absx < 0x38800000u) {                                        /* subnormal half */
        if (absx < 0x33000000u) return (uint16_t)sign;               /* < 2^-25 -> 0 (ties to even at 2^-25 -> 0) */
        uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
        int e = (int)(absx >> 23);                                   /* 102..112 */
        int shift = 126 - e;                                         /* 14..24 */
        uint32_t r = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((absx >> 13) - (112u << 10));
    uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        if (m == 0) u = sign;
        else {
            float f = (float)m * 5.9604644775390625e-08f; /* 2^-24 */
            memcpy(&u, &f, 4);
            u |= sign;
        }
    } else if (e == 31) u = sign | 0x7f800000u | (m << 13);
    else u = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}


void or_f32_to_f16_arr(const float* in, int64_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = or_f32_to_f16(in[i]);
}


/* ------------------------------------------------------------------------- */
/* 3-axis RoPE table (rope.h:25-47 rope(), :89-116 embed_nd, :119-156
 * gen_flux_img_ids with scale_rope, :159-172 gen_qwen_image_ids, :175-180
 * gen_qwen_image_pe).  Output [n_txt + n_img, 64, 2, 2] FP32 ordered
 * txt-then-img, each pair [cos, -sin, sin, cos].  h, w are LATENT sizes.    */

static void linspace_f(float start, float end, int num, float* out) {
    if (num == 1) { out[0] = start; return; }
    float step = (end - start) / (float)(num - 1);
    for (int i = 0; i < num; ++i) out[i] = start + (float)i * step;
}

void or_rope_table(int h, int w, int n_txt, float* pe) {
    const int patch = 2;
    const int axes[3] = {16, 56, 56};
    const float theta = 10000.0f;
    int h_len = (h + patch / 2) / patch;
    int w_len = (w + patch / 2) / patch;
    int n_img = h_len * w_len;
    int n = n_txt + n_img;
    float* ids = (float*)malloc(sizeof(float) * 3 * (size_t)n);
    int txt_start = h_len > w_len ? h_len : w_len;
    float* tl = (float*)malloc(sizeof(float) * (size_t)(n_txt > 0 ? n_txt : 1));
    if (n_txt > 0) linspace_f((float)txt_start, (float)(n_txt + txt_start), n_txt, tl);
    for (int j = 0; j < n_txt; ++j) ids[3 * j] = ids[3 * j + 1] = ids[3 * j + 2] = tl[j];
    free(tl);
    int hs = -(h_len / 2), ws = -(w_len / 2);
    float* rows = (float*)malloc(sizeof(float) * (size_t)h_len);
    float* cols = (float*)malloc(sizeof(float) * (size_t)w_len);
    linspace_f((float)hs, (float)(hs + h_len - 1), h_len, rows);
    linspace_f((float)ws, (float)(ws + w_len - 1), w_len, cols);
    for (int i = 0; i < h_len; ++i)
        for (int j = 0; j < w_len; ++j) {
            int p = n_txt + i * w_len + j;
            ids[3 * p] = 0.0f;
            ids[3 * p + 1] = rows[i];
            ids[3 * p + 2] = cols[j];
        }
    free(rows);
    free(cols);
    int off = 0;
    for (int a = 0; a < 3; ++a) {
        int dim = axes[a], hd = dim / 2;
        float* sc = (float*)malloc(sizeof(float) * (size_t)hd);
        linspace_f(0.0f, (dim * 1.0f - 2.0f) / dim, hd, sc);
        for (int p = 0; p < n; ++p)
            for (int j = 0; j < hd; ++j) {
                float omega = 1.0f / powf(theta, sc[j]);
                float ang = ids[3 * p + a] * omega;
                float* e = pe + (size_t)p * 256 + (size_t)(off + j) * 4;
                e[0] = cosf(ang);
                e[1] = -sinf(ang);
                e[2] = sinf(ang);
                e[3] = cosf(ang);
            }
        off += hd;
        free(sc);
    }
    free(ids);
}

