/*
 * kd_oracle.c -- CPU restatement of the CrossDiT attention hot path.
 * TEST INFRASTRUCTURE ONLY (see kd_oracle.h): the checker, never the product.
 *
 * Build: oracle/build_oracle.py (gcc -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp).
 * -ffp-contract=off keeps every a*b+c that the reference writes as two float
 * operations as two roundings; the places where ggml itself uses an FMA call
 * fmaf() explicitly.
 */
#include "kd_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__AVX2__) && defined(__F16C__) && defined(__FMA__)
#include <immintrin.h>
#define KDO_SIMD 1
#else
#define KDO_SIMD 0
#endif

/* ------------------------------------------------------------------------- */
/* conversions                                                               */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t kdo_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);          /* NaN */
    if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7c00u);         /* >= 2^16 -> inf */
    if (ax < 0x38800000u) {                                           /* below 2^-14: subnormal */
        float scaled = u2f(ax) * 16777216.0f;                        /* exact: times 2^24 */
        uint32_t m = (uint32_t)nearbyintf(scaled);                   /* ties to even */
        return (uint16_t)(sign | m);
    }
    uint32_t e = (ax >> 23) - 127u + 15u;
    uint32_t mant = ax & 0x7fffffu;
    uint32_t r = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;          /* carry may reach inf: correct */
    return (uint16_t)(sign | r);
}

float kdo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);                   /* m * 2^-24, exact */
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e - 15u + 127u) << 23) | (m << 13));
}

uint16_t kdo_f32_to_bf16(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float kdo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

void kdo_convert(const float* src, int64_t n, int32_t dst_type, void* dst) {
    if (dst_type == KDO_F32) { memcpy(dst, src, (size_t)n * 4); return; }
    uint16_t* d = (uint16_t*)dst;
    if (dst_type == KDO_F16) for (int64_t i = 0; i < n; ++i) d[i] = kdo_f32_to_f16(src[i]);
    else                     for (int64_t i = 0; i < n; ++i) d[i] = kdo_f32_to_bf16(src[i]);
}

void kdo_to_f32(const void* src, int32_t src_type, int64_t n, float* dst) {
    if (src_type == KDO_F32) { memcpy(dst, src, (size_t)n * 4); return; }
    const uint16_t* s = (const uint16_t*)src;
    if (src_type == KDO_F16) for (int64_t i = 0; i < n; ++i) dst[i] = kdo_f16_to_f32(s[i]);
    else                     for (int64_t i = 0; i < n; ++i) dst[i] = kdo_bf16_to_f32(s[i]);
}

static inline float load_as_f32(const void* p, int32_t type) {
    if (type == KDO_F32) return *(const float*)p;
    if (type == KDO_F16) return kdo_f16_to_f32(*(const uint16_t*)p);
    return kdo_bf16_to_f32(*(const uint16_t*)p);
}

/* value after rounding to `type` (what ggml's ggml_cast / q_to_vec_dot produce) */
static inline float round_to(float x, int32_t type) {
    if (type == KDO_F16) return kdo_f16_to_f32(kdo_f32_to_f16(x));
    if (type == KDO_BF16) return kdo_bf16_to_f32(kdo_f32_to_bf16(x));
    return x;
}

/* ------------------------------------------------------------------------- */
/* Philox4x32-10 + Box-Muller: src/rng.hpp:51-69 (randn), :94-112 (round),   */
/* :114-128 (10 rounds with key bumps), :130-134 (Box-Muller)                */
/* ------------------------------------------------------------------------- */

#define KDO_PHILOX_M0 0xD2511F53u
#define KDO_PHILOX_M1 0xCD9E8D57u
#define KDO_PHILOX_W0 0x9E3779B9u
#define KDO_PHILOX_W1 0xBB67AE85u

static float kdo_box_muller(float x, float y) {
    const float inv32 = 2.3283064e-10f;
    const float inv32_2pi = 2.3283064e-10f * 6.2831855f;
    float u = x * inv32 + inv32 / 2;
    float v = y * inv32_2pi + inv32_2pi / 2;
    return sqrtf(-2.0f * logf(u)) * sinf(v);
}

static void kdo_philox_one(uint32_t offset, uint32_t idx, uint64_t seed, uint32_t* o0, uint32_t* o1) {
    uint32_t c0 = offset, c1 = 0, c2 = idx, c3 = 0;
    uint32_t k0 = (uint32_t)(seed & 0xffffffffu), k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)c0 * (uint64_t)KDO_PHILOX_M0;
        uint64_t p1 = (uint64_t)c2 * (uint64_t)KDO_PHILOX_M1;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        if (r < 9) { k0 += KDO_PHILOX_W0; k1 += KDO_PHILOX_W1; }
    }
    *o0 = c0; *o1 = c1;
}

void kdo_philox_randn(uint64_t seed, uint32_t offset, uint64_t n, float* out, int nthreads) {
    (void)nthreads;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        uint32_t a, b;
        kdo_philox_one(offset, (uint32_t)i, seed, &a, &b);
        out[i] = kdo_box_muller((float)a, (float)b);
    }
}

/* ------------------------------------------------------------------------- */
/* RoPE: src/rope.hpp                                                        */
/* ------------------------------------------------------------------------- */

/* get_freqs, rope.hpp:23-29: exp(-log(theta) * i / dim) in float */
void kdo_rope_freqs(int dim, float theta, float* out) {
    for (int i = 0; i < dim; ++i) out[i] = expf(-logf(theta) * (float)i / (float)dim);
}

/* compute_text_rope, rope.hpp:36-49 */
void kdo_text_rope_table(int seq_len, int head_dim, float theta, float* out) {
    int half = head_dim / 2;
    float* f = (float*)malloc(sizeof(float) * (size_t)half);
    kdo_rope_freqs(half, theta, f);
    for (int pos = 0; pos < seq_len; ++pos)
        for (int d = 0; d < half; ++d) {
            float a = (float)pos * f[d];
            out[(size_t)pos * head_dim + 2 * d + 0] = cosf(a);
            out[(size_t)pos * head_dim + 2 * d + 1] = sinf(a);
        }
    free(f);
}

/* compute_visual_rope, rope.hpp:56-102: token idx = (t*H + h)*W + w; per axis a the
 * pairs of the axis block get angle = pos_a * freq_a[i] / scale_factor[a] */
void kdo_visual_rope_table(int n_frames, int height, int width, const int axes_dims[3],
                           const float scale_factor[3], float theta, float* out) {
    int total = axes_dims[0] + axes_dims[1] + axes_dims[2];
    float* fr[3];
    for (int a = 0; a < 3; ++a) {
        fr[a] = (float*)malloc(sizeof(float) * (size_t)(axes_dims[a] / 2 + 1));
        kdo_rope_freqs(axes_dims[a] / 2, theta, fr[a]);
    }
    for (int t = 0; t < n_frames; ++t)
        for (int h = 0; h < height; ++h)
            for (int w = 0; w < width; ++w) {
                size_t idx = ((size_t)t * height + h) * width + w;
                float* row = out + idx * total;
                int pos[3] = {t, h, w};
                int off = 0;
                for (int a = 0; a < 3; ++a) {
                    for (int d = 0; d < axes_dims[a] / 2; ++d) {
                        float ang = (float)pos[a] * fr[a][d] / scale_factor[a];
                        row[off + 2 * d + 0] = cosf(ang);
                        row[off + 2 * d + 1] = sinf(ang);
                    }
                    off += axes_dims[a];
                }
            }
    for (int a = 0; a < 3; ++a) free(fr[a]);
}

/* rope::apply, rope.hpp:109-155, on x = [head_dim, n_head, L, N] f32 in place:
 * (x0, x1) = (x[2i], x[2i+1]) -> (x0*c - x1*s, x0*s + x1*c), table row = token. */
void kdo_rope_apply(float* x, int64_t n_tokens, int64_t n_seq, int n_head, int head_dim,
                    const float* table, int nthreads) {
    (void)nthreads;
    int64_t rows = n_tokens * n_seq;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
    for (int64_t r = 0; r < rows; ++r) {
        int64_t tok = r % n_tokens;
        const float* cs = table + tok * head_dim;
        for (int h = 0; h < n_head; ++h) {
            float* v = x + (r * n_head + h) * head_dim;
            for (int i = 0; i < head_dim / 2; ++i) {
                float x0 = v[2 * i], x1 = v[2 * i + 1];
                float c = cs[2 * i], s = cs[2 * i + 1];
                float a = x0 * c;
                float b = x1 * s;
                float e = x0 * s;
                float g = x1 * c;
                v[2 * i] = a - b;
                v[2 * i + 1] = e + g;
            }
        }
    }
}

/* ggml rms_norm + mul by gain (ops.hpp:76-81): per head_dim row,
 * sum of float squares accumulated in double, mean -> float,
 * scale = 1/sqrtf(mean + eps), y = (x*scale)*g. gain == NULL means unit gain
 * (the multiply by 1 is exact). */
void kdo_rms_norm_heads(const float* x, int64_t n_rows, int head_dim, const float* gain, float eps,
                        float* y, int nthreads) {
    (void)nthreads;
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
    for (int64_t r = 0; r < n_rows; ++r) {
        const float* xr = x + r * head_dim;
        float* yr = y + r * head_dim;
        double sum = 0.0;
        for (int i = 0; i < head_dim; ++i) sum += (double)(xr[i] * xr[i]);
        float mean = (float)(sum / (double)head_dim);
        float scale = 1.0f / sqrtf(mean + eps);
        for (int i = 0; i < head_dim; ++i) {
            float t = xr[i] * scale;
            yr[i] = gain ? t * gain[i] : t;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* flash_attn_ext                                                            */
/* ------------------------------------------------------------------------- */

static int valid_type(int32_t t) { return t == KDO_F32 || t == KDO_F16 || t == KDO_BF16; }

/* f32 dot with the lane structure of ggml's AVX2 f16 dot (4 x 8-lane FMA
 * accumulators, pairwise reduce, then 8-lane horizontal add); leftovers in double. */
static inline float dot_ggml(const float* a, const float* b, int n) {
    float acc[32];
    for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
    int n32 = n & ~31;
    for (int i = 0; i < n32; i += 32)
        for (int l = 0; l < 32; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    for (int l = 0; l < 8; ++l) { acc[l] = acc[l] + acc[16 + l]; acc[8 + l] = acc[8 + l] + acc[24 + l]; }
    for (int l = 0; l < 8; ++l) acc[l] = acc[l] + acc[8 + l];
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = acc[l] + acc[4 + l];
    double s = (double)((t[0] + t[1]) + (t[2] + t[3]));
    for (int i = n32; i < n; ++i) s += (double)(a[i] * b[i]);
    return (float)s;
}

/* y = round_f16(fma(x, v, y)) over n (ggml_vec_mad_f16), y and x hold f16 values as f32 */
static inline void mad_f16(float* y, const float* x, float v, int n) {
    int i = 0;
#if KDO_SIMD
    __m256 vv = _mm256_set1_ps(v);
    for (; i + 8 <= n; i += 8) {
        __m256 r = _mm256_fmadd_ps(_mm256_loadu_ps(x + i), vv, _mm256_loadu_ps(y + i));
        _mm256_storeu_ps(y + i, _mm256_cvtph_ps(_mm256_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT)));
    }
#endif
    for (; i < n; ++i) y[i] = round_to(fmaf(x[i], v, y[i]), KDO_F16);
}

static inline void scale_f16(float* y, float v, int n) {
    int i = 0;
#if KDO_SIMD
    __m256 vv = _mm256_set1_ps(v);
    for (; i + 8 <= n; i += 8) {
        __m256 r = _mm256_mul_ps(_mm256_loadu_ps(y + i), vv);
        _mm256_storeu_ps(y + i, _mm256_cvtph_ps(_mm256_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT)));
    }
#endif
    for (; i < n; ++i) y[i] = round_to(y[i] * v, KDO_F16);
}

/* Load plane (i2, i3) of a [D, L, ., .] tensor into a dense f32 [L][D] buffer. */
static void load_plane(const kdo_tensor* t, int64_t i2, int64_t i3, float* dst) {
    const char* base = (const char*)t->data + i2 * t->nb[2] + i3 * t->nb[3];
    for (int64_t r = 0; r < t->ne[1]; ++r)
        for (int64_t d = 0; d < t->ne[0]; ++d)
            dst[r * t->ne[0] + d] = load_as_f32(base + r * t->nb[1] + d * t->nb[0], t->type);
}

int kdo_flash_attn_ext(const kdo_tensor* q, const kdo_tensor* k, const kdo_tensor* v,
                       const kdo_tensor* mask, float scale, const int32_t* kv_len, int mode,
                       float* out, float* lse, int nthreads) {
    if (!q || !k || !v || !out) return -1;
    if (!valid_type(q->type) || !valid_type(k->type) || !valid_type(v->type)) return -2;
    const int64_t DK = q->ne[0], Lq = q->ne[1], H = q->ne[2], N = q->ne[3];
    const int64_t Lk = k->ne[1], Hkv = k->ne[2], Nkv = k->ne[3], DV = v->ne[0];
    if (k->ne[0] != DK || v->ne[1] != Lk || v->ne[2] != Hkv || v->ne[3] != Nkv) return -3;
    if (Hkv <= 0 || Nkv <= 0 || H % Hkv != 0 || N % Nkv != 0) return -4;
    if (mask) {
        if (mask->type != KDO_F16 || mask->ne[0] < Lk || mask->ne[1] < Lq) return -5;
        if (mask->ne[2] <= 0 || mask->ne[3] <= 0 || H % mask->ne[2] != 0 || N % mask->ne[3] != 0) return -6;
    }
    const int64_t rk2 = H / Hkv, rk3 = N / Nkv;
    const int32_t dot_type = (k->type == KDO_F32) ? KDO_F32 : k->type;   /* q_to_vec_dot target */
    const int nth = nthreads > 0 ? nthreads : 1;
    const int64_t RB = 16;                                               /* query rows per task */
    const int64_t nrb = (Lq + RB - 1) / RB;

    /* dense f32 copies of the (exactly converted) K and V planes */
    float* kf = (float*)malloc(sizeof(float) * (size_t)(Hkv * Nkv * Lk * DK));
    float* vf = (float*)malloc(sizeof(float) * (size_t)(Hkv * Nkv * Lk * DV));
    if (!kf || !vf) { free(kf); free(vf); return -7; }
    for (int64_t n3 = 0; n3 < Nkv; ++n3)
        for (int64_t h2 = 0; h2 < Hkv; ++h2) {
            load_plane(k, h2, n3, kf + (n3 * Hkv + h2) * Lk * DK);
            load_plane(v, h2, n3, vf + (n3 * Hkv + h2) * Lk * DV);
        }

#pragma omp parallel num_threads(nth)
    {
        float* qr = (float*)malloc(sizeof(float) * (size_t)DK);
        float* acc = (float*)malloc(sizeof(float) * (size_t)DV);
        double* sbuf = (double*)malloc(sizeof(double) * (size_t)(Lk > 0 ? Lk : 1));
        double* oacc = (double*)malloc(sizeof(double) * (size_t)DV);
#pragma omp for schedule(dynamic, 1)
        for (int64_t task = 0; task < N * H * nrb; ++task) {
            const int64_t n = task / (H * nrb), h = (task / nrb) % H, rb = task % nrb;
            const int64_t hk = h / rk2, nk = n / rk3;
            const float* K = kf + (nk * Hkv + hk) * Lk * DK;
            const float* V = vf + (nk * Hkv + hk) * Lk * DV;
            int64_t lk_eff = Lk;
            if (kv_len) { int64_t kl = kv_len[n]; lk_eff = kl < 0 ? 0 : (kl < Lk ? kl : Lk); }
            for (int64_t i = rb * RB; i < Lq && i < (rb + 1) * RB; ++i) {
                const char* qp = (const char*)q->data + i * q->nb[1] + h * q->nb[2] + n * q->nb[3];
                for (int64_t d = 0; d < DK; ++d) qr[d] = round_to(load_as_f32(qp + d * q->nb[0], q->type), dot_type);
                const uint16_t* mp = NULL;
                if (mask)
                    mp = (const uint16_t*)((const char*)mask->data + i * mask->nb[1] +
                                           (h % mask->ne[2]) * mask->nb[2] + (n % mask->ne[3]) * mask->nb[3]);
                float* orow = out + ((n * Lq + i) * H + h) * DV;

                /* exact log-sum-exp and (exact mode) output in double */
                double M = -INFINITY;
                const int64_t lk_exact = (mode == KDO_MODE_EXACT || lse) ? lk_eff : 0;
                for (int64_t j = 0; j < lk_exact; ++j) {
                    double mv = 0.0;
                    if (mp) {
                        float mf = kdo_f16_to_f32(*(const uint16_t*)((const char*)mp + j * mask->nb[0]));
                        if (mf == -INFINITY) { sbuf[j] = -INFINITY; continue; }
                        mv = mf;
                    }
                    double s = 0.0;
                    for (int64_t d = 0; d < DK; ++d) s += (double)qr[d] * (double)K[j * DK + d];
                    sbuf[j] = s * (double)scale + mv;
                    if (sbuf[j] > M) M = sbuf[j];
                }
                double S = 0.0;
                for (int64_t d = 0; d < DV; ++d) oacc[d] = 0.0;
                if (M != -INFINITY) {
                    for (int64_t j = 0; j < lk_exact; ++j) {
                        if (sbuf[j] == -INFINITY) continue;
                        double p = exp(sbuf[j] - M);
                        S += p;
                        if (mode == KDO_MODE_EXACT)
                            for (int64_t d = 0; d < DV; ++d) oacc[d] += p * (double)V[j * DV + d];
                    }
                }
                if (lse) lse[(n * H + h) * Lq + i] = (M == -INFINITY) ? -INFINITY : (float)(M + log(S));

                if (mode == KDO_MODE_EXACT) {
                    for (int64_t d = 0; d < DV; ++d) orow[d] = S > 0.0 ? (float)(oacc[d] / S) : 0.0f;
                    continue;
                }

                /* ggml-faithful online softmax (ggml-cpu flash_attn_ext one-chunk kernel) */
                float Mf = -INFINITY, Sf = 0.0f;
                const int v_f16 = (v->type == KDO_F16);
                for (int64_t d = 0; d < DV; ++d) acc[d] = 0.0f;
                for (int64_t j = 0; j < lk_eff; ++j) {
                    float mv = 0.0f;
                    if (mp) {
                        mv = kdo_f16_to_f32(*(const uint16_t*)((const char*)mp + j * mask->nb[0]));
                        if (mv == -INFINITY) continue;
                    }
                    float s = dot_ggml(qr, K + j * DK, (int)DK);
                    s = s * scale;
                    s += mv;
                    const float Mold = Mf;
                    float ms = 1.0f, vs = 1.0f;
                    if (s > Mf) {
                        Mf = s;
                        ms = expf(Mold - Mf);
                        if (v_f16) scale_f16(acc, ms, (int)DV);
                        else for (int64_t d = 0; d < DV; ++d) acc[d] *= ms;
                    } else {
                        vs = expf(s - Mf);
                    }
                    if (v_f16) mad_f16(acc, V + j * DV, vs, (int)DV);
                    else for (int64_t d = 0; d < DV; ++d) acc[d] = fmaf(V[j * DV + d], vs, acc[d]);
                    Sf = Sf * ms + vs;
                }
                const float Sinv = Sf == 0.0f ? 0.0f : 1.0f / Sf;
                for (int64_t d = 0; d < DV; ++d) orow[d] = acc[d] * Sinv;
            }
        }
        free(qr); free(acc); free(sbuf); free(oacc);
    }
    free(kf); free(vf);
    return 0;
}
