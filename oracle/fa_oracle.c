/*
 * fa_oracle.c -- CPU restatement of ggml_flash_attn_ext (TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs load
 * this library; the product (acestep.cpp_b200/libacefa.so) never does.
 *
 * What it restates, and from where:
 *   - The operator contract as acestep.cpp calls it: ggml_flash_attn_ext(q, k, v,
 *     mask, scale, max_bias, softcap) with PREC_F32 (src/qwen3-lm.h:465-469,
 *     :789-794; src/qwen3-enc.h:195-199; src/dit-graph.h:227-231, :348-352).
 *   - GQA head mapping k-head = q-head / (Hq/Hkv) and batch broadcast
 *     k-batch = q-batch / (B/Bk); mask broadcast by modulo over heads and batch
 *     (src/dit-graph.h:513-529 builds [n_kv, n_q, 1, N] masks).
 *   - Mask element addressing mask[b*nb3 + qi*nb1 + ki*2] (src/dit-sampler.h:263-280,
 *     src/qwen3-lm.h:875-881); a -inf entry removes the key entirely.
 *   - Output permuted to [Dv, Hq, n_q, B] (src/dit-graph.h:233-235).
 *   - The ggml CPU kernel's per-row online softmax: keys with a -inf mask are
 *     skipped, scale then optional softcap (s = c*tanh(s*scale/c)), then
 *     slope*mask is added; an all-masked row yields 0.  Restated from ggml's
 *     published flash-attention algorithm (the ggml submodule, pinned at an
 *     unrecoverable commit, is absent from the reference tree: .gitmodules:1-3).
 *   - ALiBi slopes from max_bias (ggml convention: m0 = 2^(-max_bias/n), m1 =
 *     2^(-max_bias/2/n), n = 2^floor(log2(Hq))).
 *   - Q8_0 blocks {fp16 d; int8 qs[32]} with d = amax/127, qs = roundf(x/d).
 *
 * Parity: the attention arithmetic is UNPINNED (no ggml here, no reference
 * golden vectors); the Q8_0 format is pinned against gguf 0.19.0.
 */
#include "fa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ------------------------------------------------------------------ */
/* scalar conversions                                                  */
/* ------------------------------------------------------------------ */

uint16_t ora_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp  = (x >> 23) & 0xffu;
    uint32_t man  = x & 0x7fffffu;
    if (exp == 0xffu) {
        return (uint16_t) (sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    }
    int e = (int) exp - 127 + 15;
    if (e >= 31) {
        return (uint16_t) (sign | 0x7c00u);
    }
    if (e <= 0) {
        if (e < -10) {
            return (uint16_t) sign;
        }
        man |= 0x800000u;
        int      shift   = 14 - e;
        uint32_t h       = man >> shift;
        uint32_t rem     = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) {
            h++;
        }
        return (uint16_t) (sign | h);
    }
    uint32_t h   = ((uint32_t) e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        h++; /* a carry into the exponent is the correct rounding (up to inf) */
    }
    return (uint16_t) (sign | h);
}

float ora_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    uint32_t exp  = ((uint32_t) h >> 10) & 0x1fu;
    uint32_t man  = (uint32_t) h & 0x3ffu;
    uint32_t x;
    float    f;
    if (exp == 0) {
        f = (float) man * 5.9604644775390625e-8f; /* man * 2^-24, exact */
        memcpy(&x, &f, 4);
        x |= sign;
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    memcpy(&f, &x, 4);
    return f;
}

uint16_t ora_fp32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        return (uint16_t) ((u >> 16) | 64u); /* quiet NaN */
    }
    return (uint16_t) ((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

float ora_bf16_to_fp32(uint16_t h) {
    uint32_t u = (uint32_t) h << 16;
    float    f;
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------------ */
/* Q8_0                                                                */
/* ------------------------------------------------------------------ */

#define QK8_0 32
#define Q8_0_BYTES 34

void ora_quantize_q8_0(const float *x, uint8_t *y, int64_t n) {
    const int64_t nb = n / QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            const float v = fabsf(x[i * QK8_0 + j]);
            if (v > amax) {
                amax = v;
            }
        }
        const float d  = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t    dh = ora_fp32_to_fp16(d);
        uint8_t    *b  = y + i * Q8_0_BYTES;
        memcpy(b, &dh, 2);
        for (int j = 0; j < QK8_0; j++) {
            const float v = x[i * QK8_0 + j] * id;
            b[2 + j]      = (uint8_t) (int8_t) roundf(v);
        }
    }
}

void ora_dequantize_q8_0(const uint8_t *y, float *x, int64_t n) {
    const int64_t nb = n / QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *b = y + i * Q8_0_BYTES;
        uint16_t       dh;
        memcpy(&dh, b, 2);
        const float d = ora_fp16_to_fp32(dh);
        for (int j = 0; j < QK8_0; j++) {
            x[i * QK8_0 + j] = (float) (int8_t) b[2 + j] * d;
        }
    }
}

/* ------------------------------------------------------------------ */
/* row loaders                                                         */
/* ------------------------------------------------------------------ */

static void row_to_f32(int type, const uint8_t *row, size_t nb0, int64_t n, float *out) {
    switch (type) {
        case ORA_F32:
            for (int64_t i = 0; i < n; i++) {
                memcpy(&out[i], row + i * nb0, 4);
            }
            break;
        case ORA_F16:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                memcpy(&h, row + i * nb0, 2);
                out[i] = ora_fp16_to_fp32(h);
            }
            break;
        case ORA_BF16:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                memcpy(&h, row + i * nb0, 2);
                out[i] = ora_bf16_to_fp32(h);
            }
            break;
        case ORA_Q8_0:
            ora_dequantize_q8_0(row, out, n);
            break;
    }
}

static float alibi_slope(float max_bias, int64_t h, int64_t n_head) {
    if (max_bias <= 0.0f) {
        return 1.0f;
    }
    const uint32_t n_head_log2 = 1u << (uint32_t) floorf(log2f((float) n_head));
    const float    m0          = powf(2.0f, -(max_bias) / (float) n_head_log2);
    const float    m1          = powf(2.0f, -(max_bias / 2.0f) / (float) n_head_log2);
    return h < (int64_t) n_head_log2 ? powf(m0, (float) (h + 1)) : powf(m1, (float) (2 * (h - n_head_log2) + 1));
}

/* ------------------------------------------------------------------ */
/* ggml-cpu-like dot products (f32 accumulation, 8 lanes when F16C)   */
/* ------------------------------------------------------------------ */

#if defined(__x86_64__)
__attribute__((target("avx2,f16c,fma"))) static float dot_f16_avx(const uint16_t *a, const uint16_t *b, int64_t n) {
    __m256  acc = _mm256_setzero_ps();
    int64_t i   = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 x = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (a + i)));
        __m256 y = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (b + i)));
        acc      = _mm256_fmadd_ps(x, y, acc);
    }
    float t[8];
    _mm256_storeu_ps(t, acc);
    float s = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    for (; i < n; i++) {
        s += ora_fp16_to_fp32(a[i]) * ora_fp16_to_fp32(b[i]);
    }
    return s;
}

/* y = f16(f32(y)*ms + f32(x)*vs), rounded per element as ggml_vec_scale_f16 + ggml_vec_mad_f16 */
__attribute__((target("avx2,f16c,fma"))) static void scale_f16_avx(uint16_t *y, int64_t n, float v) {
    __m256  vv = _mm256_set1_ps(v);
    int64_t i  = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 a = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (y + i)));
        _mm_storeu_si128((__m128i *) (y + i), _mm256_cvtps_ph(_mm256_mul_ps(a, vv), 0));
    }
    for (; i < n; i++) {
        y[i] = ora_fp32_to_fp16(ora_fp16_to_fp32(y[i]) * v);
    }
}

__attribute__((target("avx2,f16c,fma"))) static void mad_f16_avx(uint16_t *y, const uint16_t *x, int64_t n, float v) {
    __m256  vv = _mm256_set1_ps(v);
    int64_t i  = 0;
    for (; i + 8 <= n; i += 8) {
        __m256 a = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (y + i)));
        __m256 b = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *) (x + i)));
        _mm_storeu_si128((__m128i *) (y + i), _mm256_cvtps_ph(_mm256_fmadd_ps(b, vv, a), 0));
    }
    for (; i < n; i++) {
        y[i] = ora_fp32_to_fp16(ora_fp16_to_fp32(y[i]) + ora_fp16_to_fp32(x[i]) * v);
    }
}
#endif

static int g_have_f16c = -1;

static int have_f16c(void) {
#if defined(__x86_64__)
    if (g_have_f16c < 0) {
        __builtin_cpu_init();
        g_have_f16c = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("f16c") && __builtin_cpu_supports("fma");
    }
    return g_have_f16c;
#else
    return 0;
#endif
}

static float dot_f16(const uint16_t *a, const uint16_t *b, int64_t n) {
#if defined(__x86_64__)
    if (have_f16c()) {
        return dot_f16_avx(a, b, n);
    }
#endif
    float s = 0.0f;
    for (int64_t i = 0; i < n; i++) {
        s += ora_fp16_to_fp32(a[i]) * ora_fp16_to_fp32(b[i]);
    }
    return s;
}

static void scale_f16(uint16_t *y, int64_t n, float v) {
#if defined(__x86_64__)
    if (have_f16c()) {
        scale_f16_avx(y, n, v);
        return;
    }
#endif
    for (int64_t i = 0; i < n; i++) {
        y[i] = ora_fp32_to_fp16(ora_fp16_to_fp32(y[i]) * v);
    }
}

static void mad_f16(uint16_t *y, const uint16_t *x, int64_t n, float v) {
#if defined(__x86_64__)
    if (have_f16c()) {
        mad_f16_avx(y, x, n, v);
        return;
    }
#endif
    for (int64_t i = 0; i < n; i++) {
        y[i] = ora_fp32_to_fp16(ora_fp16_to_fp32(y[i]) + ora_fp16_to_fp32(x[i]) * v);
    }
}

static float dot_q8_0(const uint8_t *a, const uint8_t *b, int64_t n) {
    float sumf = 0.0f;
    for (int64_t ib = 0; ib < n / QK8_0; ib++) {
        const uint8_t *x = a + ib * Q8_0_BYTES;
        const uint8_t *y = b + ib * Q8_0_BYTES;
        int            sumi = 0;
        for (int j = 0; j < QK8_0; j++) {
            sumi += (int) (int8_t) x[2 + j] * (int) (int8_t) y[2 + j];
        }
        uint16_t dx, dy;
        memcpy(&dx, x, 2);
        memcpy(&dy, y, 2);
        sumf += (float) sumi * (ora_fp16_to_fp32(dx) * ora_fp16_to_fp32(dy));
    }
    return sumf;
}

/* ------------------------------------------------------------------ */
/* the operator                                                        */
/* ------------------------------------------------------------------ */

static int check_contract(const ora_tensor *q, const ora_tensor *k, const ora_tensor *v, const ora_tensor *mask,
                          const ora_tensor *sinks) {
    if (q->type != ORA_F32) {
        return -1;
    }
    if (k->type != ORA_F16 && k->type != ORA_BF16 && k->type != ORA_Q8_0 && k->type != ORA_F32) {
        return -1;
    }
    if (v->type != ORA_F16 && v->type != ORA_BF16 && v->type != ORA_Q8_0 && v->type != ORA_F32) {
        return -1;
    }
    if (k->ne[0] != q->ne[0] || v->ne[1] != k->ne[1] || v->ne[2] != k->ne[2] || v->ne[3] != k->ne[3]) {
        return -2;
    }
    if (k->ne[2] <= 0 || q->ne[2] % k->ne[2] != 0 || k->ne[3] <= 0 || q->ne[3] % k->ne[3] != 0) {
        return -2;
    }
    if ((k->type == ORA_Q8_0 && k->ne[0] % QK8_0) || (v->type == ORA_Q8_0 && v->ne[0] % QK8_0)) {
        return -2;
    }
    if (mask) {
        if (mask->type != ORA_F16 || mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1]) {
            return -3;
        }
        if (mask->ne[2] <= 0 || q->ne[2] % mask->ne[2] != 0 || mask->ne[3] <= 0 || q->ne[3] % mask->ne[3] != 0) {
            return -3;
        }
    }
    if (sinks && (sinks->type != ORA_F32 || sinks->ne[0] < q->ne[2])) {
        return -4;
    }
    return 0;
}

int ora_flash_attn_ext(const ora_tensor *q, const ora_tensor *k, const ora_tensor *v, const ora_tensor *mask,
                       const ora_tensor *sinks, float *dst, const size_t dst_nb[4], float scale, float max_bias,
                       float softcap, int mode, int nthreads) {
    int rc = check_contract(q, k, v, mask, sinks);
    if (rc) {
        return rc;
    }
    const int64_t D = q->ne[0], n_q = q->ne[1], Hq = q->ne[2], B = q->ne[3];
    const int64_t n_kv = k->ne[1], Hkv = k->ne[2], Bk = k->ne[3];
    const int64_t Dv   = v->ne[0];
    const int64_t rk2 = Hq / Hkv, rk3 = B / Bk;
    const int64_t n_rows = B * Hq * n_q;

    float scale_eff = scale;
    if (softcap != 0.0f) {
        scale_eff /= softcap;
    }

#ifdef _OPENMP
    if (nthreads <= 0) {
        nthreads = omp_get_max_threads();
    }
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float    *qf   = (float *) malloc(sizeof(float) * (size_t) D);
        float    *kf   = (float *) malloc(sizeof(float) * (size_t) D);
        float    *vf   = (float *) malloc(sizeof(float) * (size_t) Dv);
        double   *accd = (double *) malloc(sizeof(double) * (size_t) Dv);
        float    *accf = (float *) malloc(sizeof(float) * (size_t) Dv);
        uint16_t *acch = (uint16_t *) malloc(sizeof(uint16_t) * (size_t) Dv);
        uint16_t *qh   = (uint16_t *) malloc(sizeof(uint16_t) * (size_t) D);
        uint8_t  *qq   = (uint8_t *) malloc((size_t) (D / QK8_0 + 1) * Q8_0_BYTES);

#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (int64_t r = 0; r < n_rows; r++) {
            /* row r -> (b, hq, iq) with iq fastest so rows sharing K stay together */
            const int64_t iq  = r % n_q;
            const int64_t hq  = (r / n_q) % Hq;
            const int64_t b   = r / (n_q * Hq);
            const int64_t ik2 = hq / rk2;
            const int64_t ik3 = b / rk3;

            const float    slope = alibi_slope(max_bias, hq, Hq);
            const uint8_t *mrow  = NULL;
            if (mask) {
                mrow = (const uint8_t *) mask->data + iq * mask->nb[1] + (hq % mask->ne[2]) * mask->nb[2] +
                       (b % mask->ne[3]) * mask->nb[3];
            }
            const uint8_t *qrow = (const uint8_t *) q->data + iq * q->nb[1] + hq * q->nb[2] + b * q->nb[3];
            row_to_f32(ORA_F32, qrow, q->nb[0], D, qf);

            const uint8_t *kbase = (const uint8_t *) k->data + ik2 * k->nb[2] + ik3 * k->nb[3];
            const uint8_t *vbase = (const uint8_t *) v->data + ik2 * v->nb[2] + ik3 * v->nb[3];

            float *out = (float *) ((uint8_t *) dst + hq * dst_nb[1] + iq * dst_nb[2] + b * dst_nb[3]);

            if (mode == ORA_MODE_F32) {
                double M = -INFINITY, S = 0.0;
                for (int64_t d = 0; d < Dv; d++) {
                    accd[d] = 0.0;
                }
                for (int64_t j = 0; j < n_kv; j++) {
                    double mv = 0.0;
                    if (mrow) {
                        uint16_t mh;
                        memcpy(&mh, mrow + j * 2, 2);
                        const float mf = ora_fp16_to_fp32(mh);
                        if (mf == -INFINITY) {
                            continue;
                        }
                        mv = (double) slope * (double) mf;
                    }
                    row_to_f32(k->type, kbase + j * k->nb[1], k->nb[0], D, kf);
                    double s = 0.0;
                    for (int64_t d = 0; d < D; d++) {
                        s += (double) qf[d] * (double) kf[d];
                    }
                    s *= (double) scale_eff;
                    if (softcap != 0.0f) {
                        s = (double) softcap * tanh(s);
                    }
                    s += mv;
                    if (s == -INFINITY) {
                        continue;
                    }
                    row_to_f32(v->type, vbase + j * v->nb[1], v->nb[0], Dv, vf);
                    double ms = 1.0, vs = 1.0;
                    if (s > M) {
                        const double Mold = M;
                        M                 = s;
                        ms                = exp(Mold - M);
                        for (int64_t d = 0; d < Dv; d++) {
                            accd[d] *= ms;
                        }
                    } else {
                        vs = exp(s - M);
                    }
                    for (int64_t d = 0; d < Dv; d++) {
                        accd[d] += vs * (double) vf[d];
                    }
                    S = S * ms + vs;
                }
                if (sinks) {
                    const double sk = (double) ((const float *) sinks->data)[hq];
                    double       ms = 1.0, vs = 1.0;
                    if (sk > M) {
                        ms = exp(M - sk);
                        for (int64_t d = 0; d < Dv; d++) {
                            accd[d] *= ms;
                        }
                    } else {
                        vs = exp(sk - M);
                    }
                    S = S * ms + vs;
                }
                const double S_inv = S == 0.0 ? 0.0 : 1.0 / S;
                for (int64_t d = 0; d < Dv; d++) {
                    float o = (float) (accd[d] * S_inv);
                    memcpy((uint8_t *) out + d * dst_nb[0], &o, 4);
                }
            } else {
                /* ggml-cpu arithmetic: Q converted to K's vec-dot type, f32 scores,
                 * F16 accumulator for F16 V. */
                if (k->type == ORA_F16) {
                    for (int64_t d = 0; d < D; d++) {
                        qh[d] = ora_fp32_to_fp16(qf[d]);
                    }
                } else if (k->type == ORA_BF16) {
                    for (int64_t d = 0; d < D; d++) {
                        qh[d] = ora_fp32_to_bf16(qf[d]);
                    }
                } else if (k->type == ORA_Q8_0) {
                    ora_quantize_q8_0(qf, qq, D);
                }
                const int v_f16 = v->type == ORA_F16;
                float     M = -INFINITY, S = 0.0f;
                for (int64_t d = 0; d < Dv; d++) {
                    accf[d] = 0.0f;
                    acch[d] = 0;
                }
                for (int64_t j = 0; j < n_kv; j++) {
                    float mv = 0.0f;
                    if (mrow) {
                        uint16_t mh;
                        memcpy(&mh, mrow + j * 2, 2);
                        mv = slope * ora_fp16_to_fp32(mh);
                        if (mv == -INFINITY) {
                            continue;
                        }
                    }
                    const uint8_t *krow = kbase + j * k->nb[1];
                    float          s;
                    if (k->type == ORA_F16 && k->nb[0] == 2) {
                        s = dot_f16(qh, (const uint16_t *) krow, D);
                    } else if (k->type == ORA_BF16) {
                        s = 0.0f;
                        for (int64_t d = 0; d < D; d++) {
                            uint16_t kh;
                            memcpy(&kh, krow + d * k->nb[0], 2);
                            s += ora_bf16_to_fp32(qh[d]) * ora_bf16_to_fp32(kh);
                        }
                    } else if (k->type == ORA_Q8_0) {
                        s = dot_q8_0(qq, krow, D);
                    } else {
                        row_to_f32(k->type, krow, k->nb[0], D, kf);
                        s = 0.0f;
                        for (int64_t d = 0; d < D; d++) {
                            s += (k->type == ORA_F16 ? ora_fp16_to_fp32(ora_fp32_to_fp16(qf[d])) : qf[d]) * kf[d];
                        }
                    }
                    s = s * scale_eff;
                    if (softcap != 0.0f) {
                        s = softcap * tanhf(s);
                    }
                    s += mv;
                    const float Mold = M;
                    float       ms = 1.0f, vs = 1.0f;
                    const uint8_t *vrow = vbase + j * v->nb[1];
                    if (v_f16 && v->nb[0] == 2) {
                        if (s > M) {
                            M  = s;
                            ms = expf(Mold - M);
                            scale_f16(acch, Dv, ms);
                        } else {
                            vs = expf(s - M);
                        }
                        mad_f16(acch, (const uint16_t *) vrow, Dv, vs);
                    } else {
                        if (s > M) {
                            M  = s;
                            ms = expf(Mold - M);
                            for (int64_t d = 0; d < Dv; d++) {
                                accf[d] *= ms;
                            }
                        } else {
                            vs = expf(s - M);
                        }
                        row_to_f32(v->type, vrow, v->nb[0], Dv, vf);
                        for (int64_t d = 0; d < Dv; d++) {
                            accf[d] += vf[d] * vs;
                        }
                    }
                    S = S * ms + vs;
                }
                if (v_f16 && v->nb[0] == 2) {
                    for (int64_t d = 0; d < Dv; d++) {
                        accf[d] = ora_fp16_to_fp32(acch[d]);
                    }
                }
                if (sinks) {
                    const float sk = ((const float *) sinks->data)[hq];
                    float       ms = 1.0f, vs = 1.0f;
                    if (sk > M) {
                        ms = expf(M - sk);
                        for (int64_t d = 0; d < Dv; d++) {
                            accf[d] *= ms;
                        }
                    } else {
                        vs = expf(sk - M);
                    }
                    S = S * ms + vs;
                }
                const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
                for (int64_t d = 0; d < Dv; d++) {
                    float o = accf[d] * S_inv;
                    memcpy((uint8_t *) out + d * dst_nb[0], &o, 4);
                }
            }
        }
        free(qf);
        free(kf);
        free(vf);
        free(accd);
        free(accf);
        free(acch);
        free(qh);
        free(qq);
    }
    return 0;
}

/* RMSNorm + RoPE NEOX of contiguous rows (see fa_oracle.h).  The frequency of
 * pair k is powf(theta_base, -2k/D) in f32, the same table the library
 * computes on the host, so both rotate by identical f32 angles. */
void ora_rope_norm(float *x, int64_t rows, int D, const float *weight, float eps, float theta_base,
                   const int32_t *pos) {
    float inv_freq[256];
    for (int k = 0; k < D / 2 && k < 256; ++k) {
        inv_freq[k] = powf(theta_base, -(float) (2 * k) / (float) D);
    }
    for (int64_t r = 0; r < rows; ++r) {
        float *y = x + r * D;
        if (weight) {
            double ss = 0.0;
            for (int d = 0; d < D; ++d) {
                ss += (double) y[d] * y[d];
            }
            const float sc = 1.0f / sqrtf((float) (ss / D) + eps);
            for (int d = 0; d < D; ++d) {
                y[d] = (y[d] * sc) * weight[d];
            }
        }
        if (theta_base > 0.0f) {
            for (int k = 0; k < D / 2; ++k) {
                const float a  = (float) pos[r] * inv_freq[k];
                const float c  = cosf(a), s = sinf(a);
                const float x0 = y[k], x1 = y[k + D / 2];
                y[k]           = x0 * c - x1 * s;
                y[k + D / 2]   = x0 * s + x1 * c;
            }
        }
    }
}

/* CFG logit combine + compaction (see fa_oracle.h), the host loop of
 * src/pipeline-lm.cpp:471-492: lc[i] = lu[i] + cfg_scale * (lc[i] - lu[i]) on
 * the EOS column and the audio-code range, then the compact copy.  Each
 * operation rounds to f32 on its own, as the reference's x86-64 build computes
 * it (its baseline ISA has no FMA, so nothing is contracted). */
void ora_cfg_logit_combine(const float *cond, const float *uncond, int64_t row_stride, int n, int eos_idx,
                           int code_offset, int code_count, float cfg_scale, float *compact) {
    const int cols = code_count + (eos_idx >= 0 ? 1 : 0);
    for (int a = 0; a < n; ++a) {
        const float *lc = cond + (int64_t) a * row_stride;
        const float *lu = uncond ? uncond + (int64_t) a * row_stride : NULL;
        float       *o  = compact + (int64_t) a * cols;
        for (int j = 0; j < cols; ++j) {
            const int64_t col = eos_idx >= 0 ? (j == 0 ? eos_idx : code_offset + j - 1) : code_offset + j;
            float         r   = lc[col];
            if (lu) {
                const float d = lc[col] - lu[col];
                const float m = cfg_scale * d;
                r             = lu[col] + m;
            }
            o[j] = r;
        }
    }
}
