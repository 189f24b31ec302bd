/*
 * bitcache CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference bitcache kernels (anishesg/bitcache,
 * src/*.cu), used as the checker for the B200 kernels and as the timed CPU
 * baseline.  Nothing in the product path links, loads or calls this file; only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may.
 *
 * Parity of this restatement is pinned against fixtures produced by running
 * the reference's own CUDA kernels (compiled from their sources into
 * oracle/_ref/) on seeded inputs; see tests/golden/make_golden.py.
 *
 * Each function names the reference file:line it follows.  Data is held in a
 * structure-of-arrays form (one array per field) instead of the reference's
 * BinaryVec / ResidualVec structs; the field values are identical.
 *
 * Known divergence: the reference is built with --use_fast_math, so the GPU
 * computes `7.0f / absmax` (residual.cu:54, online_encode.cu:106) with an
 * approximate division.  This file uses IEEE division.  An INT4 code can then
 * differ by one where residual * (7/absmax) lies within a few ulps of a
 * rounding tie; the tests count and bound such cases.  Power-of-two divisions
 * (the mean |x| scale for head_dim a power of two) are exact in both.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_BLOCK 128 /* blockDim.x of every reference encode kernel */

/* ------------------------------------------------------------------ */
/* fp16 conversions (IEEE binary16, round-to-nearest-even)              */
/* ------------------------------------------------------------------ */

float orc_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: value = man * 2^-24 */
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) { /* inf or nan */
        if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
        return (uint16_t)(sign | 0x7C00u);
    }
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    if (ax < 0x38800000u) {                                   /* fp16 subnormal / zero */
        if (ax < 0x33000000u) return (uint16_t)sign;         /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e; /* value = m * 2^(e-150); target unit 2^-24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* __float2int_rn: round to nearest, ties to even (default FP environment). */
static int orc_f2i_rn(float x) {
    if (x != x) return 0;
    float r = nearbyintf(x);
    if (r >= 2147483647.0f) return 2147483647;
    if (r <= -2147483648.0f) return (int)0x80000000;
    return (int)r;
}

/* ------------------------------------------------------------------ */
/* Encoders                                                            */
/* ------------------------------------------------------------------ */

/*
 * Mean |x| with the reference block reduction: thread t (of 128) sums
 * x_t, x_{t+128}, ... sequentially, then a stride-halving tree
 * p[t] += p[t+stride] for stride = 64, 32, ..., 1
 * (binary_encode.cu:32-50; same order in online_encode.cu:56-72 and
 * adaptive_precision.cu:46-58).
 */
static float orc_tree_abs_sum(const float* x, int d) {
    float p[ORC_BLOCK];
    for (int t = 0; t < ORC_BLOCK; ++t) {
        float s = 0.0f;
        for (int i = t; i < d; i += ORC_BLOCK) s += fabsf(x[i]);
        p[t] = s;
    }
    for (int stride = ORC_BLOCK / 2; stride > 0; stride >>= 1)
        for (int t = 0; t < stride; ++t) p[t] += p[t + stride];
    return p[0];
}

/* Sign packing: bit i%32 of word i/32 is set iff x_i >= 0.0f
 * (binary_encode.cu:36-39, binary_encode.cuh:36-38). NaN -> 0, -0.0 -> 1. */
static void orc_pack_signs(const float* x, int d, uint32_t* words) {
    for (int w = 0; w < d / 32; ++w) {
        uint32_t v = 0;
        for (int b = 0; b < 32; ++b)
            if (x[w * 32 + b] >= 0.0f) v |= 1u << b;
        words[w] = v;
    }
}

/* binary_encode_kernel, binary_encode.cu:8-60. */
void orc_binary_encode(const uint16_t* src, int64_t n, int d, uint32_t* words, uint16_t* scale) {
    const int nw = d / 32;
#pragma omp parallel for schedule(static)
    for (int64_t v = 0; v < n; ++v) {
        float x[256];
        for (int i = 0; i < d; ++i) x[i] = orc_h2f(src[v * d + i]);
        orc_pack_signs(x, d, words + v * nw);
        float mean_abs = orc_tree_abs_sum(x, d) / (float)d;
        scale[v] = orc_f2h(mean_abs);
    }
}

/*
 * Residual quantisation shared by residual.cu:30-77 and online_encode.cu:85-119.
 * s is the binary scale the residual is taken against: the fp16-rounded stored
 * scale in residual.cu:28, the unrounded fp32 mean in online_encode.cu:74.
 */
static void orc_quantise_residual(const float* x, const uint32_t* words, float s, int d, uint8_t* nib,
                                  uint16_t* rscale, float* codes_pre /* optional: r*inv per element */) {
    float r[256];
    float local[ORC_BLOCK];
    for (int t = 0; t < ORC_BLOCK; ++t) local[t] = 0.0f;
    for (int i = 0; i < d; ++i) {
        int bit = (words[i / 32] >> (i % 32)) & 1u;
        float rec = bit ? s : -s;
        r[i] = x[i] - rec;
        local[i % ORC_BLOCK] = fmaxf(local[i % ORC_BLOCK], fabsf(r[i]));
    }
    for (int stride = ORC_BLOCK / 2; stride > 0; stride >>= 1)
        for (int t = 0; t < stride; ++t) local[t] = fmaxf(local[t], local[t + stride]);
    float absmax = local[0];
    float inv = (absmax > 0.0f) ? (7.0f / absmax) : 0.0f;
    *rscale = orc_f2h(absmax);
    for (int i = 0; i < d / 2; ++i) {
        float a = r[2 * i] * inv, b = r[2 * i + 1] * inv;
        if (codes_pre) {
            codes_pre[2 * i] = a;
            codes_pre[2 * i + 1] = b;
        }
        int q0 = orc_f2i_rn(a), q1 = orc_f2i_rn(b);
        q0 = q0 < -7 ? -7 : (q0 > 7 ? 7 : q0);
        q1 = q1 < -7 ? -7 : (q1 > 7 ? 7 : q1);
        nib[i] = (uint8_t)((q0 & 0x0F) | ((q1 & 0x0F) << 4));
    }
}

/* residual_encode_kernel, residual.cu:9-78 (binary scale read back as fp16, :28). */
void orc_residual_encode(const uint16_t* src, const uint32_t* words, const uint16_t* bscale, int64_t n, int d,
                         uint8_t* nib, uint16_t* rscale, float* codes_pre) {
    const int nw = d / 32;
#pragma omp parallel for schedule(static)
    for (int64_t v = 0; v < n; ++v) {
        float x[256];
        for (int i = 0; i < d; ++i) x[i] = orc_h2f(src[v * d + i]);
        orc_quantise_residual(x, words + v * nw, orc_h2f(bscale[v]), d, nib + v * (d / 2), rscale + v,
                              codes_pre ? codes_pre + v * d : NULL);
    }
}

/* online_encode_token_kernel, online_encode.cu:17-120: binary + residual in one
 * pass, the residual taken against the fp32 (unrounded) mean (:74, :88). */
void orc_online_encode(const uint16_t* src, int64_t n, int d, uint32_t* words, uint16_t* bscale, uint8_t* nib,
                       uint16_t* rscale, float* codes_pre) {
    const int nw = d / 32;
#pragma omp parallel for schedule(static)
    for (int64_t v = 0; v < n; ++v) {
        float x[256];
        for (int i = 0; i < d; ++i) x[i] = orc_h2f(src[v * d + i]);
        orc_pack_signs(x, d, words + v * nw);
        float s = orc_tree_abs_sum(x, d) / (float)d;
        bscale[v] = orc_f2h(s);
        orc_quantise_residual(x, words + v * nw, s, d, nib + v * (d / 2), rscale + v,
                              codes_pre ? codes_pre + v * d : NULL);
    }
}

/* ------------------------------------------------------------------ */
/* Scoring and attention                                               */
/* ------------------------------------------------------------------ */

static inline int orc_popc(uint32_t x) { return __builtin_popcount(x); }

/* nibble_lo / nibble_hi, residual.cuh:42-52; dequant_nibble :37-39. */
static inline int orc_nib(uint8_t byte, int hi) {
    int raw = hi ? ((byte >> 4) & 0x0F) : (byte & 0x0F);
    return raw >= 8 ? raw - 16 : raw;
}

/*
 * XNOR popcount of a query against n binary keys: sum_w popc(~(q_w ^ k_w))
 * (xnor_dot.cuh:20-27).  q packed with pack_sign_bits (xnor_dot.cuh:36-52).
 */
void orc_xnor_popcount(const uint16_t* q, const uint32_t* kwords, int64_t n, int d, int32_t* out) {
    float qf[256];
    uint32_t qs[8];
    for (int i = 0; i < d; ++i) qf[i] = orc_h2f(q[i]);
    orc_pack_signs(qf, d, qs);
    const int nw = d / 32;
    for (int64_t s = 0; s < n; ++s) {
        int p = 0;
        for (int w = 0; w < nw; ++w) p += orc_popc(~(qs[w] ^ kwords[s * nw + w]));
        out[s] = p;
    }
}

typedef struct {
    const uint32_t* words; /* [slots][kv_stride][d/32] */
    const uint16_t* bscale; /* [slots][kv_stride] */
    const uint8_t* nib;     /* [slots][kv_stride][d/2] (may be NULL for binary-only) */
    const uint16_t* rscale; /* [slots][kv_stride] */
} orc_planes;

/* Score of one key, compensated_attention.cu:79-80 (xnor_dot + residual_dot) or
 * binary_attention.cu:56 (xnor_dot only), times 1/sqrt(d). */
static inline float orc_score(const float* qf, const uint32_t* qs, float scale_q, const orc_planes* K, int64_t idx,
                              int d, int compensated, float inv_sqrt_d) {
    const int nw = d / 32;
    int pop = 0;
    for (int w = 0; w < nw; ++w) pop += orc_popc(~(qs[w] ^ K->words[idx * nw + w]));
    float xd = scale_q * orc_h2f(K->bscale[idx]) * (float)(2 * pop - d);
    if (!compensated) return xd * inv_sqrt_d;
    /* residual_dot, compensated_attention.cu:23-37 */
    float rs = orc_h2f(K->rscale[idx]);
    const uint8_t* nb = K->nib + idx * (d / 2);
    float dot = 0.0f;
    for (int i = 0; i < d / 2; ++i) {
        float r0 = ((float)orc_nib(nb[i], 0) / 7.0f) * rs;
        float r1 = ((float)orc_nib(nb[i], 1) / 7.0f) * rs;
        dot += qf[2 * i] * r0 + qf[2 * i + 1] * r1;
    }
    return (xd + dot) * inv_sqrt_d;
}

/*
 * Decode attention for n_q query heads over one KV layout.
 * compensated != 0: compensated_attention_kernel, compensated_attention.cu:42-109.
 * compensated == 0: binary_attention_kernel, binary_attention.cu:8-82.
 * Query head h reads KV slot (h / group); group = 1 is the reference's MHA
 * indexing.  Slot j's keys are positions [0, seq_len) at stride kv_stride.
 */
void orc_attention(const uint16_t* q, const orc_planes* K, const orc_planes* V, int64_t n_q, int group, int seq_len,
                   int64_t kv_stride, int d, int compensated, uint16_t* out, int nthreads) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t h = 0; h < n_q; ++h) {
        float qf[256], acc[256];
        uint32_t qs[8];
        for (int i = 0; i < d; ++i) qf[i] = orc_h2f(q[h * d + i]);
        orc_pack_signs(qf, d, qs);
        float scale_q = 0.0f;
        for (int i = 0; i < d; ++i) scale_q += fabsf(qf[i]);
        scale_q /= (float)d;
        const int64_t base = (h / group) * kv_stride;
        float running_max = -1e38f;
        for (int s = 0; s < seq_len; ++s) {
            float sc = orc_score(qf, qs, scale_q, K, base + s, d, compensated, inv_sqrt_d);
            if (sc > running_max) running_max = sc;
        }
        float running_sum = 0.0f;
        for (int i = 0; i < d; ++i) acc[i] = 0.0f;
        const int nw = d / 32;
        for (int s = 0; s < seq_len; ++s) {
            const int64_t idx = base + s;
            float sc = orc_score(qf, qs, scale_q, K, idx, d, compensated, inv_sqrt_d);
            float w = expf(sc - running_max);
            running_sum += w;
            float sv = orc_h2f(V->bscale[idx]);
            const uint32_t* vw = V->words + idx * nw;
            for (int i = 0; i < d; ++i) {
                int bit = (vw[i / 32] >> (i % 32)) & 1u;
                acc[i] += w * (bit ? sv : -sv);
            }
            if (compensated) { /* dequant_residual_add, compensated_attention.cu:6-20 */
                float rs = orc_h2f(V->rscale[idx]);
                const uint8_t* nb = V->nib + idx * (d / 2);
                for (int i = 0; i < d / 2; ++i) {
                    float r0 = ((float)orc_nib(nb[i], 0) / 7.0f) * rs;
                    float r1 = ((float)orc_nib(nb[i], 1) / 7.0f) * rs;
                    acc[2 * i] += w * r0;
                    acc[2 * i + 1] += w * r1;
                }
            }
        }
        float inv_sum = (running_sum > 0.0f) ? (1.0f / running_sum) : 0.0f;
        for (int i = 0; i < d; ++i) out[h * d + i] = orc_f2h(acc[i] * inv_sum);
    }
}

/* Exact attention from fp16 K/V, reference_attention.cu:6-69. K, V: [n_q][seq_len][d]. */
void orc_reference_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t n_q, int seq_len,
                             int d, uint16_t* out) {
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t h = 0; h < n_q; ++h) {
        float qf[256], acc[256];
        for (int i = 0; i < d; ++i) qf[i] = orc_h2f(q[h * d + i]);
        const uint16_t* kb = k + h * (int64_t)seq_len * d;
        const uint16_t* vb = v + h * (int64_t)seq_len * d;
        float mx = -1e38f;
        for (int s = 0; s < seq_len; ++s) {
            float dot = 0.0f;
            for (int i = 0; i < d; ++i) dot += qf[i] * orc_h2f(kb[(int64_t)s * d + i]);
            float sc = dot * inv_sqrt_d;
            if (sc > mx) mx = sc;
        }
        for (int i = 0; i < d; ++i) acc[i] = 0.0f;
        float sum = 0.0f;
        for (int s = 0; s < seq_len; ++s) {
            float dot = 0.0f;
            for (int i = 0; i < d; ++i) dot += qf[i] * orc_h2f(kb[(int64_t)s * d + i]);
            float w = expf(dot * inv_sqrt_d - mx);
            sum += w;
            for (int i = 0; i < d; ++i) acc[i] += w * orc_h2f(vb[(int64_t)s * d + i]);
        }
        float inv = (sum > 0.0f) ? (1.0f / sum) : 0.0f;
        for (int i = 0; i < d; ++i) out[h * d + i] = orc_f2h(acc[i] * inv);
    }
}

/*
 * Per-head entropy of the softmax over binary scores (no 1/sqrt(d)),
 * compute_head_entropy_kernel, adaptive_precision.cu:13-130: Q scale by the
 * 128-thread tree, per-thread strided partials over s, stride-halving trees.
 */
void orc_head_entropy(const uint16_t* q, const uint32_t* kwords, const uint16_t* kscale, int64_t n_q, int seq_len,
                      int64_t kv_stride, int d, float* out) {
    const int nw = d / 32;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t h = 0; h < n_q; ++h) {
        float qf[256];
        uint32_t qs[8];
        for (int i = 0; i < d; ++i) qf[i] = orc_h2f(q[h * d + i]);
        orc_pack_signs(qf, d, qs);
        float scale_q = orc_tree_abs_sum(qf, d) / (float)d;
        const int64_t base = h * kv_stride;
        float p[ORC_BLOCK], p2[ORC_BLOCK];
        for (int t = 0; t < ORC_BLOCK; ++t) {
            float m = -1e30f;
            for (int s = t; s < seq_len; s += ORC_BLOCK) {
                int pop = 0;
                for (int w = 0; w < nw; ++w) pop += orc_popc(~(qs[w] ^ kwords[(base + s) * nw + w]));
                float sc = scale_q * orc_h2f(kscale[base + s]) * (float)(2 * pop - d);
                m = fmaxf(m, sc);
            }
            p[t] = m;
        }
        for (int stride = ORC_BLOCK / 2; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; ++t) p[t] = fmaxf(p[t], p[t + stride]);
        const float gmax = p[0];
        for (int t = 0; t < ORC_BLOCK; ++t) {
            float es = 0.0f, ws = 0.0f;
            for (int s = t; s < seq_len; s += ORC_BLOCK) {
                int pop = 0;
                for (int w = 0; w < nw; ++w) pop += orc_popc(~(qs[w] ^ kwords[(base + s) * nw + w]));
                float sc = scale_q * orc_h2f(kscale[base + s]) * (float)(2 * pop - d);
                float e = expf(sc - gmax);
                es += e;
                ws += e * sc;
            }
            p[t] = es;
            p2[t] = ws;
        }
        for (int stride = ORC_BLOCK / 2; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; ++t) {
                p[t] += p[t + stride];
                p2[t] += p2[t + stride];
            }
        float log_z = logf(p[0]) + gmax;
        out[h] = log_z - p2[0] / fmaxf(p[0], 1e-12f);
    }
}

/* adaptive_select_kernel, adaptive_precision.cu:133-144: entropy >= thr -> 0 (BINARY) else 1. */
void orc_adaptive_select(const float* entropy, int64_t n, float thr, uint8_t* modes) {
    for (int64_t i = 0; i < n; ++i) modes[i] = (entropy[i] >= thr) ? 0 : 1;
}

/* ------------------------------------------------------------------ */
/* Extensions with no reference kernel                                  */
/* ------------------------------------------------------------------ */

/*
 * Per-vector adaptive precision: within each slot keep the residual of the
 * n_keep vectors with the largest residual energy key
 *     key = fp32(rs * rs) * (float)sum_i n_i^2      (rs = fp16 residual scale)
 * ties broken toward the lower position.  keep[s] = 1 for kept vectors.
 */
void orc_select_residual_topk(const uint8_t* nib, const uint16_t* rscale, int64_t n_slots, int seq_len,
                              int64_t kv_stride, int d, int n_keep, uint8_t* keep /* [slots][kv_stride] */) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t j = 0; j < n_slots; ++j) {
        float* key = (float*)malloc(sizeof(float) * (seq_len > 0 ? seq_len : 1));
        for (int s = 0; s < seq_len; ++s) {
            const int64_t idx = j * kv_stride + s;
            int ss = 0;
            for (int i = 0; i < d / 2; ++i) {
                int a = orc_nib(nib[idx * (d / 2) + i], 0), b = orc_nib(nib[idx * (d / 2) + i], 1);
                ss += a * a + b * b;
            }
            float rs = orc_h2f(rscale[idx]);
            float rr = rs * rs;
            key[s] = rr * (float)ss;
        }
        for (int s = 0; s < seq_len; ++s) {
            /* rank = number of vectors strictly ahead of s in (key desc, index asc) order */
            int rank = 0;
            for (int t = 0; t < seq_len && rank < n_keep; ++t)
                if (key[t] > key[s] || (key[t] == key[s] && t < s)) ++rank;
            keep[j * kv_stride + s] = (uint8_t)(rank < n_keep);
        }
        free(key);
    }
}

/*
 * Log-sum-exp merge of split partials (split-K inside one GPU and the
 * cross-GPU sequence split).  Partial p of head h: m = max score (natural log
 * domain), l = sum exp(score - m), o[d] = sum exp(score - m) * v (unnormalised).
 * Layout: part[(p * n_heads + h) * (d + 2) + {0: m, 1: l, 2..: o}].
 */
void orc_lse_merge(const float* part, int n_parts, int64_t n_heads, int d, float* out /* [n_heads][d] */) {
    for (int64_t h = 0; h < n_heads; ++h) {
        double M = -INFINITY;
        for (int p = 0; p < n_parts; ++p) {
            const float* r = part + ((int64_t)p * n_heads + h) * (d + 2);
            if (r[1] > 0.0f && r[0] > M) M = r[0];
        }
        double L = 0.0;
        for (int i = 0; i < d; ++i) out[h * d + i] = 0.0f;
        double acc[256] = {0};
        for (int p = 0; p < n_parts; ++p) {
            const float* r = part + ((int64_t)p * n_heads + h) * (d + 2);
            if (!(r[1] > 0.0f)) continue;
            double f = exp((double)r[0] - M);
            L += f * r[1];
            for (int i = 0; i < d; ++i) acc[i] += f * r[2 + i];
        }
        for (int i = 0; i < d; ++i) out[h * d + i] = (L > 0.0) ? (float)(acc[i] / L) : 0.0f;
    }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
