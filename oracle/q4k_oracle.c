/* CPU oracle for the Qwen3-4B Q4_K/Q6_K decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker used by tests/, smoke() and the
 * cpu_baseline leg of bench.py; the product never loads it. Each function
 * restates the reference behaviour at the cited file:line. Built with
 * -ffp-contract=off and no fast-math so every float operation is a single
 * IEEE rounding in the order written.
 */
#include "q4k_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float orc_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int exponent = (h >> 10) & 0x1f;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else { /* subnormal half: value = mantissa * 2^-24, exact in float */
            float f = (float)mantissa * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((uint32_t)(exponent + 112) << 23) | (mantissa << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

uint16_t orc_float_to_half(float f) {
    /* Round to nearest even through double arithmetic on the exact value. */
    uint32_t bits;
    memcpy(&bits, &f, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    if (isnan(f)) return (uint16_t)(sign | 0x7e00u);
    double a = fabs((double)f);
    if (a >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (a < 6.103515625e-05) {                            /* half subnormal range: step 2^-24 */
        double q = nearbyint(a * 16777216.0);              /* default rounding mode: ties to even */
        return (uint16_t)(sign | (uint16_t)q);
    }
    int e;
    double m = frexp(a, &e); /* a = m * 2^e, m in [0.5, 1) */
    double q = nearbyint(m * 2048.0); /* 11 significant bits */
    if (q >= 2048.0) {
        q /= 2.0;
        e += 1;
    }
    /* value = q * 2^(e-11); half exponent field = e - 1 + 15 */
    const int field = e - 1 + 15;
    if (field >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | (uint16_t)(field << 10) | (uint16_t)((uint32_t)q - 1024u));
}

static float half_at(const uint8_t* p) { return orc_half_to_float((uint16_t)(p[0] | (p[1] << 8))); }

/* embedding.cu:14-31 (dequantize_q4k); bit fields as in matmul.cu:24-54. */
void orc_dequant_block_q4k(const uint8_t* block, float* out) {
    const float d = half_at(block);
    const float dmin = half_at(block + 2);
    const uint8_t* s = block + 4;
    for (int g = 0; g < 8; ++g) {
        int scale, minimum;
        if (g < 4) {
            scale = s[g] & 63;
            minimum = s[g + 4] & 63;
        } else {
            scale = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
            minimum = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
        }
        const float ds = d * (float)scale;
        const float dm = dmin * (float)minimum;
        for (int i = 0; i < 32; ++i) {
            const int code = (block[16 + (g / 2) * 32 + i] >> ((g % 2) * 4)) & 15;
            out[g * 32 + i] = ds * (float)code - dm;
        }
    }
}

/* embedding.cu:42-58 (dequantize_q6k); bit fields as in matmul.cu:61-84. */
void orc_dequant_block_q6k(const uint8_t* block, float* out) {
    const float d = half_at(block + 208);
    const int8_t* scales = (const int8_t*)(block + 192);
    for (int p = 0; p < 256; ++p) {
        const int half = p / 128, group = (p % 128) / 32, lane = p % 32;
        const int low = (block[half * 64 + (group % 2) * 32 + lane] >> (4 * (group / 2))) & 15;
        const int high = (block[128 + half * 32 + lane] >> (2 * group)) & 3;
        const int code = ((high << 4) | low) - 32;
        out[p] = (d * (float)scales[p / 16]) * (float)code;
    }
}

static void dequant_row(const uint8_t* row, int type, size_t width, float* out) {
    const size_t nb = width / 256;
    for (size_t b = 0; b < nb; ++b) {
        if (type == ORC_Q4_K)
            orc_dequant_block_q4k(row + b * 144, out + b * 256);
        else
            orc_dequant_block_q6k(row + b * 210, out + b * 256);
    }
}

/* embedding.cu:65-84 — rejects types other than Q4_K/Q6_K (embedding.cu:69-70). */
int orc_dequantize_rows(const void* packed, float* out, size_t rows, size_t width, size_t row_bytes, int type) {
    if (rows == 0) return 0;
    if (type != ORC_Q4_K && type != ORC_Q6_K) return -1;
    const uint8_t* base = (const uint8_t*)packed;
    for (size_t r = 0; r < rows; ++r) dequant_row(base + r * row_bytes, type, width, out + r * width);
    return 0;
}

/* matmul.cu:8-22 == MatmulReference.hpp:11-29. */
void orc_quantize_q8(const float* x, size_t count, int8_t* codes, float* scales) {
    for (size_t begin = 0; begin < count; begin += 32) {
        float maximum = 0.0f;
        for (size_t i = 0; i < 32; ++i) {
            const float a = fabsf(x[begin + i]);
            if (a > maximum) maximum = a;
        }
        scales[begin / 32] = maximum / 127.0f;
        for (size_t i = 0; i < 32; ++i)
            codes[begin + i] = maximum == 0.0f ? 0 : (int8_t)roundf((x[begin + i] / maximum) * 127.0f);
    }
}

/* MatmulReference.hpp:42-64 with the OpenMP row loop of the CPU baseline. */
int orc_matmul(const float* x, const void* weight, int type, size_t K, size_t N, size_t rows, double* y, int threads) {
    if (type != ORC_Q4_K && type != ORC_Q6_K) return -1;
    if (K == 0 || K % 256 != 0 || N == 0) return -2;
    if (rows == 0) return 0;
    const size_t count = rows * K;
    int8_t* codes = (int8_t*)malloc(count);
    float* scales = (float*)malloc(sizeof(float) * (count / 32));
    float* xq = (float*)malloc(sizeof(float) * count);
    if (!codes || !scales || !xq) {
        free(codes);
        free(scales);
        free(xq);
        return -3;
    }
    orc_quantize_q8(x, count, codes, scales);
    /* MatmulReference.hpp:25: round(x / max * 127) * scale, a float product. */
    for (size_t i = 0; i < count; ++i) xq[i] = (float)codes[i] * scales[i / 32];

    const size_t row_bytes = (K / 256) * (type == ORC_Q4_K ? 144 : 210);
    const uint8_t* w = (const uint8_t*)weight;
#ifdef _OPENMP
    const int nthreads = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float* decoded = (float*)malloc(sizeof(float) * K);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long long n = 0; n < (long long)N; ++n) {
            dequant_row(w + (size_t)n * row_bytes, type, K, decoded);
            for (size_t r = 0; r < rows; ++r) {
                double s = 0.0;
                const float* xr = xq + r * K;
                for (size_t i = 0; i < K; ++i) s += (double)xr[i] * (double)decoded[i];
                y[r * N + (size_t)n] = s;
            }
        }
        free(decoded);
    }
    (void)threads;
    free(codes);
    free(scales);
    free(xq);
    return 0;
}

/* rms_norm.cu:6-24, accumulated in double. */
void orc_rms_norm(const float* x, const float* gamma, float* y, size_t rows, size_t width, float eps) {
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * width;
        double ss = 0.0;
        for (size_t i = 0; i < width; ++i) ss += (double)xr[i] * (double)xr[i];
        const double inv = 1.0 / sqrt(ss / (double)width + (double)eps);
        for (size_t i = 0; i < width; ++i) y[r * width + i] = (float)((double)xr[i] * inv * (double)gamma[i]);
    }
}

/* rope.cu:7-24: angle = float(pos) * powf(base, -2j/d) in float, as the
 * reference forms it; the rotation itself in double. */
void orc_rope(float* x, size_t tokens, size_t heads, size_t head_dim, size_t position_offset, float base) {
    const size_t half = head_dim / 2;
    for (size_t t = 0; t < tokens; ++t) {
        const size_t position = position_offset + t;
        for (size_t h = 0; h < heads; ++h) {
            float* row = x + (t * heads + h) * head_dim;
            for (size_t j = 0; j < half; ++j) {
                const float frequency = powf(base, -2.0f * (float)j / (float)head_dim);
                const float angle = (float)position * frequency;
                const double c = cos((double)angle), s = sin((double)angle);
                const double a = row[j], b = row[j + half];
                row[j] = (float)(a * c - b * s);
                row[j + half] = (float)(a * s + b * c);
            }
        }
    }
}

/* attention.cu:23-91 semantics (AttentionReference.hpp:42-48): scale
 * 1/sqrt(d), causal mask, softmax, weighted sum of V; double throughout. */
int orc_attention(const float* q, const float* k, const float* v, float* out, size_t tokens, size_t heads,
                  size_t kv_heads, size_t head_dim, size_t offset) {
    if (tokens == 0) return 0;
    if (kv_heads == 0 || heads == 0 || heads % kv_heads != 0 || head_dim == 0) return -1;
    const size_t group = heads / kv_heads;
    const size_t kv_width = kv_heads * head_dim;
    const size_t keys_max = offset + tokens;
    const double scale = 1.0 / sqrt((double)head_dim);
#ifdef _OPENMP
#pragma omp parallel
#endif
    {
        double* scores = (double*)malloc(sizeof(double) * keys_max);
        double* acc = (double*)malloc(sizeof(double) * head_dim);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long long row = 0; row < (long long)(tokens * heads); ++row) {
            const size_t t = (size_t)row / heads, h = (size_t)row % heads;
            const size_t kvh = h / group;
            const size_t keys = offset + t + 1;
            const float* qr = q + (size_t)row * head_dim;
            double maximum = -INFINITY;
            for (size_t p = 0; p < keys; ++p) {
                const float* kr = k + p * kv_width + kvh * head_dim;
                double dot = 0.0;
                for (size_t d = 0; d < head_dim; ++d) dot += (double)qr[d] * (double)kr[d];
                scores[p] = dot * scale;
                if (scores[p] > maximum) maximum = scores[p];
            }
            double total = 0.0;
            for (size_t p = 0; p < keys; ++p) {
                scores[p] = exp(scores[p] - maximum);
                total += scores[p];
            }
            for (size_t d = 0; d < head_dim; ++d) acc[d] = 0.0;
            for (size_t p = 0; p < keys; ++p) {
                const float* vr = v + p * kv_width + kvh * head_dim;
                for (size_t d = 0; d < head_dim; ++d) acc[d] += scores[p] * (double)vr[d];
            }
            for (size_t d = 0; d < head_dim; ++d) out[(size_t)row * head_dim + d] = (float)(acc[d] / total);
        }
        free(scores);
        free(acc);
    }
    return 0;
}

/* silu_multiply.cu:9-10. */
void orc_silu_multiply(const float* gate, const float* up, float* out, size_t count) {
    for (size_t i = 0; i < count; ++i) {
        const double g = gate[i];
        out[i] = (float)(g / (1.0 + exp(-g)) * (double)up[i]);
    }
}

/* residual_add.cu:6-9. */
void orc_residual_add(float* state, const float* branch, size_t count) {
    for (size_t i = 0; i < count; ++i) state[i] += branch[i];
}

/* argmax.cu:19-23, :37-43, :89-97. */
uint32_t orc_argmax(const float* logits, size_t count) {
    size_t best = (size_t)-1;
    float score = -INFINITY;
    for (size_t i = 0; i < count; ++i) {
        if (logits[i] > score) {
            score = logits[i];
            best = i;
        }
    }
    return best == (size_t)-1 ? UINT32_MAX : (uint32_t)best;
}

static int matmul_f(const float* x, const void* w, int type, size_t K, size_t N, size_t rows, float* y, double* tmp,
                    int threads) {
    const int rc = orc_matmul(x, w, type, K, N, rows, tmp, threads);
    if (rc) return rc;
    for (size_t i = 0; i < rows * N; ++i) y[i] = (float)tmp[i];
    return 0;
}

/* Buffers of one block over T rows (Engine.cpp:57-67's per-step buffers). */
typedef struct {
    float *nrm, *q, *qn, *kk, *att, *branch, *gate, *up, *act;
    double* tmp;
} orc_work;

static void work_free(orc_work* w) {
    free(w->nrm);
    free(w->q);
    free(w->qn);
    free(w->kk);
    free(w->att);
    free(w->branch);
    free(w->gate);
    free(w->up);
    free(w->act);
    free(w->tmp);
}

/* tmp_extra: doubles the caller needs from tmp besides the layer's products. */
static int work_alloc(const orc_model* m, size_t T, size_t tmp_extra, orc_work* w) {
    const size_t W = (size_t)m->hidden, QW = (size_t)m->heads * m->head_dim, KW = (size_t)m->kv_heads * m->head_dim;
    const size_t F = (size_t)m->ffn;
    const size_t big = (F > QW ? F : QW) > W ? (F > QW ? F : QW) : W;
    w->nrm = (float*)malloc(sizeof(float) * T * W);
    w->q = (float*)malloc(sizeof(float) * T * QW);
    w->qn = (float*)malloc(sizeof(float) * T * QW);
    w->kk = (float*)malloc(sizeof(float) * T * KW);
    w->att = (float*)malloc(sizeof(float) * T * QW);
    w->branch = (float*)malloc(sizeof(float) * T * W);
    w->gate = (float*)malloc(sizeof(float) * T * F);
    w->up = (float*)malloc(sizeof(float) * T * F);
    w->act = (float*)malloc(sizeof(float) * T * F);
    w->tmp = (double*)malloc(sizeof(double) * (T * big > tmp_extra ? T * big : tmp_extra));
    if (!w->nrm || !w->q || !w->qn || !w->kk || !w->att || !w->branch || !w->gate || !w->up || !w->act || !w->tmp) {
        work_free(w);
        return -3;
    }
    return 0;
}

/* Engine.cpp:71-103: one block on rows x [T][hidden] (updated in place) at
 * positions pos .. pos+T-1; kc/vc this layer's caches [capacity][kv_width]. */
static int layer_body(const orc_model* m, int layer, float* x, float* kc, float* vc, size_t T, size_t pos,
                      int kv_round_f16, orc_work* w, int threads) {
    const size_t W = (size_t)m->hidden, H = (size_t)m->heads, KVH = (size_t)m->kv_heads, D = (size_t)m->head_dim;
    const size_t F = (size_t)m->ffn, QW = H * D, KW = KVH * D;
    const void* const* tp = m->tensors + ORC_SLOTS * layer;
    const int* ty = m->types + ORC_SLOTS * layer;
    float* new_k = kc + pos * KW;
    float* new_v = vc + pos * KW;
    int rc;
    orc_rms_norm(x, (const float*)tp[ORC_ATTN_NORM], w->nrm, T, W, m->eps);
    if ((rc = matmul_f(w->nrm, tp[ORC_Q], ty[ORC_Q], W, QW, T, w->q, w->tmp, threads))) return rc;
    if ((rc = matmul_f(w->nrm, tp[ORC_K], ty[ORC_K], W, KW, T, w->kk, w->tmp, threads))) return rc;
    if ((rc = matmul_f(w->nrm, tp[ORC_V], ty[ORC_V], W, KW, T, new_v, w->tmp, threads))) return rc;
    orc_rms_norm(w->q, (const float*)tp[ORC_Q_NORM], w->qn, T * H, D, m->eps);
    orc_rms_norm(w->kk, (const float*)tp[ORC_K_NORM], new_k, T * KVH, D, m->eps);
    orc_rope(w->qn, T, H, D, pos, m->rope_base);
    orc_rope(new_k, T, KVH, D, pos, m->rope_base);
    if (kv_round_f16) {
        for (size_t i = 0; i < T * KW; ++i) {
            new_k[i] = orc_half_to_float(orc_float_to_half(new_k[i]));
            new_v[i] = orc_half_to_float(orc_float_to_half(new_v[i]));
        }
    }
    orc_attention(w->qn, kc, vc, w->att, T, H, KVH, D, pos);
    if ((rc = matmul_f(w->att, tp[ORC_O], ty[ORC_O], QW, W, T, w->branch, w->tmp, threads))) return rc;
    orc_residual_add(x, w->branch, T * W);
    orc_rms_norm(x, (const float*)tp[ORC_FFN_NORM], w->nrm, T, W, m->eps);
    if ((rc = matmul_f(w->nrm, tp[ORC_GATE], ty[ORC_GATE], W, F, T, w->gate, w->tmp, threads))) return rc;
    if ((rc = matmul_f(w->nrm, tp[ORC_UP], ty[ORC_UP], W, F, T, w->up, w->tmp, threads))) return rc;
    orc_silu_multiply(w->gate, w->up, w->act, T * F);
    if ((rc = matmul_f(w->act, tp[ORC_DOWN], ty[ORC_DOWN], F, W, T, w->branch, w->tmp, threads))) return rc;
    orc_residual_add(x, w->branch, T * W);
    return 0;
}

int orc_layer(const orc_model* m, int layer, float* x, float* k_cache, float* v_cache, size_t capacity, size_t tokens,
              size_t pos, int kv_round_f16, int threads) {
    if (tokens == 0) return -1;
    if (layer < 0 || layer >= m->layers) return -5;
    if (pos + tokens > capacity) return -2;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    orc_work w;
    int rc = work_alloc(m, tokens, 0, &w);
    if (rc) return rc;
    rc = layer_body(m, layer, x, k_cache, v_cache, tokens, pos, kv_round_f16, &w, threads);
    work_free(&w);
    return rc;
}

/* Engine.cpp:37-114 (Engine::inference), one call over `tokens` new tokens. */
int orc_forward(const orc_model* m, float* k_cache, float* v_cache, size_t capacity, const uint32_t* token_ids,
                size_t tokens, size_t pos, int kv_round_f16, float* logits, float* hidden, uint32_t* next_token,
                int threads) {
    if (tokens == 0) return -1;
    if (pos + tokens > capacity) return -2; /* ChatSession.hpp:40-41 */
#ifdef _OPENMP
    /* the attention's parallel region takes the same thread count */
    if (threads > 0) omp_set_num_threads(threads);
#endif
    const size_t W = (size_t)m->hidden, V = (size_t)m->vocab, KW = (size_t)m->kv_heads * m->head_dim;
    const size_t T = tokens;
    orc_work w;
    if (work_alloc(m, T, V, &w)) return -3;
    float* x = (float*)malloc(sizeof(float) * T * W);
    float* lg = (float*)malloc(sizeof(float) * V);
    int rc = 0;
    if (!x || !lg) {
        rc = -3;
        goto done;
    }

    /* EmbedLookup.cpp:49-78: dequantised token_embd rows. */
    {
        const int et = m->types[ORC_SLOTS * m->layers + 1];
        const uint8_t* table = (const uint8_t*)m->tensors[ORC_SLOTS * m->layers + 1];
        const size_t row_bytes = (W / 256) * (et == ORC_Q4_K ? 144 : 210);
        for (size_t t = 0; t < T; ++t) {
            if (token_ids[t] >= V) {
                rc = -4;
                goto done;
            }
            dequant_row(table + (size_t)token_ids[t] * row_bytes, et, W, x + t * W);
        }
    }
    if (hidden) memcpy(hidden, x + (T - 1) * W, sizeof(float) * W);

    for (int layer = 0; layer < m->layers; ++layer) {
        if ((rc = layer_body(m, layer, x, k_cache + (size_t)layer * capacity * KW, v_cache + (size_t)layer * capacity * KW,
                             T, pos, kv_round_f16, &w, threads)))
            goto done;
        if (hidden) memcpy(hidden + (size_t)(layer + 1) * W, x + (T - 1) * W, sizeof(float) * W);
    }

    /* Engine.cpp:105-111: last token only, tied output head, greedy argmax. */
    orc_rms_norm(x + (T - 1) * W, (const float*)m->tensors[ORC_SLOTS * m->layers + 0], w.nrm, 1, W, m->eps);
    if ((rc = matmul_f(w.nrm, m->tensors[ORC_SLOTS * m->layers + 1], m->types[ORC_SLOTS * m->layers + 1], W, V, 1, lg,
                       w.tmp, threads)))
        goto done;
    if (logits) memcpy(logits, lg, sizeof(float) * V);
    if (next_token) *next_token = orc_argmax(lg, V);

done:
    free(x);
    free(lg);
    work_free(&w);
    return rc;
}
