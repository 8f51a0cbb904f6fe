/*
 * CPU oracle for the XTR-base T5 encoder hot path.  TEST INFRASTRUCTURE ONLY:
 * this file is the checker that the CUDA path is compared against (tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg).
 * Nothing in the product path links or calls it.
 *
 * It restates, in plain C (f32, OpenMP), the default `t5-quantized` CPU path of
 * dropbox/witchcraft, which dequantises every Q4_K weight to f32 at load time
 * (src/quantized_t5.rs:39-49) and then runs an f32 graph:
 *   - Q4_K super-block dequant: the GGML Q4_K layout read by candle's
 *     k_quants::BlockQ4K (third-party, candle rev 5bd5618, Cargo.toml:24-26;
 *     invoked at src/quantized_t5.rs:44).  The same arithmetic is published in
 *     gguf-py 0.19.0 (gguf/quants.py, Q4_K.dequantize_blocks), which pins it.
 *   - T5LayerNorm (RMSNorm, no mean, no bias):  src/quantized_t5.rs:162-173
 *   - gated-GELU FF (gelu_tanh(x W0^T) * (x W1^T)) W^T: src/quantized_t5.rs:231-252
 *   - self-attention without 1/sqrt(d) scaling, T5 bidirectional relative
 *     position buckets computed once (block 0) and reused:  :374-503, :640-668
 *   - residual adds (fast_add): src/quantized_t5.rs:291, :533
 *   - final RMSNorm + 768->128 projection:  :669, :690, :700
 *
 * Each sequence b of a batch is encoded exactly as the reference encodes a
 * batch-1 input of its first lengths[b] tokens (the reference never pads).
 * Output rows at positions >= lengths[b] are written as zeros.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* ------------------------------------------------------------------ */
/* Q4_K                                                                */
/* ------------------------------------------------------------------ */

/* IEEE half -> float, exact. */
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal half: normalise */
            int e = -1;
            do { e++; mant <<= 1; } while ((mant & 0x400u) == 0);
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* 6-bit scale/min unpack of sub-block j (0..7) from the 12 packed bytes
 * (GGML Q4_K "get_scale_min_k4"; gguf/quants.py Q4_K.get_scale_min). */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Dequantise nblocks consecutive 144-byte Q4_K super-blocks to 256*nblocks
 * floats.  value = (d*sc_j)*q - (dmin*m_j), each product rounded to f32, then
 * the difference rounded (gguf/quants.py Q4_K.dequantize_blocks). */
void oracle_q4k_dequant(const uint8_t *src, int64_t nblocks, float *dst) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; b++) {
        const uint8_t *blk = src + b * 144;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        const float d = half_to_float(dh);
        const float dmin = half_to_float(mh);
        const uint8_t *scales = blk + 4;
        const uint8_t *qs = blk + 16;
        float *out = dst + b * 256;
        for (int c = 0; c < 4; c++) { /* 32-byte chunk c: sub-blocks 2c (low), 2c+1 (high) */
            int sc0, m0, sc1, m1;
            q4k_scale_min(scales, 2 * c, &sc0, &m0);
            q4k_scale_min(scales, 2 * c + 1, &sc1, &m1);
            volatile float d0 = d * (float)sc0, dm0 = dmin * (float)m0;
            volatile float d1 = d * (float)sc1, dm1 = dmin * (float)m1;
            for (int l = 0; l < 32; l++) {
                volatile float p0 = d0 * (float)(qs[32 * c + l] & 0x0f);
                volatile float p1 = d1 * (float)(qs[32 * c + l] >> 4);
                out[64 * c + l] = p0 - dm0;
                out[64 * c + 32 + l] = p1 - dm1;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* T5 building blocks                                                  */
/* ------------------------------------------------------------------ */

/* y[m, n] = sum_k x[m, k] * w[n, k]   (x: M x K, w: N x K, row-major) */
static void gemm_xwT(const float *x, const float *w, float *y, int M, int N, int K) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int mb = 0; mb < M; mb += 16) {
        for (int nb = 0; nb < N; nb += 64) {
            int me = mb + 16 < M ? mb + 16 : M;
            int ne = nb + 64 < N ? nb + 64 : N;
            for (int m = mb; m < me; m++) {
                const float *xr = x + (int64_t)m * K;
                for (int n = nb; n < ne; n++) {
                    const float *wr = w + (int64_t)n * K;
                    float acc = 0.f;
#pragma omp simd reduction(+ : acc)
                    for (int k = 0; k < K; k++) acc += xr[k] * wr[k];
                    y[(int64_t)m * N + n] = acc;
                }
            }
        }
    }
}

/* T5LayerNorm: x / sqrt(mean(x^2) + eps) * w  (src/quantized_t5.rs:162-173) */
static void rmsnorm(const float *x, const float *w, float *y, int M, int D, float eps) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        const float *xr = x + (int64_t)m * D;
        float ss = 0.f;
        for (int i = 0; i < D; i++) ss += xr[i] * xr[i];
        float var = ss / (float)D;
        float den = sqrtf(var + eps);
        for (int i = 0; i < D; i++) y[(int64_t)m * D + i] = xr[i] / den * w[i];
    }
}

/* Bidirectional T5 relative-position bucket for query i, key j
 * (src/quantized_t5.rs:447-483; Rust f32::log(x, b) = ln(x) / ln(b)). */
int oracle_t5_bucket(int i, int j, int num_buckets_total, int max_distance) {
    const int nb = num_buckets_total / 2;
    const int max_exact = nb / 2;
    if (i < j) {
        int dlt = j - i;
        if (dlt < max_exact) return dlt + nb;
        float b = (logf((float)dlt / (float)max_exact) /
                   logf((float)max_distance / (float)max_exact)) *
                  (float)(nb - max_exact);
        int v = max_exact + nb + (int)(uint32_t)b;
        return v < num_buckets_total - 1 ? v : num_buckets_total - 1;
    } else {
        int dlt = i - j;
        if (dlt < max_exact) return dlt;
        float b = (logf((float)dlt / (float)max_exact) /
                   logf((float)max_distance / (float)max_exact)) *
                  (float)(nb - max_exact);
        int v = max_exact + (int)(uint32_t)b;
        return v < nb - 1 ? v : nb - 1;
    }
}

/* One (sequence, head) attention: o = softmax(q k^T + bias) v, no scaling.
 * q/k/v rows have stride ld; bias_tab is [num_buckets][H] (the
 * relative_attention_bias embedding, row = bucket). */
static void attn_head(const float *q, const float *k, const float *v, int ld, float *o, int ldo,
                      int len, int h, int H, int dh, const float *bias_tab, const int *bucket_lut,
                      int lut_off, float *scratch) {
    for (int i = 0; i < len; i++) {
        float mx = -INFINITY;
        for (int j = 0; j < len; j++) {
            float s = 0.f;
            for (int t = 0; t < dh; t++) s += q[(int64_t)i * ld + t] * k[(int64_t)j * ld + t];
            s += bias_tab[bucket_lut[j - i + lut_off] * H + h];
            scratch[j] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.f;
        for (int j = 0; j < len; j++) {
            scratch[j] = expf(scratch[j] - mx);
            sum += scratch[j];
        }
        for (int t = 0; t < dh; t++) {
            float acc = 0.f;
            for (int j = 0; j < len; j++) acc += scratch[j] * v[(int64_t)j * ld + t];
            o[(int64_t)i * ldo + t] = acc / sum;
        }
    }
}

typedef struct {
    int vocab, d_model, n_heads, d_kv, d_ff, n_layers, num_buckets, max_distance, d_proj;
    float eps;
    const float *embed;        /* vocab x d_model */
    const float *rel_bias;     /* num_buckets x n_heads */
    const float *const *ln0;   /* [layer] -> d_model */
    const float *const *wq, *const *wk, *const *wv, *const *wo_attn; /* [layer] -> inner x d_model */
    const float *const *ln1;
    const float *const *wi0, *const *wi1; /* [layer] -> d_ff x d_model */
    const float *const *wo_ff;            /* [layer] -> d_model x d_ff */
    const float *final_ln;                /* d_model */
    const float *proj;                    /* d_proj x d_model */
} oracle_t5_weights;

/* Attention over a padded batch: qkv token-major [B*L][3*inner] (q|k|v),
 * output [B*L][inner].  Rows at positions >= lengths[b] are zeroed. */
void oracle_attention(const float *qkv, int B, int L, int H, int dh, const int32_t *lengths,
                      const float *bias_tab, int num_buckets, int max_distance, float *out) {
    const int inner = H * dh;
    const int ld = 3 * inner;
    int *lut = (int *)malloc(sizeof(int) * (2 * L - 1));
    for (int dlt = -(L - 1); dlt <= L - 1; dlt++)
        lut[dlt + L - 1] = dlt >= 0 ? oracle_t5_bucket(0, dlt, num_buckets, max_distance)
                                    : oracle_t5_bucket(-dlt, 0, num_buckets, max_distance);
    memset(out, 0, sizeof(float) * (size_t)B * L * inner);
#pragma omp parallel
    {
        float *scratch = (float *)malloc(sizeof(float) * L);
#pragma omp for collapse(2) schedule(dynamic)
        for (int b = 0; b < B; b++)
            for (int h = 0; h < H; h++) {
                const float *base = qkv + (int64_t)b * L * ld;
                attn_head(base + h * dh, base + inner + h * dh, base + 2 * inner + h * dh, ld,
                          out + (int64_t)b * L * inner + h * dh, inner, lengths[b], h, H, dh,
                          bias_tab, lut, L - 1, scratch);
            }
        free(scratch);
    }
    free(lut);
}

static float gelu_tanh(float g) {
    return 0.5f * g * (1.0f + tanhf(0.7978845608f * (g + 0.044715f * g * g * g)));
}

/* Full encoder forward.  out: [B][L][d_proj] raw projection (not normalised).
 * If hidden_out != NULL, the final-normed hidden states [B][L][d_model] are
 * written there too. */
void oracle_t5_encode(const oracle_t5_weights *w, const uint32_t *ids, const int32_t *lengths,
                      int B, int L, float *out) {
    const int D = w->d_model, H = w->n_heads, dh = w->d_kv, F = w->d_ff;
    const int inner = H * dh;
    memset(out, 0, sizeof(float) * (size_t)B * L * w->d_proj);
    for (int b = 0; b < B; b++) {
        const int n = lengths[b];
        if (n <= 0) continue;
        float *x = (float *)malloc(sizeof(float) * (size_t)n * D);
        float *xn = (float *)malloc(sizeof(float) * (size_t)n * D);
        float *qkv = (float *)malloc(sizeof(float) * (size_t)n * 3 * inner);
        float *tmp = (float *)malloc(sizeof(float) * (size_t)n * inner);
        float *att = (float *)malloc(sizeof(float) * (size_t)n * inner);
        float *g = (float *)malloc(sizeof(float) * (size_t)n * F);
        float *u = (float *)malloc(sizeof(float) * (size_t)n * F);
        float *y = (float *)malloc(sizeof(float) * (size_t)n * D);
        for (int t = 0; t < n; t++)
            memcpy(x + (size_t)t * D, w->embed + (size_t)ids[(size_t)b * L + t] * D, sizeof(float) * D);
        for (int l = 0; l < w->n_layers; l++) {
            /* self-attention sub-layer */
            rmsnorm(x, w->ln0[l], xn, n, D, w->eps);
            gemm_xwT(xn, w->wq[l], tmp, n, inner, D);
            for (int t = 0; t < n; t++) memcpy(qkv + (size_t)t * 3 * inner, tmp + (size_t)t * inner, sizeof(float) * inner);
            gemm_xwT(xn, w->wk[l], tmp, n, inner, D);
            for (int t = 0; t < n; t++) memcpy(qkv + (size_t)t * 3 * inner + inner, tmp + (size_t)t * inner, sizeof(float) * inner);
            gemm_xwT(xn, w->wv[l], tmp, n, inner, D);
            for (int t = 0; t < n; t++) memcpy(qkv + (size_t)t * 3 * inner + 2 * inner, tmp + (size_t)t * inner, sizeof(float) * inner);
            int32_t len1 = n;
            oracle_attention(qkv, 1, n, H, dh, &len1, w->rel_bias, w->num_buckets, w->max_distance, att);
            gemm_xwT(att, w->wo_attn[l], y, n, D, inner);
            for (size_t i = 0; i < (size_t)n * D; i++) x[i] = x[i] + y[i];
            /* gated-GELU feed-forward sub-layer */
            rmsnorm(x, w->ln1[l], xn, n, D, w->eps);
            gemm_xwT(xn, w->wi0[l], g, n, F, D);
            gemm_xwT(xn, w->wi1[l], u, n, F, D);
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n * F; i++) g[i] = gelu_tanh(g[i]) * u[i];
            gemm_xwT(g, w->wo_ff[l], y, n, D, F);
            for (size_t i = 0; i < (size_t)n * D; i++) x[i] = x[i] + y[i];
        }
        rmsnorm(x, w->final_ln, xn, n, D, w->eps);
        float *o = (float *)malloc(sizeof(float) * (size_t)n * w->d_proj);
        gemm_xwT(xn, w->proj, o, n, w->d_proj, D);
        for (int t = 0; t < n; t++)
            memcpy(out + ((size_t)b * L + t) * w->d_proj, o + (size_t)t * w->d_proj, sizeof(float) * w->d_proj);
        free(o); free(x); free(xn); free(qkv); free(tmp); free(att); free(g); free(u); free(y);
    }
}

/* Plain f32 GEMM y = x w^T for the GEMM microbench's CPU leg. */
void oracle_gemm(const float *x, const float *w, float *y, int M, int N, int K) { gemm_xwT(x, w, y, M, N, K); }

int oracle_num_threads(void) { return omp_get_max_threads(); }
void oracle_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
