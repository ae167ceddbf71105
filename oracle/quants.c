/*
 * oracle/quants.c -- CPU restatement of the GGUF block formats used on the
 * verify step, and of the quantized matmul the reference performs on them.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this file.  It is the checker: tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py are its only users.
 *
 * What it restates
 * ----------------
 * The reference never dequantizes by hand: every quantized linear layer is a
 * `candle_core::quantized::QMatMul::forward` call (candle 0.8.4, pinned in
 * Cargo.lock:285-358, source not vendored).  Call sites:
 *   crates/speculate/src/model/quantized_llama_local.rs:47-49  (Mlp w1/w3/w2)
 *   crates/speculate/src/model/quantized_llama_local.rs:73-90  (wq/wk/wv)
 *   crates/speculate/src/model/quantized_llama_local.rs:135    (wo)
 *   crates/speculate/src/model/quantized_llama_local.rs:316-318 (output / lm_head)
 *   crates/speculate/src/model/quantized_qwen2_local.rs:41-44,71-82,138,314-316
 * and the embedding table is dequantized once at load
 *   (quantized_llama_local.rs:242-243, quantized_qwen2_local.rs:232-233).
 * QMatMul computes y = x . W^T where W is stored as GGUF blocks.  The block
 * layouts are the public GGML/GGUF specification (the same one candle and the
 * `gguf` 0.19.0 Python package implement); the per-format decode below follows
 * that specification:
 *
 *   Q4_K: 256 elements / 144 bytes = f16 d, f16 dmin, 12 bytes of packed
 *         6-bit (scale, min) x 8, 128 bytes of 4-bit codes.
 *         w = (d*sc_j) * q - (dmin*m_j), sub-block j of 32 elements.
 *   Q5_K: 256 / 176 = f16 d, f16 dmin, 12 bytes scales, 32 bytes high bits,
 *         128 bytes low nibbles.  q = nibble + 16*highbit, same formula.
 *   Q6_K: 256 / 210 = 128 bytes low nibbles, 64 bytes 2-bit highs,
 *         16 int8 scales, f16 d.  w = (d*sc_j) * (q - 32), sub-block of 16.
 *   Q8_0: 32 / 34 = f16 d, 32 int8.  w = d * q.
 *
 * The decode is pinned bit-exactly against gguf 0.19.0's
 * `gguf.quants.dequantize` by tests/golden (see tests/golden/make_golden.py).
 *
 * oq_qmatmul accumulates in double: it is the "ideal arithmetic" statement of
 * y = x . W^T that the GPU kernels are compared against with a tolerance.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OQ_F32 = 0, OQ_F16 = 1, OQ_Q8_0 = 8, OQ_Q4_K = 12, OQ_Q5_K = 13, OQ_Q6_K = 14, OQ_BF16 = 30 };

static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400));
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf2f(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Unpack the j-th 6-bit (scale, min) pair of a Q4_K / Q5_K superblock. */
static void scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

int oq_block_elems(int fmt) {
    switch (fmt) {
        case OQ_Q4_K: case OQ_Q5_K: case OQ_Q6_K: return 256;
        case OQ_Q8_0: return 32;
        case OQ_F32: case OQ_F16: case OQ_BF16: return 1;
    }
    return 0;
}

int oq_block_bytes(int fmt) {
    switch (fmt) {
        case OQ_Q4_K: return 144;
        case OQ_Q5_K: return 176;
        case OQ_Q6_K: return 210;
        case OQ_Q8_0: return 34;
        case OQ_F32: return 4;
        case OQ_F16: case OQ_BF16: return 2;
    }
    return 0;
}

static void deq_q4k(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; c++) {
        uint8_t sc, m;
        scale_min_k4(2 * c, scales, &sc, &m);
        const float d1 = d * sc, m1 = dmin * m;
        scale_min_k4(2 * c + 1, scales, &sc, &m);
        const float d2 = d * sc, m2 = dmin * m;
        for (int l = 0; l < 32; l++) y[64 * c + l] = d1 * (qs[32 * c + l] & 0xF) - m1;
        for (int l = 0; l < 32; l++) y[64 * c + 32 + l] = d2 * (qs[32 * c + l] >> 4) - m2;
    }
}

static void deq_q5k(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int c = 0; c < 4; c++) {
        uint8_t sc, m;
        const uint8_t u1 = (uint8_t)(1u << (2 * c)), u2 = (uint8_t)(2u << (2 * c));
        scale_min_k4(2 * c, scales, &sc, &m);
        const float d1 = d * sc, m1 = dmin * m;
        scale_min_k4(2 * c + 1, scales, &sc, &m);
        const float d2 = d * sc, m2 = dmin * m;
        for (int l = 0; l < 32; l++)
            y[64 * c + l] = d1 * ((qs[32 * c + l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
        for (int l = 0; l < 32; l++)
            y[64 * c + 32 + l] = d2 * ((qs[32 * c + l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
    }
}

static void deq_q6k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = h2f(rd16(b + 208));
    for (int n = 0; n < 2; n++) {
        const uint8_t* l8 = ql + 64 * n;
        const uint8_t* h8 = qh + 32 * n;
        const int8_t* s8 = sc + 8 * n;
        float* yy = y + 128 * n;
        for (int l = 0; l < 32; l++) {
            const int is = l / 16;
            const int q1 = (int)((l8[l] & 0xF) | (((h8[l] >> 0) & 3) << 4)) - 32;
            const int q2 = (int)((l8[l + 32] & 0xF) | (((h8[l] >> 2) & 3) << 4)) - 32;
            const int q3 = (int)((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
            const int q4 = (int)((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
            yy[l] = d * s8[is + 0] * q1;
            yy[l + 32] = d * s8[is + 2] * q2;
            yy[l + 64] = d * s8[is + 4] * q3;
            yy[l + 96] = d * s8[is + 6] * q4;
        }
    }
}

static void deq_q80(const uint8_t* b, float* y) {
    const float d = h2f(rd16(b));
    const int8_t* q = (const int8_t*)(b + 2);
    for (int l = 0; l < 32; l++) y[l] = d * q[l];
}

/* Dequantize n elements (a multiple of the format's block size). */
int oq_dequant(int fmt, const uint8_t* src, int64_t n, float* out) {
    const int be = oq_block_elems(fmt), bb = oq_block_bytes(fmt);
    if (be == 0 || n % be) return -1;
    const int64_t nb = n / be;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t* b = src + i * bb;
        float* y = out + i * be;
        switch (fmt) {
            case OQ_Q4_K: deq_q4k(b, y); break;
            case OQ_Q5_K: deq_q5k(b, y); break;
            case OQ_Q6_K: deq_q6k(b, y); break;
            case OQ_Q8_0: deq_q80(b, y); break;
            case OQ_F32: memcpy(y, b, 4); break;
            case OQ_F16: y[0] = h2f(rd16(b)); break;
            case OQ_BF16: y[0] = bf2f(rd16(b)); break;
            default: return -1;
        }
    }
    return 0;
}

/*
 * y[m][n] = sum_k W[n][k] * x[m][k]   (W: N rows of K elements in `fmt` blocks)
 * Each row is dequantized into a scratch buffer and dotted with every
 * activation row.  `acc_double` != 0 accumulates in double (the ideal
 * arithmetic the GPU kernels are checked against); 0 accumulates in float in
 * 16 independent lanes (the vectorisable form used when this file is timed as
 * the CPU baseline).  Rows are spread over `nthreads` OpenMP threads (<= 0:
 * all available).
 */
int oq_qmatmul(int fmt, const uint8_t* W, int64_t N, int64_t K, const float* x, int64_t M,
               float* y, int nthreads, int acc_double) {
    const int be = oq_block_elems(fmt), bb = oq_block_bytes(fmt);
    if (be == 0 || K % be || K > (1 << 20)) return -1;
    const int64_t row_bytes = (K / be) * bb;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    int err = 0;
#pragma omp parallel reduction(| : err)
    {
        float* rowbuf = (float*)malloc(sizeof(float) * (size_t)K);
        if (!rowbuf) err |= 1;
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            if (!rowbuf) continue;
            if (oq_dequant(fmt, W + n * row_bytes, K, rowbuf)) { err |= 1; continue; }
            for (int64_t m = 0; m < M; m++) {
                const float* xm = x + m * K;
                if (acc_double) {
                    double acc = 0.0;
                    for (int64_t k = 0; k < K; k++) acc += (double)rowbuf[k] * (double)xm[k];
                    y[m * N + n] = (float)acc;
                } else {
                    float lane[16] = {0};
                    int64_t k = 0;
                    for (; k + 16 <= K; k += 16)
                        for (int j = 0; j < 16; j++) lane[j] += rowbuf[k + j] * xm[k + j];
                    float acc = 0.f;
                    for (; k < K; k++) acc += rowbuf[k] * xm[k];
                    for (int j = 0; j < 16; j++) acc += lane[j];
                    y[m * N + n] = acc;
                }
            }
        }
        free(rowbuf);
    }
    return err ? -1 : 0;
}

/*
 * oq_attention: the attention core of one layer for M new rows, the CPU leg
 * of the verify-step timing (bench.py cpu_baseline / --impl reference).
 * Restates run_attn (crates/speculate/src/model/quantized_llama_local.rs:
 * 107-136): scores q . k^T / sqrt(hd) plus the causal bias (causal_bias,
 * :332-350: the T - M prefix keys are visible to every row, new key j to new
 * row i iff j <= i), softmax over the keys, times v; the G = n_heads / n_kv
 * query heads of a KV head share it (repeat_kv, :115-123).
 *   q   [n_heads][M][hd]   (rows already rotated)
 *   k,v [n_kv][T][hd]      (T = prefix + M keys, the new rows last)
 *   out [M][n_heads * hd]
 * f32 throughout (the reference's quantized model keeps f32 activations);
 * heads run in parallel with OpenMP.
 */
int oq_attention(const float* q, const float* k, const float* v, int n_heads, int n_kv, int M, int T, int hd,
                 float* out, int nthreads) {
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || M <= 0 || T < M || hd <= 0) return -1;
    const int G = n_heads / n_kv, prefix = T - M;
    const float scale = 1.0f / sqrtf((float)hd);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    int err = 0;
#pragma omp parallel reduction(| : err)
    {
        float* s = (float*)malloc(sizeof(float) * (size_t)T);
        if (!s) err |= 1;
#pragma omp for schedule(static)
        for (int hm = 0; hm < n_heads * M; hm++) {
            if (!s) continue;
            const int h = hm / M, i = hm % M, kvh = h / G;
            const float* qi = q + ((size_t)h * M + i) * hd;
            const float* kh = k + (size_t)kvh * T * hd;
            const float* vh = v + (size_t)kvh * T * hd;
            const int visible = prefix + i + 1;
            float mx = -INFINITY;
            for (int j = 0; j < visible; j++) {
                float acc = 0.f;
                for (int d = 0; d < hd; d++) acc += qi[d] * kh[(size_t)j * hd + d];
                s[j] = acc * scale;
                if (s[j] > mx) mx = s[j];
            }
            float sum = 0.f;
            for (int j = 0; j < visible; j++) {
                s[j] = expf(s[j] - mx);
                sum += s[j];
            }
            float* o = out + (size_t)i * n_heads * hd + (size_t)h * hd;
            for (int d = 0; d < hd; d++) o[d] = 0.f;
            for (int j = 0; j < visible; j++) {
                const float p = s[j] / sum;
                for (int d = 0; d < hd; d++) o[d] += p * vh[(size_t)j * hd + d];
            }
        }
        free(s);
    }
    return err ? -1 : 0;
}
