/*
 * CPU restatement of the Block-GTQ hot path - TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker for the CUDA library, never part of it: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.  It restates the
 * reference algorithm for the two hot paths:
 *
 *   encode       src/webgpu/mixed.wgsl:15-41 (= src/model/codec.wgsl:11-33,
 *                src/reference/production_math.py:4-24) with packing from
 *                src/reference/mixed_layout.py:21-27 and FP16 rounding from
 *                src/webgpu/half.wgsl:2-12
 *   reconstruct  src/webgpu/mixed.wgsl:43-56 (= src/reference/production_math.py:27-31)
 *   attention    src/reference/attention.py:5-22 (logits / softmax / P.V)
 *
 * Tables are the reference's flattened interchange format (src/webgpu/layout.ts:24-31):
 *   config u32: [d, groups, rowBytes, normStride, nibbleDims, maxCentroids,
 *                off_perm, off_groupOf, off_posToCb, off_codeLut, ...payload]
 *   table  f32: [rotation d*d (row j = output j), centroids d*maxC, offsets d, invScales d]
 *
 * Canonical FP32 operation order (shared bit-for-bit with the CUDA encoder):
 *   - group sums of squares and centroid squares accumulate sequentially in ascending
 *     dimension order with fused multiply-add;
 *   - y_j = sum over i of xn_i * R[j][i], sequential in ascending i with fused
 *     multiply-add (off-group entries are exact zeros, so restricting i to the group
 *     gives the same bits);
 *   - raw group norm n_g = sqrt(sum + 1e-30); the corrected scale divides n_g directly,
 *     as the WGSL encoder does (the PyTorch emulator averages repeated per-position
 *     norms instead, which differs by at most an ulp of FP32 before FP16 rounding).
 * Attention accumulates in double and rounds each output to float once.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define CFG_D 0
#define CFG_GROUPS 1
#define CFG_ROW 2
#define CFG_NSTRIDE 3
#define CFG_NIB 4
#define CFG_MAXC 5
#define CFG_PERM 6
#define CFG_GROUP 7
#define CFG_CB 8
#define CFG_LUT 9

/* IEEE binary16 round-to-nearest-even of a finite float; follows half.wgsl:2-12. */
uint16_t orc_half_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int e = (int)((bits >> 23) & 255u) - 112;
    uint32_t fraction = bits & 0x7FFFFFu;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e < -10) return (uint16_t)sign;
    uint32_t mantissa = fraction, shift = 13u, exponent = (uint32_t)(e > 0 ? e : 0) << 10;
    if (e <= 0) { mantissa |= 0x800000u; shift = (uint32_t)(14 - e); exponent = 0; }
    uint32_t base = mantissa >> shift, rem = mantissa & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    uint32_t inc = (rem > half || (rem == half && (base & 1u))) ? 1u : 0u;
    return (uint16_t)(sign | (exponent + base + inc));
}

/* binary16 -> float, exact; follows half.wgsl:13-18. */
float orc_half_value(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u, bits;
    float f;
    if (e == 0) { f = (float)m * 5.960464477539063e-8f; return (h & 0x8000u) ? -f : f; }
    if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    memcpy(&f, &bits, 4);
    return f;
}

static int group_of(const uint32_t *cfg, int i) { return (int)cfg[cfg[CFG_GROUP] + i]; }

/* Byte address and nibble shift of code i inside a packed row (mixed.wgsl:36-40). */
static void code_position(const uint32_t *cfg, int i, int *byte, int *shift) {
    int ns = (int)cfg[CFG_NIB];
    if (i < ns) { *byte = i / 2; *shift = (i % 2) * 4; }
    else { *byte = ns / 2 + i - ns; *shift = 0; }
}

/* Encode rows of FP16 keys (natural dimension order, `in_stride` elements apart).
 * Writes packed rows (`row_stride` bytes apart, logical bytes then zero padding) and
 * FP16 scale bits (`scale_stride` halves apart, groups then zero padding).  Optional
 * outputs: codes [n][d] in packed (head-permuted) order, rotated y [n][d], corrected
 * FP32 scales [n][groups]. */
void orc_encode_f16(const uint32_t *cfg, const float *tab, const uint16_t *rows, long n, long in_stride,
                    uint8_t *packed, long row_stride, uint16_t *scales, long scale_stride,
                    uint8_t *codes_out, float *y_out, float *corrected_out, int threads) {
    const int d = (int)cfg[CFG_D], ng = (int)cfg[CFG_GROUPS], maxc = (int)cfg[CFG_MAXC];
    const float *rot = tab, *cent = tab + (size_t)d * d, *off = cent + (size_t)d * maxc, *inv = off + d;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (long r = 0; r < n; r++) {
        float x[128], y[128], len[8] = {0}, clen[8] = {0}, norm[8];
        uint8_t codes[128];
        const uint16_t *row = rows + r * in_stride;
        for (int i = 0; i < d; i++) {
            x[i] = orc_half_value(row[cfg[cfg[CFG_PERM] + i]]);
            int g = group_of(cfg, i);
            len[g] = fmaf(x[i], x[i], len[g]);
        }
        for (int g = 0; g < ng; g++) norm[g] = sqrtf(len[g] + 1e-30f);
        for (int i = 0; i < d; i++) {
            float nn = norm[group_of(cfg, i)];
            x[i] = x[i] / (nn > 1e-10f ? nn : 1.0f);
        }
        for (int j = 0; j < d; j++) {
            float acc = 0.0f;
            for (int i = 0; i < d; i++) acc = fmaf(x[i], rot[(size_t)j * d + i], acc);
            y[j] = acc;
            float t = (acc - off[j]) * inv[j];
            t = t < 0.0f ? 0.0f : (t > 255.0f ? 255.0f : t);
            uint32_t bin = (uint32_t)t;
            uint32_t code = cfg[cfg[CFG_LUT] + cfg[cfg[CFG_CB] + j] * 256u + bin];
            codes[j] = (uint8_t)code;
            float c = cent[(size_t)j * maxc + code];
            int g = group_of(cfg, j);
            clen[g] = fmaf(c, c, clen[g]);
        }
        uint16_t *srow = scales + r * scale_stride;
        for (int g = 0; g < scale_stride; g++) srow[g] = 0;
        for (int g = 0; g < ng; g++) {
            float s = norm[g] / fmaxf(sqrtf(clen[g]), 1e-10f);
            srow[g] = orc_half_bits(s);
            if (corrected_out) corrected_out[r * ng + g] = s;
        }
        uint8_t *prow = packed + r * row_stride;
        memset(prow, 0, (size_t)row_stride);
        for (int i = 0; i < d; i++) {
            int b, sh;
            code_position(cfg, i, &b, &sh);
            prow[b] |= (uint8_t)(codes[i] << sh);
        }
        if (codes_out) memcpy(codes_out + r * d, codes, (size_t)d);
        if (y_out) memcpy(y_out + r * d, y, sizeof(float) * (size_t)d);
    }
}

/* Same encoder fed from FP32 activations that are first rounded to FP16, with the
 * row stride and head offset of the model path (codec.wgsl:14). */
void orc_encode_f32(const uint32_t *cfg, const float *tab, const float *act, long n, long row_elems, long head_offset,
                    uint8_t *packed, long row_stride, uint16_t *scales, long scale_stride, int threads) {
    const int d = (int)cfg[CFG_D];
    uint16_t *tmp = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(n > 0 ? n : 1) * d);
    for (long r = 0; r < n; r++)
        for (int i = 0; i < d; i++) tmp[r * d + i] = orc_half_bits(act[r * row_elems + head_offset + i]);
    orc_encode_f16(cfg, tab, tmp, n, d, packed, row_stride, scales, scale_stride, NULL, NULL, NULL, threads);
    free(tmp);
}

/* Reconstruct FP32 keys in natural dimension order (mixed.wgsl:43-56). */
void orc_reconstruct(const uint32_t *cfg, const float *tab, const uint8_t *packed, long row_stride,
                     const uint16_t *scales, long scale_stride, long n, float *out, int threads) {
    const int d = (int)cfg[CFG_D], maxc = (int)cfg[CFG_MAXC];
    const float *rot = tab, *cent = tab + (size_t)d * d;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (long r = 0; r < n; r++) {
        float val[128];
        const uint8_t *prow = packed + r * row_stride;
        for (int i = 0; i < d; i++) {
            int b, sh;
            code_position(cfg, i, &b, &sh);
            uint32_t code = (uint32_t)(prow[b] >> sh) & (i < (int)cfg[CFG_NIB] ? 15u : 255u);
            val[i] = cent[(size_t)i * maxc + code] * orc_half_value(scales[r * scale_stride + group_of(cfg, i)]);
        }
        for (int j = 0; j < d; j++) {
            float acc = 0.0f;
            for (int i = 0; i < d; i++) acc = fmaf(val[i], rot[(size_t)i * d + j], acc);
            out[r * d + cfg[cfg[CFG_PERM] + j]] = acc;
        }
    }
}

/* Attention of nq query rows over T keys of width d (attention.py:5-22) in double.
 * K and V are float rows `k_stride` / `v_stride` elements apart.  logits / probs may be
 * NULL; masked logits are -inf and their probabilities exactly 0. */
void orc_attention(const float *q, long nq, const float *k, long k_stride, const float *v, long v_stride,
                   long T, int d, const uint32_t *positions, int causal, float *logits, float *probs, float *out,
                   int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (long r = 0; r < nq; r++) {
        double *lg = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1));
        double m = -INFINITY, scale = 1.0 / sqrt((double)d);
        long end = causal ? (long)positions[r] + 1 : T;
        for (long t = 0; t < T; t++) {
            if (t >= end) { lg[t] = -INFINITY; continue; }
            double s = 0.0;
            for (int i = 0; i < d; i++) s += (double)q[r * d + i] * (double)k[t * k_stride + i];
            lg[t] = s * scale;
            if (lg[t] > m) m = lg[t];
        }
        double sum = 0.0;
        for (long t = 0; t < end; t++) sum += exp(lg[t] - m);
        double acc[128] = {0};
        for (long t = 0; t < end; t++) {
            double p = exp(lg[t] - m) / sum;
            for (int i = 0; i < d; i++) acc[i] += p * (double)v[t * v_stride + i];
        }
        for (int i = 0; i < d; i++) out[r * d + i] = (float)acc[i];
        if (logits) for (long t = 0; t < T; t++) logits[r * T + t] = (float)lg[t];
        if (probs) for (long t = 0; t < T; t++) probs[r * T + t] = t < end ? (float)(exp(lg[t] - m) / sum) : 0.0f;
        free(lg);
    }
}
