// Block-GTQ K encode for sm_100a (replaces src/webgpu/mixed.wgsl:15-41 and
// src/model/codec.wgsl:11-33; arithmetic of src/reference/production_math.py:4-24,
// packing of src/reference/mixed_layout.py:21-27, FP16 rounding of src/webgpu/half.wgsl:2-12).
//
// Bulk (a prefix of many tokens): one thread encodes one key; a persistent CTA of 128
// threads walks tiles of 128 keys so the rotation, codebooks and code LUT are staged in
// shared memory once per CTA.  Few keys (decode steps): one warp per key, tables read
// through the L1 cache (encode_warp_kernel).
// Per key, in the canonical order the CPU oracle shares bit for bit:
//   x_i   = FP16 key element perm[i]              (exact promotion)
//   n_g   = sqrt(sum_{i in g} x_i^2 + 1e-30)      (sequential FMA, ascending i)
//   xn_i  = x_i / (n_g > 1e-10 ? n_g : 1)         (IEEE division)
//   y_j   = sum_i xn_i R[j][i]                    (sequential FMA over the group of j)
//   bin_j = trunc(clamp((y_j - off_j) * inv_j, 0, 255)); code_j = LUT[cb_j][bin_j]
//   s_g   = n_g / max(sqrt(sum_{j in g} cent[j][code_j]^2), 1e-10) -> FP16 (RNE)
// This file is compiled with -fmad=false so no separate multiply/add pair is contracted;
// every fused multiply-add above is an explicit fmaf.
#include <cuda_fp16.h>

#include <cstdlib>

#include "bgtq_internal.h"
#include "encode_impl.cuh"

namespace bgtq {
namespace {

constexpr int kThreads = 128;
// Launches of at most this many keys per head use the warp-per-key kernel.
constexpr uint32_t kWarpKeysMax = 4096;

__device__ __forceinline__ bool bit_set(const uint32_t (&m)[4], int j) { return (m[j >> 5] >> (j & 31)) & 1u; }
// The same bit at a run-time index, chosen from the four registers by selects (an indexed
// register array would be placed in local memory).
__device__ __forceinline__ bool bit_set_rt(const uint32_t (&m)[4], uint32_t j) {
    const uint32_t w = j >> 5;
    const uint32_t word = w == 0 ? m[0] : w == 1 ? m[1] : w == 2 ? m[2] : m[3];
    return (word >> (j & 31)) & 1u;
}
// Quotient n / d for n * d < 2^32 from one high multiply by m = ceil(2^32 / d) (d > 1):
// n * m / 2^32 = n / d + n * e / (d * 2^32) with e = m * d - 2^32 < d, whose second term
// stays below 1 / d, so the floor is exact.
__device__ __forceinline__ uint32_t div_small(uint32_t n, uint32_t d, uint32_t m) { return d == 1 ? n : __umulhi(n, m); }

template <int D>
__global__ void __launch_bounds__(kThreads) encode_kernel(const __grid_constant__ EncodeArgs a, uint32_t d,
                                                          uint32_t cent_alloc, uint32_t lut_bytes, uint32_t total) {
    const EncodeHead &h = a.head[blockIdx.y];
    constexpr int SW = D / 2 + 1;  // staged input words per key (odd: conflict-free gathers)
    const uint32_t row_words = h.row_stride / 4, ow = row_words | 1u;  // odd: conflict-free row stores
    const uint32_t sc_words = h.scale_stride / 2, sw = sc_words + 1;

    extern __shared__ __align__(16) unsigned char smem[];
    float *rot_s = reinterpret_cast<float *>(smem);           // [D][D]
    float *cent_s = rot_s + D * D;                            // [cent_alloc]
    float *off_s = cent_s + cent_alloc;                       // [D]
    float *inv_s = off_s + D;                                 // [D]
    float *norm_s = inv_s + D;                                // [kMaxGroups][kThreads]
    uint32_t *stage_s = reinterpret_cast<uint32_t *>(norm_s + kMaxGroups * kThreads);  // [kThreads][SW]
    uint32_t *out_s = stage_s + kThreads * SW;                // [kThreads][ow]
    uint32_t *sc_s = out_s + kThreads * ow;                   // [kThreads][sw]
    uint16_t *cbbase_s = reinterpret_cast<uint16_t *>(sc_s + kThreads * sw);  // [D]
    uint8_t *lut_s = reinterpret_cast<uint8_t *>(cbbase_s + D);               // [lut_bytes]
    uint8_t *perm_s = lut_s + lut_bytes;                      // [D]
    uint8_t *cbidx_s = perm_s + D;                            // [D]
    uint8_t *glo_s = cbidx_s + D;                             // [D] group start of dim j
    uint8_t *ghi_s = glo_s + D;                               // [D] group end (exclusive); 128 fits

    const int tid = threadIdx.x;
    // ---- stage the tables once per CTA ----
    for (uint32_t i = tid; i < (uint32_t)(D * D); i += kThreads) {
        const uint32_t j = i / D, c = i % D;
        rot_s[i] = (j < d && c < d) ? h.t.rot[j * d + c] : 0.0f;
    }
    for (uint32_t i = tid; i < cent_alloc; i += kThreads) cent_s[i] = i < h.n_cent ? h.t.cent[i] : 0.0f;
    for (uint32_t i = tid; i < (uint32_t)D; i += kThreads) {
        const bool live = i < d;
        off_s[i] = live ? h.t.off[i] : 0.0f;
        inv_s[i] = live ? h.t.inv[i] : 0.0f;
        perm_s[i] = live ? h.t.perm[i] : (uint8_t)i;
        cbidx_s[i] = live ? h.t.cbidx[i] : 0;
        cbbase_s[i] = live ? h.t.cb_base[i] : 0;
        const uint32_t g = live ? h.t.group_of[i] : 0;
        glo_s[i] = live ? (uint8_t)h.group_off[g] : 0;
        ghi_s[i] = live ? (uint8_t)h.group_off[g + 1] : 0;
    }
    for (uint32_t i = tid; i < lut_bytes; i += kThreads) lut_s[i] = i < h.ncb * 256u ? h.t.lut[i] : 0;
    uint32_t bm[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) bm[w] = h.bound_mask[w];
    const uint32_t ns = h.ns, ng = h.ng, count = a.count;
    // row-word and scale-word quotients by high multiplies (w < kThreads * 64 words)
    const uint32_t rw_magic = row_words > 1 ? (uint32_t)((0x100000000ull + row_words - 1) / row_words) : 0u;
    const uint32_t sw_magic = sc_words > 1 ? (uint32_t)((0x100000000ull + sc_words - 1) / sc_words) : 0u;
    const bool vec16 = !a.src_f32 && d == (uint32_t)D &&
                       (((uintptr_t)a.src | ((a.seq_stride | a.row_stride | h.src_head_offset) * 2u)) & 15u) == 0;
    __shared__ uint64_t rsrc_s[kThreads], rdst_s[kThreads], rsc_s[kThreads];
    __syncthreads();

    const uint32_t n_tiles = (total + kThreads - 1) / kThreads;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const uint32_t first = tile * kThreads;
        const uint32_t nrows = min((uint32_t)kThreads, total - first);
        // ---- per-row source element and destination offsets (one division per row) ----
        if ((uint32_t)tid < nrows) {
            const uint32_t q = first + tid, s = q / count, rr = q % count;
            const uint64_t dseq = a.seq_first + s, dst_row = (a.row0 ? a.row0[s] : a.row0_scalar) + rr;
            rsrc_s[tid] = (uint64_t)s * a.seq_stride + (uint64_t)rr * a.row_stride + h.src_head_offset;
            rdst_s[tid] = dseq * h.k_seq_stride + dst_row * h.row_stride;
            rsc_s[tid] = dseq * h.s_seq_stride + dst_row * h.scale_stride;
        }
        __syncthreads();
        // ---- stage the input rows as FP16 words (coalesced) ----
        const uint32_t in_words = d / 2;
        if (vec16) {
            // full-width FP16 rows on 16-byte boundaries: one 16-byte load per 8 elements
            for (uint32_t w = tid; w < nrows * (uint32_t)(D / 8); w += kThreads) {
                const uint32_t r = w / (D / 8), c = w % (D / 8);
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.src) + rsrc_s[r] + 8u * c));
                uint32_t *dst = stage_s + r * SW + 4u * c;
                dst[0] = v.x;
                dst[1] = v.y;
                dst[2] = v.z;
                dst[3] = v.w;
            }
        } else for (uint32_t w = tid; w < nrows * (uint32_t)(D / 2); w += kThreads) {
            const uint32_t r = w / (D / 2), c = w % (D / 2);
            uint32_t word = 0;
            if (c < in_words) {
                const uint64_t e = rsrc_s[r] + 2u * c;
                if (a.src_f32) {
                    const float2 f = *reinterpret_cast<const float2 *>(static_cast<const float *>(a.src) + e);
                    word = (uint32_t)__half_as_ushort(__float2half_rn(f.x)) |
                           ((uint32_t)__half_as_ushort(__float2half_rn(f.y)) << 16);
                } else {
                    word = *reinterpret_cast<const uint32_t *>(static_cast<const uint16_t *>(a.src) + e);
                }
            }
            stage_s[r * SW + c] = word;
        }
        __syncthreads();

        if ((uint32_t)tid < nrows) {
            const uint16_t *st = reinterpret_cast<const uint16_t *>(stage_s + tid * SW);
            float x[D];
#pragma unroll
            for (int i = 0; i < D; ++i) x[i] = __half2float(__ushort_as_half(st[perm_s[i]]));
            // group sums of squares, ascending dimension order
            {
                uint32_t g = 0;
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    acc = fmaf(x[i], x[i], acc);
                    if (i + 1 < D && bit_set(bm, i + 1)) {
                        norm_s[g * kThreads + tid] = sqrtf(acc + 1e-30f);
                        ++g;
                        acc = 0.0f;
                    }
                }
                norm_s[g * kThreads + tid] = sqrtf(acc + 1e-30f);
            }
            // normalise each group by its own norm
            {
                uint32_t g = 0;
                float n = norm_s[tid];
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    if (i > 0 && bit_set(bm, i)) {
                        ++g;
                        n = norm_s[g * kThreads + tid];
                    }
                    x[i] = x[i] / (n > 1e-10f ? n : 1.0f);
                }
            }
            uint32_t *orow = out_s + tid * ow;
            uint16_t *srow = reinterpret_cast<uint16_t *>(sc_s + tid * sw);
            for (uint32_t w = 0; w < ow; ++w) orow[w] = 0;
            for (uint32_t w = 0; w < sw; ++w) sc_s[tid * sw + w] = 0;
            uint8_t *ob = reinterpret_cast<uint8_t *>(orow);
            uint32_t g = 0, pend = 0;
            float n = norm_s[tid], cl = 0.0f;
            // Four outputs per pass: four independent FMA chains, each still summed in
            // ascending i.  The pass covers the union of the four rows' group ranges; a
            // row's entries outside its own group are exact zeros and change nothing.
            for (uint32_t j0 = 0; j0 < d; j0 += 4) {
                const uint32_t jl = min(j0 + 3u, d - 1u);
                const int lo = glo_s[j0], hi = ghi_s[jl];
                const float *rj = rot_s + j0 * D;
                float y[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int c = 0; c < D / 8; ++c) {
                    if (c * 8 < hi && c * 8 + 8 > lo) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 r0 = *reinterpret_cast<const float4 *>(rj + q * D + c * 8);
                            const float4 r1 = *reinterpret_cast<const float4 *>(rj + q * D + c * 8 + 4);
                            y[q] = fmaf(x[c * 8 + 0], r0.x, y[q]);
                            y[q] = fmaf(x[c * 8 + 1], r0.y, y[q]);
                            y[q] = fmaf(x[c * 8 + 2], r0.z, y[q]);
                            y[q] = fmaf(x[c * 8 + 3], r0.w, y[q]);
                            y[q] = fmaf(x[c * 8 + 4], r1.x, y[q]);
                            y[q] = fmaf(x[c * 8 + 5], r1.y, y[q]);
                            y[q] = fmaf(x[c * 8 + 6], r1.z, y[q]);
                            y[q] = fmaf(x[c * 8 + 7], r1.w, y[q]);
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t j = j0 + q;
                    if (j >= d) break;
                    float t = (y[q] - off_s[j]) * inv_s[j];
                    t = fminf(fmaxf(t, 0.0f), 255.0f);
                    const uint32_t bin = (uint32_t)t;
                    const uint32_t code = lut_s[(uint32_t)cbidx_s[j] * 256u + bin];
                    const float cv = cent_s[cbbase_s[j] + code];
                    cl = fmaf(cv, cv, cl);
                    if (j < ns) {
                        if (j & 1u) ob[j >> 1] = (uint8_t)(pend | (code << 4));
                        else pend = code;
                    } else {
                        ob[(ns >> 1) + (j - ns)] = (uint8_t)code;
                    }
                    const uint32_t jn = j + 1;
                    if (jn == d || bit_set_rt(bm, jn)) {
                        const float s = n / fmaxf(sqrtf(cl), 1e-10f);
                        srow[g] = __half_as_ushort(__float2half_rn(s));
                        ++g;
                        cl = 0.0f;
                        if (g < ng) n = norm_s[g * kThreads + tid];
                    }
                }
            }
        }
        __syncthreads();
        // ---- write packed rows and scales (coalesced words) ----
        for (uint32_t w = tid; w < nrows * row_words; w += kThreads) {
            const uint32_t r = div_small(w, row_words, rw_magic), c = w - r * row_words;
            reinterpret_cast<uint32_t *>(h.packed + rdst_s[r])[c] = out_s[r * ow + c];
        }
        for (uint32_t w = tid; w < nrows * sc_words; w += kThreads) {
            const uint32_t r = div_small(w, sc_words, sw_magic), c = w - r * sc_words;
            reinterpret_cast<uint32_t *>(h.scales + rsc_s[r])[c] = sc_s[r * sw + c];
        }
        __syncthreads();
    }
    // ---- publish the new lengths ----
    if (blockIdx.x == 0 && h.lengths) {
        for (uint32_t s = tid; s < a.seq_count; s += kThreads)
            h.lengths[a.seq_first + s] = (a.row0 ? a.row0[s] : a.row0_scalar) + count;
    }
}

// Packed FP32 FMA (two lanes, each rounded to nearest like fmaf) in PTX.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// ---- bulk encode, head dims up to 64: tiles of keys, every phase over the whole tile ----
//
// A persistent CTA of 256 threads stages one head's tables once and walks tiles of KT = 128
// keys.  Per tile, in shared memory, the work the oracle does key by key, in its operation
// order:
//   1. input rows staged as FP16 words (coalesced), gathered through the permutation into
//      X[i][k] (FP32, key-minor: lanes over keys read consecutive words);
//   2. one thread per (key, group): the group's sum of squares (sequential FMAs, ascending
//      dims), its norm, and the division of the group's elements by it;
//   3. the block-diagonal rotation as a register-blocked product: one warp per output dim
//      pair (j, j + 1) of a group, each lane 4 keys, one packed FMA (fma.rn.f32x2) per two
//      keys and dimension - every y_j still one sequential FMA chain over its group in
//      ascending i, so each value is the oracle's bit for bit - and straight on to the LUT
//      bin and the code, stored as bytes (the FP32 outputs never leave registers).  The dim
//      pairs are dealt to the warps longest-group-first (a pair costs its group's size);
//   4. one thread per (key, group): the codebook values' squares summed in ascending dims,
//      the FP16 corrected scale, and the group's packed row bytes;
//   5. rows and scales written with coalesced word stores.
// The rotation blocks are kept duplicated ((R[j][i], R[j][i]) float pairs, the operand
// layout of the packed FMA) and compact (only the blocks on the diagonal).
constexpr int kTileKeys = 128, kTileThreads = 256, kTileWarps = kTileThreads / 32;

template <int D>
struct TileSmem {
    uint32_t rdup, jc, cent, x, nrm, uni, codes, out, sc, rows, lut, perm, task, total;
};

template <int D>
__host__ __device__ TileSmem<D> tile_smem(uint32_t rdup_pairs, uint32_t cent_alloc, uint32_t lut_bytes, uint32_t row_stride,
                      uint32_t scale_stride) {
    auto a16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    const uint32_t ow = (row_stride / 4) | 1u, sw = scale_stride / 2 + 1;
    TileSmem<D> t{};
    uint32_t o = 0;
    t.rdup = o; o += a16(8u * rdup_pairs);
    t.jc = o; o += 16u * D;
    t.cent = o; o += a16(4u * cent_alloc);
    t.x = o; o += 4u * D * kTileKeys;
    t.nrm = o; o += 4u * kMaxGroups * kTileKeys;
    // the staged FP16 input (phase 1) shares its space with the codes, rows and scales
    // (phases 3-5)
    const uint32_t stage = 4u * kTileKeys * (D / 2 + 1);
    const uint32_t codes = a16(D * kTileKeys), out = a16(4u * kTileKeys * ow), sc = a16(4u * kTileKeys * sw);
    t.uni = o;
    t.codes = o; t.out = o + codes; t.sc = o + codes + out;
    o += a16(stage > codes + out + sc ? stage : codes + out + sc);
    t.rows = o; o += 8u * 3u * kTileKeys;
    t.lut = o; o += a16(lut_bytes);
    t.perm = o; o += a16(D);
    t.task = o; o += 8u * (D / 2) * kTileWarps;
    t.total = a16(o);
    return t;
}

// Output dims j0 .. j0 + NJ - 1 (NJ = 2 or 4, one group [lo, hi)) of the lane's 4 keys: each y
// one sequential FMA chain over the group in ascending i (packed: two keys per instruction),
// then straight to the LUT bin and code; codes stored as one word per dim (4 keys).
template <int NJ>
__device__ __forceinline__ void rotate_codes(const float2 *rdup, const float *X, const float4 *jc,
                                             const uint8_t *lut_s, uint8_t *codes, uint32_t base, uint32_t j0,
                                             uint32_t lo, uint32_t hi, int lane) {
    constexpr int KT = kTileKeys;
    const uint32_t n = hi - lo, rstep = n / 2;                  // float4 per block row
    const float4 *rb = reinterpret_cast<const float4 *>(rdup + base + (j0 - lo));
    const float4 *xp = reinterpret_cast<const float4 *>(X + lo * KT + 4 * lane);
    float2 ya[NJ], yb[NJ];                                      // keys (0, 1) and (2, 3) of dim j0 + q
#pragma unroll
    for (int q = 0; q < NJ; ++q) ya[q] = yb[q] = make_float2(0.0f, 0.0f);
#pragma unroll 4
    for (uint32_t i = 0; i < n; ++i) {
        const float4 x = xp[i * (KT / 4)];
        const float2 xa = make_float2(x.x, x.y), xb = make_float2(x.z, x.w);
#pragma unroll
        for (int q2 = 0; q2 < NJ / 2; ++q2) {
            const float4 r = rb[i * rstep + q2];
            const float2 r0 = make_float2(r.x, r.y), r1 = make_float2(r.z, r.w);
            ya[2 * q2] = ffma2(xa, r0, ya[2 * q2]);
            yb[2 * q2] = ffma2(xb, r0, yb[2 * q2]);
            ya[2 * q2 + 1] = ffma2(xa, r1, ya[2 * q2 + 1]);
            yb[2 * q2 + 1] = ffma2(xb, r1, yb[2 * q2 + 1]);
        }
    }
#pragma unroll
    for (int q = 0; q < NJ; ++q) {
        const uint32_t j = j0 + q;
        const float4 c4 = jc[j];
        const float y[4] = {ya[q].x, ya[q].y, yb[q].x, yb[q].y};
        uint32_t word = 0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            float tv = (y[kk] - c4.x) * c4.y;
            tv = fminf(fmaxf(tv, 0.0f), 255.0f);
            word |= (uint32_t)lut_s[__float_as_uint(c4.z) + (uint32_t)tv] << (8 * kk);
        }
        reinterpret_cast<uint32_t *>(codes + j * KT)[lane] = word;
    }
}

template <int D>
__global__ void __launch_bounds__(kTileThreads, 2) encode_tile_kernel(const __grid_constant__ EncodeArgs a, uint32_t d,
                                                                      uint32_t cent_alloc, uint32_t lut_bytes,
                                                                      uint32_t rdup_pairs, uint32_t total) {
    constexpr int KT = kTileKeys, W = kTileWarps, SW = D / 2 + 1;
    const EncodeHead &h = a.head[blockIdx.y];
    const uint32_t row_words = h.row_stride / 4, ow = row_words | 1u;
    const uint32_t sc_words = h.scale_stride / 2, sw = sc_words + 1;
    const uint32_t ng = h.ng, ns = h.ns, count = a.count;
    const TileSmem<D> L = tile_smem<D>(rdup_pairs, cent_alloc, lut_bytes, h.row_stride, h.scale_stride);

    extern __shared__ __align__(16) unsigned char smem[];
    float2 *rdup = reinterpret_cast<float2 *>(smem + L.rdup);      // diagonal blocks, (R[j][i], R[j][i])
    float4 *jc = reinterpret_cast<float4 *>(smem + L.jc);          // [D]: off, inv, lut base, cent base
    float *cent_s = reinterpret_cast<float *>(smem + L.cent);
    float *X = reinterpret_cast<float *>(smem + L.x);              // [D][KT]
    float *nrm = reinterpret_cast<float *>(smem + L.nrm);          // [kMaxGroups][KT]
    uint32_t *stage_s = reinterpret_cast<uint32_t *>(smem + L.uni);  // [KT][SW] (phase 1 only)
    uint8_t *codes = smem + L.codes;                               // [D][KT]
    uint32_t *out_s = reinterpret_cast<uint32_t *>(smem + L.out);  // [KT][ow]
    uint32_t *sc_s = reinterpret_cast<uint32_t *>(smem + L.sc);    // [KT][sw]
    uint64_t *rsrc_s = reinterpret_cast<uint64_t *>(smem + L.rows), *rdst_s = rsrc_s + KT, *rsc_s = rdst_s + KT;
    uint8_t *lut_s = smem + L.lut;
    uint8_t *perm_s = smem + L.perm;
    uint2 *task_s = reinterpret_cast<uint2 *>(smem + L.task);      // [W][D/2]
    __shared__ uint32_t task_n[W];
    __shared__ uint2 pair_s[D / 2];   // per dim pair: j0 | group start << 8 | group end << 16, block base

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // ---- the head's tables, once per CTA ----
    for (uint32_t g = 0; g < ng; ++g) {
        const uint32_t lo = h.group_off[g], n = h.group_off[g + 1] - lo;
        uint32_t base = 0;
        for (uint32_t q = 0; q < g; ++q) base += (h.group_off[q + 1] - h.group_off[q]) * (h.group_off[q + 1] - h.group_off[q]);
        for (uint32_t e = tid; e < n * n; e += kTileThreads) {
            const uint32_t i = e / n, j = e % n;   // block element (i, j): R[lo + j][lo + i]
            const float r = h.t.rot[(lo + j) * d + lo + i];
            rdup[base + e] = make_float2(r, r);
        }
    }
    for (uint32_t j = tid; j < (uint32_t)D; j += kTileThreads) {
        const bool live = j < d;
        jc[j] = make_float4(live ? h.t.off[j] : 0.0f, live ? h.t.inv[j] : 0.0f,
                            __uint_as_float(live ? (uint32_t)h.t.cbidx[j] * 256u : 0u),
                            __uint_as_float(live ? (uint32_t)h.t.cb_base[j] : 0u));
        perm_s[j] = live ? h.t.perm[j] : (uint8_t)j;
    }
    for (uint32_t e = tid; e < cent_alloc; e += kTileThreads) cent_s[e] = e < h.n_cent ? h.t.cent[e] : 0.0f;
    for (uint32_t e = tid; e < lut_bytes; e += kTileThreads) lut_s[e] = e < h.ncb * 256u ? h.t.lut[e] : 0;
    // tasks: each group's dims in fours from its start, a last pair where the size leaves two;
    // word j0 | group start << 8 | group end << 16 | four dims << 24 | valid << 25, and the
    // group's rotation block offset; kept at the slot of the task's first dim pair
    constexpr uint32_t kQuad = 1u << 24, kValid = 1u << 25;
    for (uint32_t p = tid; p < (uint32_t)D / 2; p += kTileThreads) {
        uint2 w = make_uint2(0u, 0u);
        const uint32_t j0 = 2u * p;
        if (j0 < d) {
            const uint32_t g = h.t.group_of[j0], lo = h.group_off[g], hi = h.group_off[g + 1];
            uint32_t base = 0;
            for (uint32_t q = 0; q < g; ++q)
                base += (h.group_off[q + 1] - h.group_off[q]) * (h.group_off[q + 1] - h.group_off[q]);
            if ((j0 - lo) % 4 == 0) w = make_uint2(j0 | lo << 8 | hi << 16 | (j0 + 4 <= hi ? kQuad : 0u) | kValid, base);
        }
        pair_s[p] = w;
    }
    __syncthreads();
    if (tid == 0) {
        // longest-processing-time deal of the tasks to the warps; a task costs its group size
        // times its dim pairs
        uint32_t load[W];
        for (int w = 0; w < W; ++w) load[w] = 0, task_n[w] = 0;
        uint64_t taken = 0;
        for (;;) {
            int best = -1;
            uint32_t best_cost = 0;
            for (int p = 0; p < D / 2; ++p) {
                const uint32_t w = pair_s[p].x;
                if (((taken >> p) & 1u) || !(w & kValid)) continue;
                const uint32_t cost = (((w >> 16) & 0xffu) - ((w >> 8) & 0xffu)) * ((w & kQuad) ? 2u : 1u);
                if (best < 0 || cost > best_cost) best = p, best_cost = cost;
            }
            if (best < 0) break;
            int wmin = 0;
            for (int w = 1; w < W; ++w)
                if (load[w] < load[wmin]) wmin = w;
            taken |= 1ull << best;
            task_s[wmin * (D / 2) + task_n[wmin]++] = pair_s[best];
            load[wmin] += best_cost;
        }
    }
    const bool vec16 = !a.src_f32 && d == (uint32_t)D &&
                       (((uintptr_t)a.src | ((a.seq_stride | a.row_stride | h.src_head_offset) * 2u)) & 15u) == 0;
    const uint32_t rw_magic = row_words > 1 ? (uint32_t)((0x100000000ull + row_words - 1) / row_words) : 0u;
    const uint32_t sw_magic = sc_words > 1 ? (uint32_t)((0x100000000ull + sc_words - 1) / sc_words) : 0u;
    __syncthreads();

    const uint32_t n_tiles = (total + KT - 1) / KT;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const uint32_t first = tile * KT;
        const uint32_t nrows = min((uint32_t)KT, total - first);
        // ---- 0. per-key source and destination offsets ----
        if ((uint32_t)tid < nrows) {
            const uint32_t q = first + tid, s = q / count, rr = q % count;
            const uint64_t dseq = a.seq_first + s, dst_row = (a.row0 ? a.row0[s] : a.row0_scalar) + rr;
            rsrc_s[tid] = (uint64_t)s * a.seq_stride + (uint64_t)rr * a.row_stride + h.src_head_offset;
            rdst_s[tid] = dseq * h.k_seq_stride + dst_row * h.row_stride;
            rsc_s[tid] = dseq * h.s_seq_stride + dst_row * h.scale_stride;
        }
        __syncthreads();
        // ---- 1. input rows as FP16 words (coalesced), then X[i][k] through the permutation ----
        if (vec16) {
            for (uint32_t w = tid; w < nrows * (uint32_t)(D / 8); w += kTileThreads) {
                const uint32_t r = w / (D / 8), c = w % (D / 8);
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(a.src) + rsrc_s[r] + 8u * c));
                uint32_t *dst = stage_s + r * SW + 4u * c;
                dst[0] = v.x;
                dst[1] = v.y;
                dst[2] = v.z;
                dst[3] = v.w;
            }
        } else {
            for (uint32_t w = tid; w < nrows * (uint32_t)(D / 2); w += kTileThreads) {
                const uint32_t r = w / (D / 2), c = w % (D / 2);
                uint32_t word = 0;
                if (2u * c < d) {
                    const uint64_t e = rsrc_s[r] + 2u * c;
                    if (a.src_f32) {
                        const float *f = static_cast<const float *>(a.src) + e;
                        word = (uint32_t)__half_as_ushort(__float2half_rn(f[0])) |
                               ((uint32_t)__half_as_ushort(__float2half_rn(f[1])) << 16);
                    } else {
                        const uint16_t *p16 = static_cast<const uint16_t *>(a.src) + e;
                        word = (uint32_t)p16[0] | ((uint32_t)p16[1] << 16);
                    }
                }
                stage_s[r * SW + c] = word;
            }
        }
        __syncthreads();
        {
            // thread = key (lanes over keys: conflict-free, SW odd) x a quarter of the dims
            const uint32_t k = tid % KT, i0 = tid / KT;
            const __half *st = reinterpret_cast<const __half *>(stage_s + k * SW);
#pragma unroll 8
            for (uint32_t i = i0; i < (uint32_t)D; i += kTileThreads / KT) X[i * KT + k] = __half2float(st[perm_s[i]]);
        }
        __syncthreads();
        // ---- 2. group norms and normalisation, one thread per (key, group) ----
        for (uint32_t t = tid; t < KT * ng; t += kTileThreads) {
            const uint32_t k = t % KT, g = t / KT;
            const uint32_t lo = h.group_off[g], hi = h.group_off[g + 1];
            float acc = 0.0f;
            const float *xk = X + k;
#pragma unroll 4
            for (uint32_t i = lo; i < hi; ++i) {
                const float x = xk[i * KT];
                acc = fmaf(x, x, acc);
            }
            const float n = sqrtf(acc + 1e-30f);
            nrm[g * KT + k] = n;
            const float dv = n > 1e-10f ? n : 1.0f;
            if (!isinf(dv)) {
                // the IEEE quotient from one reciprocal per group (Markstein, IBM J. Res. Dev.
                // 34(1), 1990): with y = RN(1/dv) and q0 = RN(x y) within an ulp of x / dv,
                // the residual x - dv q0 is exact in one FMA and RN(q0 + r y) = RN(x / dv)
                // (no overflow or underflow here: |x| <= dv and x is FP16)
                const float y = __frcp_rn(dv);
#pragma unroll 4
                for (uint32_t i = lo; i < hi; ++i) {
                    const float x = X[i * KT + k], q0 = __fmul_rn(x, y);
                    X[i * KT + k] = __fmaf_rn(__fmaf_rn(-dv, q0, x), y, q0);
                }
            } else {
                for (uint32_t i = lo; i < hi; ++i) X[i * KT + k] = X[i * KT + k] / dv;
            }
        }
        __syncthreads();
        // ---- 3. rotation + codes: warp = 2 or 4 output dims of a group, lane = 4 keys ----
        {
            const uint32_t ntask = task_n[warp];
            for (uint32_t t = 0; t < ntask; ++t) {
                const uint2 task = task_s[warp * (D / 2) + t];
                const uint32_t j0 = task.x & 0xffu, lo = (task.x >> 8) & 0xffu, hi = (task.x >> 16) & 0xffu;
                if (task.x & (1u << 24)) rotate_codes<4>(rdup, X, jc, lut_s, codes, task.y, j0, lo, hi, lane);
                else rotate_codes<2>(rdup, X, jc, lut_s, codes, task.y, j0, lo, hi, lane);
            }
        }
        __syncthreads();
        // ---- 4. corrected scales and packed bytes, one thread per (key, group) ----
        for (uint32_t t = tid; t < KT * ng; t += kTileThreads) {
            const uint32_t k = t % KT, g = t / KT;
            const uint32_t lo = h.group_off[g], hi = h.group_off[g + 1];
            uint8_t *ob = reinterpret_cast<uint8_t *>(out_s + k * ow);
            float cl = 0.0f;
#pragma unroll 4
            for (uint32_t j = lo; j < hi; j += 2) {
                const uint32_t c0 = codes[j * KT + k], c1 = codes[(j + 1) * KT + k];
                const float v0 = cent_s[__float_as_uint(jc[j].w) + c0], v1 = cent_s[__float_as_uint(jc[j + 1].w) + c1];
                cl = fmaf(v0, v0, cl);
                cl = fmaf(v1, v1, cl);
                if (j < ns) {
                    ob[j >> 1] = (uint8_t)(c0 | (c1 << 4));
                } else {
                    ob[(ns >> 1) + (j - ns)] = (uint8_t)c0;
                    ob[(ns >> 1) + (j - ns) + 1] = (uint8_t)c1;
                }
            }
            reinterpret_cast<uint16_t *>(sc_s + k * sw)[g] =
                __half_as_ushort(__float2half_rn(nrm[g * KT + k] / fmaxf(sqrtf(cl), 1e-10f)));
        }
        // row padding and unused scale slots are zero
        for (uint32_t k = tid; k < KT; k += kTileThreads) {
            uint8_t *ob = reinterpret_cast<uint8_t *>(out_s + k * ow);
            for (uint32_t b = ns / 2 + (d - ns); b < row_words * 4; ++b) ob[b] = 0;
            uint16_t *sr = reinterpret_cast<uint16_t *>(sc_s + k * sw);
            for (uint32_t g = ng; g < sc_words * 2; ++g) sr[g] = 0;
        }
        __syncthreads();
        // ---- 5. rows and scales out (coalesced words) ----
        for (uint32_t w = tid; w < nrows * row_words; w += kTileThreads) {
            const uint32_t r = div_small(w, row_words, rw_magic), c = w - r * row_words;
            reinterpret_cast<uint32_t *>(h.packed + rdst_s[r])[c] = out_s[r * ow + c];
        }
        for (uint32_t w = tid; w < nrows * sc_words; w += kTileThreads) {
            const uint32_t r = div_small(w, sc_words, sw_magic), c = w - r * sc_words;
            reinterpret_cast<uint32_t *>(h.scales + rsc_s[r])[c] = sc_s[r * sw + c];
        }
        __syncthreads();
    }
    if (blockIdx.x == 0 && h.lengths) {
        for (uint32_t s = tid; s < a.seq_count; s += kTileThreads)
            h.lengths[a.seq_first + s] = (a.row0 ? a.row0[s] : a.row0_scalar) + count;
    }
}

// Few keys (a decode step appends one token per sequence): one warp per key, lanes over
// dimensions, so a launch of a few hundred keys spreads over many SMs instead of a couple
// of threads-per-key CTAs.
// stage_bytes != 0: the head's encode tables are staged in shared memory first, as in
// kv_rope_append_kernel.
__global__ void __launch_bounds__(kThreads) encode_warp_kernel(const __grid_constant__ EncodeArgs a, uint32_t d,
                                                               uint32_t total, uint32_t stage_bytes) {
    constexpr int W = kThreads / 32;
    extern __shared__ __align__(16) unsigned char tab_s[];
    __shared__ __align__(16) unsigned char hs_raw[sizeof(EncodeHead)];
    EncodeHead &hs = *reinterpret_cast<EncodeHead *>(hs_raw);
    __shared__ __align__(8) uint64_t stage_bar;
    if (stage_bytes) stage_head_tables(a.head[blockIdx.y], tab_s, hs, &stage_bar);
    const bool staged = stage_bytes && staged_tables_ready(&stage_bar, a.status);
    const EncodeHead &h = staged ? hs : a.head[blockIdx.y];
    __shared__ WarpKey wks[W];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t count = a.count;
    WarpKey &wk = wks[w];
    for (uint32_t q = blockIdx.x * W + w; q < total; q += gridDim.x * W) {
        const uint32_t s = q / count, rr = q % count;
        const uint64_t e0 = (uint64_t)s * a.seq_stride + (uint64_t)rr * a.row_stride + h.src_head_offset;
        for (uint32_t i = lane; i < d; i += 32) {
            const uint64_t e = e0 + h.t.perm[i];
            const __half x = a.src_f32 ? __float2half_rn(static_cast<const float *>(a.src)[e])
                                       : __ushort_as_half(static_cast<const uint16_t *>(a.src)[e]);
            wk.xs[i] = __half2float(x);
        }
        const uint32_t dst_row = (a.row0 ? a.row0[s] : a.row0_scalar) + rr;
        if (staged) warp_encode<true>(h, d, wk, a.seq_first + s, dst_row, lane);
        else warp_encode<false>(h, d, wk, a.seq_first + s, dst_row, lane);
    }
    if (stage_bytes) staged_tables_drain(&stage_bar, staged);
    if (blockIdx.x == 0 && h.lengths) {
        for (uint32_t s = threadIdx.x; s < a.seq_count; s += kThreads)
            h.lengths[a.seq_first + s] = (a.row0 ? a.row0[s] : a.row0_scalar) + count;
    }
}

// K/V append of one layer for every KV head in one launch.  One warp per (new token, KV
// head) reads the token's K and V (FP16 or FP32), optionally applies split-half RoPE to K at
// the token's cache row (the model path, src/model/decoder.ts:44-50 and
// src/model/kernels.wgsl:49-54, rounded like separate multiplies and adds), encodes K into
// the packed store (FP16-rounded first, as every append is) and writes V to the FP16 value
// store.  Start rows come from the first key store's device lengths, so the launch is
// stream-ordered against earlier appends without host round trips; the last CTA to finish
// bumps the lengths.

//
// stage_bytes != 0: every head's encode tables (rotation, codebooks, offsets, inverse scales,
// code LUT, permutation, group and codebook indices: the leading part of its table blob, up to
// the attention lookup) fit in stage_bytes of dynamic shared memory.  Each CTA copies its
// head's part once with 16-byte loads and encodes from shared memory, so a key's dependent
// table lookups cost shared-memory latency instead of one L2 round trip each.  The arithmetic
// and its order are the same either way.
__global__ void __launch_bounds__(kThreads) kv_rope_append_kernel(const __grid_constant__ KvRopeArgs a, uint32_t d,
                                                                  uint32_t total, uint32_t stage_bytes) {
    constexpr int W = kThreads / 32;
    const uint32_t hd = blockIdx.y;
    __shared__ WarpKey wks[W];
    __shared__ float kr[W][kMaxDim];
    extern __shared__ __align__(16) unsigned char tab_s[];
    __shared__ __align__(16) unsigned char hs_raw[sizeof(EncodeHead)];
    EncodeHead &hs = *reinterpret_cast<EncodeHead *>(hs_raw);
    __shared__ __align__(8) uint64_t stage_bar;
    // the tables are the store's own (never written by other kernels): their copy starts
    // while the kernel before this one finishes (programmatic launch)
    if (stage_bytes) stage_head_tables(a.head[hd], tab_s, hs, &stage_bar);
    pdl_wait();
    pdl_trigger();
    const bool staged = stage_bytes && staged_tables_ready(&stage_bar, a.status);
    const EncodeHead &h = staged ? hs : a.head[hd];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    WarpKey &wk = wks[w];
    const uint32_t pairs = d / 2;
    for (uint32_t q = blockIdx.x * W + w; q < total; q += gridDim.x * W) {
        const uint32_t s = q / a.count, rr = q % a.count, seq = a.seq_first + s;
        const uint64_t at = (uint64_t)s * a.seq_stride + (uint64_t)rr * a.row_stride + (uint64_t)hd * d;
        // the lane's K and V source elements (lane + 32 u), fetched in the same round trip as
        // the row position
        float kx[kMaxDim / 32], vx[kMaxDim / 32];
#pragma unroll
        for (uint32_t u = 0; u < (uint32_t)kMaxDim / 32; ++u) {
            const uint32_t e = lane + 32u * u;
            kx[u] = e < d ? src_elem(a.k_src, at + e, a.k_f16) : 0.0f;
            vx[u] = e < d ? src_elem(a.v_src, at + e, a.v_f16) : 0.0f;
        }
        const uint32_t pos = a.start[seq] + rr;
        if (pos >= a.capacity) {  // replayed past the capacity the host checked: refuse, report
            if (lane == 0) atomicOr(a.status, kStatusBadLength);
            continue;
        }
#pragma unroll
        for (uint32_t u = 0; u < (uint32_t)kMaxDim / 32; ++u)
            if (lane + 32u * u < d) kr[w][lane + 32u * u] = kx[u];
        __syncwarp();
        if (a.rope) {
            for (uint32_t p = lane; p < pairs; p += 32) {
                const float ang = __fmul_rn((float)pos, a.inv_freq[p]);
                const float c = cosf(ang), sn = sinf(ang);
                const float x = kr[w][p], y = kr[w][p + pairs];
                kr[w][p] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn));
                kr[w][p + pairs] = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
            }
            __syncwarp();
        }
        for (uint32_t i = lane; i < d; i += 32) wk.xs[i] = __half2float(__float2half_rn(kr[w][h.t.perm[i]]));
        if (staged) warp_encode<true>(h, d, wk, seq, pos, lane);
        else warp_encode<false>(h, d, wk, seq, pos, lane);
        // V row: FP32 -> FP16, chunk-swizzled for head dims 64 / 128
        __half *vrow = reinterpret_cast<__half *>(a.v[hd]) + (uint64_t)seq * a.v_seq_stride[hd] + (uint64_t)pos * a.vD;
#pragma unroll
        for (uint32_t u = 0; u < (uint32_t)kMaxDim / 32; ++u) {
            const uint32_t e = lane + 32u * u;
            if (e >= a.vD) break;
            const float x = vx[u];  // zero past the head dim
            uint32_t de = e;
            if (a.v_swizzle) {
                const uint32_t c = e >> 3;
                de = (((c & ~7u) | ((c ^ pos) & 7u)) << 3) | (e & 7u);
            }
            vrow[de] = __float2half_rn(x);
        }
    }
    if (stage_bytes) staged_tables_drain(&stage_bar, staged);
    // The last CTA to finish moves every store's lengths on.  Each CTA read its start rows
    // before taking a ticket, so none reads a bumped length; the ticket is left at zero for
    // the next launch (or graph replay).
    __shared__ uint32_t s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(a.ticket, 1u) == gridDim.x * gridDim.y - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        // independent (sequence, head) updates, unrolled so their loads overlap
#pragma unroll 8
        for (uint32_t idx = threadIdx.x; idx < a.seq_count * a.heads; idx += blockDim.x) {
            const uint32_t s = a.seq_first + idx / a.heads, hh = idx % a.heads;
            const uint32_t kl = a.head[hh].lengths[s], vl = a.v_lengths[hh][s];
            a.head[hh].lengths[s] = min(kl + a.count, a.capacity);
            a.v_lengths[hh][s] = min(vl + a.count, a.capacity);
        }
        if (threadIdx.x == 0) *a.ticket = 0u;
    }
}

template <int D>
size_t encode_smem(uint32_t cent_alloc, uint32_t lut_bytes, uint32_t row_stride, uint32_t scale_stride) {
    const size_t ow = (row_stride / 4) | 1u, sw = scale_stride / 2 + 1;
    size_t b = sizeof(float) * ((size_t)D * D + cent_alloc + 2 * D + kMaxGroups * kThreads);
    b += sizeof(uint32_t) * (size_t)kThreads * ((D / 2 + 1) + ow + sw);
    b += sizeof(uint16_t) * D + lut_bytes + 4 * D;
    return (b + 15) & ~(size_t)15;
}

template <int D>
cudaError_t run_encode(const EncodeArgs &a, uint32_t d, uint32_t cent_alloc, uint32_t max_ncb, cudaStream_t s) {
    uint32_t row_stride = 0, scale_stride = 0;
    for (uint32_t h = 0; h < a.heads; ++h) {
        row_stride = row_stride > a.head[h].row_stride ? row_stride : a.head[h].row_stride;
        scale_stride = scale_stride > a.head[h].scale_stride ? scale_stride : a.head[h].scale_stride;
    }
    const uint32_t lut_bytes = (max_ncb * 256u + 15u) & ~15u;
    const size_t smem = encode_smem<D>(cent_alloc, lut_bytes, row_stride, scale_stride);
    int dev = 0, sms = 0, max_optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (smem > (size_t)max_optin) return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(encode_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, encode_kernel<D>, kThreads, smem);
    if (per_sm < 1) per_sm = 1;
    const uint32_t total = a.count * a.seq_count;
    const uint32_t tiles = (total + kThreads - 1) / kThreads;
    uint32_t grid_x = (uint32_t)(sms * per_sm) / (a.heads ? a.heads : 1);
    if (grid_x < 1) grid_x = 1;
    if (grid_x > tiles) grid_x = tiles;
    dim3 grid(grid_x, a.heads);
    encode_kernel<D><<<grid, kThreads, smem, s>>>(a, d, cent_alloc, lut_bytes, total);
    return cudaGetLastError();
}

template <int D>
cudaError_t run_encode_tile(const EncodeArgs &a, uint32_t d, uint32_t cent_alloc, uint32_t max_ncb, cudaStream_t s) {
    uint32_t row_stride = 0, scale_stride = 0, rdup_pairs = 0;
    for (uint32_t h = 0; h < a.heads; ++h) {
        const EncodeHead &e = a.head[h];
        row_stride = row_stride > e.row_stride ? row_stride : e.row_stride;
        scale_stride = scale_stride > e.scale_stride ? scale_stride : e.scale_stride;
        uint32_t pairs = 0;
        for (uint32_t g = 0; g < e.ng; ++g) pairs += (e.group_off[g + 1] - e.group_off[g]) * (e.group_off[g + 1] - e.group_off[g]);
        rdup_pairs = rdup_pairs > pairs ? rdup_pairs : pairs;
    }
    const uint32_t lut_bytes = (max_ncb * 256u + 15u) & ~15u;
    const uint32_t smem = tile_smem<D>(rdup_pairs, cent_alloc, lut_bytes, row_stride, scale_stride).total;
    int dev = 0, sms = 0, max_optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (smem > (uint32_t)max_optin) return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(encode_tile_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, encode_tile_kernel<D>, kTileThreads, smem);
    if (per_sm < 1) per_sm = 1;
    const uint32_t total = a.count * a.seq_count;
    const uint32_t tiles = (total + kTileKeys - 1) / kTileKeys;
    uint32_t grid_x = (uint32_t)(sms * per_sm) / (a.heads ? a.heads : 1);
    if (grid_x < 1) grid_x = 1;
    if (grid_x > tiles) grid_x = tiles;
    encode_tile_kernel<D><<<dim3(grid_x, a.heads), kTileThreads, smem, s>>>(a, d, cent_alloc, lut_bytes, rdup_pairs,
                                                                            total);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_kv_rope_append(const KvRopeArgs &a, uint32_t d, cudaStream_t s) {
    const uint32_t total = a.count * a.seq_count;
    if (!total) return cudaSuccess;
    const uint32_t blocks = (total + kThreads / 32 - 1) / (kThreads / 32);
    const uint32_t stage = encode_stage_bytes(a.head, a.heads);
    return launch_pdl(kv_rope_append_kernel, dim3(blocks, a.heads), dim3(kThreads), stage, s, a, d, total, stage);
}

cudaError_t launch_encode(const EncodeArgs &a, uint32_t d, uint32_t cent_alloc, uint32_t max_ncb, cudaStream_t s) {
    if (a.count == 0 || a.seq_count == 0) return cudaSuccess;
    const uint32_t total = a.count * a.seq_count;
    if (total <= kWarpKeysMax) {
        // a warp per key: at most 4 keys per CTA, so even one sequence's token uses a CTA
        // and a decode step of a few hundred sequences spreads over the SMs
        const uint32_t blocks = (total + kThreads / 32 - 1) / (kThreads / 32);
        const uint32_t stage = encode_stage_bytes(a.head, a.heads);
        encode_warp_kernel<<<dim3(blocks, a.heads), kThreads, stage, s>>>(a, d, total, stage);
        return cudaGetLastError();
    }
    if (d <= 16) return run_encode_tile<16>(a, d, cent_alloc, max_ncb, s);
    if (d <= 32) return run_encode_tile<32>(a, d, cent_alloc, max_ncb, s);
    if (d <= 64) return run_encode_tile<64>(a, d, cent_alloc, max_ncb, s);
    return run_encode<128>(a, d, cent_alloc, max_ncb, s);
}

}  // namespace bgtq
