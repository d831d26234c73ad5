// Flash-decoding attention over the Block-GTQ key cache (sm_100a).
//
// Replaces the reference's three-pass WGSL attention - fused packed-K dot
// (src/attention/fused-dot.wgsl:15-37), parallel softmax and weighted sum
// (src/attention/parallel-tail.wgsl:10-33), the model's compressed_dot / softmax /
// weighted kernels (src/model/compressed-dot.wgsl:14-31, src/model/attention.wgsl:13-39)
// and the baseline FP16/FP32-K passes (src/attention/attention.wgsl:17-43) - with a query
// rotation kernel plus one attention kernel per (split, KV head, sequence) with a last-CTA
// split combine.  Semantics follow src/reference/attention.py:5-22: logits = q.k/sqrt(d),
// positions t > pos masked when causal, softmax, P.V, FP32 accumulation.
//
// Packed keys are never reconstructed.  The query is rotated once into the code domain,
//   qt_i = sum_{j in group(i)} R[i][j] q[perm[j]] / sqrt(d),
// so that q.k = sum_g s_g sum_{i in g} qt_i cent[i][code_i] (k = reconstruct(codes) of
// src/reference/production_math.py:27-31, R block-diagonal as PackedKeys enforces).
//
// Data movement: each warp owns two shared-memory K tiles (packed rows + FP16 scales) and
// one V tile, filled by cp.async.bulk (TMA bulk copies, no multicast) that complete on
// mbarriers.  The next K tile is fetched while the current one is computed; the next V tile
// is fetched right after the current P.V and lands during the next dequant + QK, so one V
// buffer suffices and three CTAs fit on an SM.  Every mbarrier wait is bounded and reports
// a timeout through the device status word instead of spinning forever.  Tiles are always
// copied whole: capacity is padded to 64 rows and zero-filled, and tokens past the end of
// a split get probability 0.
//
// Compute:
//   dequant + QK   lane = token.  Packed rows sit in shared memory at an odd word stride,
//                  so the 32 lanes reading word w of their rows hit 32 banks.  The nibble
//                  region is walked in runs of 4 dimension pairs (one 32-bit code word),
//                  the byte region in runs of 4 pairs (two words), group by group, with the
//                  group's FP16 scale applied once at its end; per-pair query records and
//                  codebook offsets come from small shared tables built per (sequence,
//                  head).
//   softmax        online, in log2 units, with per-lane running sums (reduced once at the
//                  end) and a lazily moved maximum: a warp vote skips the warp-wide max and
//                  the rescale of O unless a score exceeds the running maximum by 2^3.
//   P.V            tensor cores (mma.sync m16n8k16, FP16 in, FP32 accumulate) for FP16 V of
//                  64/128 dims: P is scaled by 2^12 and split into high and low FP16 parts
//                  (about 22 significant bits).  Up to 4 query rows compute O^T = V^T P^T
//                  with the parts in B columns 0-3 and 4-7 (16 dims per MMA); up to 8 rows
//                  put them in A rows 0-7 and 8-15 (8 dims per MMA).  V tiles arrive
//                  chunk-swizzled from the value
//                  store so ldmatrix reads them without bank conflicts.  FP32 V and small
//                  head dims use FP32 FMAs with lane = 16-byte slice of V.
#pragma once

#include <cuda_fp16.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace attn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
constexpr uint32_t kWaitLimit = 1u << 22;
// Scores are kept in log2 units (the query records carry log2(e)/sqrt(d)), and
// probabilities are scaled by 2^kPShift so that their FP16 high/low split for the P.V MMA
// keeps about 22 significant bits; the running sums carry the same factor, which cancels
// in O / l and is taken out of the log-sum-exp.
constexpr float kPShift = 12.0f;
// Lazy rescaling: the running maximum moves only when a score exceeds it by more than
// kLazy (log2 units), so probabilities stay below 2^(kPShift + kLazy) = 32768, inside FP16.
constexpr float kLazy = 3.0f;

template <int D>
struct Geo {
    static constexpr int TPL = D <= 64 ? 2 : 1;  // tokens per lane in the lane=token phase
    static constexpr int TT = 32 * TPL;          // tokens per warp tile
};
template <int QM>
struct QPad {
    static constexpr int QP = QM <= 1 ? 1 : QM <= 2 ? 2 : QM <= 4 ? 4 : 8;
};
// Shared tables of the packed path: one record per dimension pair, laid out group by group,
// each group padded with zero records to a whole number of 4-pair blocks.  A record holds,
// for each query row r, the pair's rotated query values (q_2b,r, q_2b+1,r) as a float2, then
// the absolute shared-memory byte offsets of the two dimensions' codebooks; RP words,
// padded to 16 bytes.
template <int D, int QM>
struct RecGeo {
    static constexpr int RP = (2 * QM + 2 + 3) & ~3;         // words per pair record
    static constexpr int NP = D / 2 + 3 * kMaxGroups;        // pair records incl. padding
    static constexpr int BYTES = (NP * RP * 4 + 15) & ~15;
};

template <int D, bool VF32>
struct UseMma {
    static constexpr bool value = !VF32 && (D == 64 || D == 128);
};

// Group structure of the packed keys.  RuntimeGroups reads it from the head at run time; a
// kernel specialised for one layout (compiled at run time, jit.cpp) supplies a policy with
// kStatic = true and the layout as constants (kNG groups, kNS nibble dims, group offsets
// go(g) as a constexpr function, which folds where an array might be placed in memory), so
// every group and run loop unrolls.
struct RuntimeGroups {
    static constexpr bool kStatic = false;
    static constexpr uint32_t kNG = 0, kNS = 0;
    static __host__ __device__ constexpr uint32_t go(uint32_t) { return 0; }
};

// Shared-memory plan of one CTA.  Each warp owns a V tile buffer and a ring of `stages`
// K tile buffers (packed rows + FP16 scales, or dense rows): the next tile's keys are
// fetched while the current tile is computed, and the next tile's values are fetched as
// soon as the current P.V is done, behind the next tile's dequant + QK.
struct Plan {
    uint32_t cent, qrec, stage, pbuf, bars, total;
    uint32_t kbytes, sbytes, vbytes, kstage_bytes, warp_bytes, cent_alloc;
    uint32_t stages;  // K buffers per warp: 2, or 1 when two do not fit
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }
__host__ __device__ inline uint32_t align128(uint32_t x) { return (x + 127u) & ~127u; }

#ifndef __CUDACC_RTC__
inline Plan make_plan(KKind kk, int v_f32, uint32_t D, uint32_t QP, uint32_t TT, uint32_t row_stride,
                      uint32_t scale_stride, uint32_t n_cent, uint32_t smem_limit = 227u * 1024u,
                      uint32_t stages = 2, uint32_t QM = 0) {
    Plan p{};
    p.stages = stages;
    uint32_t off = 0;
    // the lookup table first: its slots' byte offsets must keep their 256-byte (nibble runs)
    // and size (byte dims) alignment; the 256 zero floats after it cover any code byte of
    // a padding record
    p.cent = off;
    p.cent_alloc = kk == KKind::Packed ? n_cent + 256u : 0u;
    off = align16(off + 4u * p.cent_alloc);
    p.qrec = off;  // dense: [D][QP] query records; packed: RecGeo tables
    const uint32_t rp = (2u * (QM ? QM : QP) + 2u + 3u) & ~3u;
    const uint32_t rec_bytes = kk == KKind::Packed ? align16((D / 2u + 3u * kMaxGroups) * rp * 4u) : 4u * D * QP;
    off = align16(off + rec_bytes);
    p.kbytes = TT * row_stride;
    p.sbytes = kk == KKind::Packed ? TT * scale_stride * 2u : 0u;
    p.vbytes = TT * D * (v_f32 ? 4u : 2u);
    // 16 spare bytes after the K rows: the code-word reads of the last row run past its end
    p.kstage_bytes = align128(align16(p.kbytes) + 16u + align16(p.sbytes));
    p.warp_bytes = align128(p.vbytes) + stages * p.kstage_bytes;
    off = align128(off);
    p.stage = off;
    off += kWarps * p.warp_bytes;
    p.pbuf = off;
    off = align16(off + kWarps * (TT + 8u) * (QM ? QM : QP) * 4u);
    p.bars = off;
    off += kWarps * 4u * 8u;  // per warp: K barriers 0, 1 and the V barrier
    p.total = align16(off);
    if (p.total > smem_limit && stages == 2)
        return make_plan(kk, v_f32, D, QP, TT, row_stride, scale_stride, n_cent, smem_limit, 1, QM);
    return p;
}
#endif  // __CUDACC_RTC__

// ---- PTX helpers: mbarrier + bulk async copies (sm_90+, no multicast), tensor cores ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// Loads at 32-bit byte offsets into the kernel's dynamic shared memory (plain C++ loads,
// so the compiler keeps them ordered after barrier waits but may schedule them freely).
__device__ __forceinline__ uint32_t lds_u32(const unsigned char *sm, uint32_t off) {
    return *reinterpret_cast<const uint32_t *>(sm + off);
}
__device__ __forceinline__ float lds_f32(const unsigned char *sm, uint32_t off) {
    return *reinterpret_cast<const float *>(sm + off);
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// C (16x8, f32) += A (16x16, f16) * B (16x8, f16); fragments as in the PTX ISA for
// mma.m16n8k16 (row g = lane/4, column pair 2*(lane%4)).
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x on the special-function unit (PTX ex2.approx.ftz: relative error below 2^-22,
// 2^-inf = +0, results below 2^-126 flushed to 0, which is far below any probability that
// matters here).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed FP32 FMA (two lanes, round to nearest) in PTX, so kernels built by nvcc and by
// NVRTC (whose headers declare the intrinsic differently) get the same instruction.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xffffu))); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

template <int QP>
__device__ __forceinline__ void load_q(const float *p, float (&q)[QP]) {
    if constexpr (QP == 1) {
        q[0] = p[0];
    } else if constexpr (QP == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        q[0] = v.x; q[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < QP; i += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(p + i);
            q[i] = v.x; q[i + 1] = v.y; q[i + 2] = v.z; q[i + 3] = v.w;
        }
    }
}

// Build the packed-path pair records for one (sequence, head) from the query records qt
// [D][QP] and the head's lookup-layout offsets: group g's pairs [off_g/2, off_{g+1}/2)
// padded to 4*ceil(pairs/4) records; padding records carry zero query values (their
// lookups stay inside the table and its zero tail, so whatever code bytes they meet
// contribute exactly 0).
template <int D, int QM, int QP>
// qt_generic: qt may be shared memory (plain loads; __ldg is for global memory only).
// lko_s: the head's lookup offsets in shared memory, or null (read from the table blob).
__device__ __forceinline__ void build_tables(const AttnHead &h, const float *qt, unsigned char *rec, uint32_t d,
                                             uint32_t cent_off, int tid, bool qt_generic = false,
                                             const uint16_t *lko_s = nullptr) {
    auto qload = [&](const float *p) { return qt_generic ? *p : __ldg(p); };
    using G = RecGeo<D, QM>;
    uint32_t *recs = reinterpret_cast<uint32_t *>(rec);
    // records of all groups (each padded to a multiple of 4) flattened over the threads, so
    // a thread's loads are independent of one another (one round trip, not one per group)
    uint32_t total = 0;
    for (uint32_t g = 0; g < h.ng; ++g) total += ((h.group_off[g + 1] / 2 - h.group_off[g] / 2 + 3) / 4) * 4;
    for (uint32_t rix = tid; rix < total; rix += kThreads) {
        uint32_t g = 0, base = 0, p0 = 0, p1 = 0;
        for (;; ++g) {
            p0 = h.group_off[g] / 2;
            p1 = h.group_off[g + 1] / 2;
            const uint32_t n = ((p1 - p0 + 3) / 4) * 4;
            if (rix < base + n) break;
            base += n;
        }
        uint32_t *rp = recs + rix * G::RP;
        const uint32_t pr = p0 + (rix - base), j0 = 2 * pr;
        const bool live = pr < p1;
        for (int r = 0; r < QM; ++r) {
            rp[2 * r] = __float_as_uint(live ? qload(qt + j0 * QP + r) : 0.0f);
            rp[2 * r + 1] = __float_as_uint(live ? qload(qt + (j0 + 1) * QP + r) : 0.0f);
        }
        const uint32_t ja = min(j0, d - 1u), jb = min(j0 + 1, d - 1u);
        rp[2 * QM] = cent_off + 4u * (lko_s ? lko_s[ja] : __ldg(h.lookup_off + ja));
        rp[2 * QM + 1] = cent_off + 4u * (lko_s ? lko_s[jb] : __ldg(h.lookup_off + jb));
        for (int x = 2 * QM + 2; x < G::RP; ++x) rp[x] = 0u;
    }
}

// Dequantise + QK for the TPL tokens of this lane (see the file comment).  Groups are
// walked in order; inside a group, straight-line blocks of 4 dimension pairs (no branches)
// accumulate each pair into a float2 (even, odd dims) with one packed FMA per query row,
// and the group's FP16 scale is applied once at the group's end.  Codebooks sit in the
// lookup layout (layout.cpp, build_lookup_layout), so a lookup address is one instruction
// from the code word: a nibble lookup is a byte permute of (code * 4, run slot address) plus
// a constant offset, a byte lookup an OR (or shifted add) of code * 4 into the dimension's
// size-aligned slot address from the pair record.  Code bytes are read as (unaligned)
// words: a nibble block needs 4 bytes, a byte block 8.
template <int D, int QM, class LP>
__device__ __forceinline__ void packed_qk(const AttnHead &h, const unsigned char *sm, uint32_t kb_s,
                                          const uint16_t *sb, const unsigned char *rec, uint32_t cb_s, int lane,
                                          float (&acc)[Geo<D>::TPL][QM]) {
    using G = RecGeo<D, QM>;
    constexpr int TPL = Geo<D>::TPL, RP = G::RP;
    const uint32_t *recs = reinterpret_cast<const uint32_t *>(rec);
    const uint32_t krow = h.row_stride, ns = h.ns;
    uint32_t row[TPL];
    uint32_t sw[TPL][4];
    float2 part[TPL][QM], acc2[TPL][QM];
#pragma unroll
    for (int tt = 0; tt < TPL; ++tt) {
        const int tl = tt * 32 + lane;
        row[tt] = kb_s + (uint32_t)tl * krow;
        if (h.scale_stride == 4) {
            const uint2 v = *reinterpret_cast<const uint2 *>(sb + (size_t)tl * 4);
            sw[tt][0] = v.x; sw[tt][1] = v.y; sw[tt][2] = 0u; sw[tt][3] = 0u;
        } else {
            const uint4 v = *reinterpret_cast<const uint4 *>(sb + (size_t)tl * 8);
            sw[tt][0] = v.x; sw[tt][1] = v.y; sw[tt][2] = v.z; sw[tt][3] = v.w;
        }
#pragma unroll
        for (int r = 0; r < QM; ++r) { acc2[tt][r] = make_float2(0.0f, 0.0f); part[tt][r] = make_float2(0.0f, 0.0f); }
    }
    // one dimension pair: the record's query values against the two codebook entries of each
    // token at byte addresses ia + OA, ib + OB
    auto pair = [&](const uint32_t *rp, const uint32_t (&ia)[TPL], const uint32_t (&ib)[TPL], uint32_t OA,
                    uint32_t OB) {
        uint32_t v[RP];
#pragma unroll
        for (int x = 0; x < RP; x += 4) {
            const uint4 t = *reinterpret_cast<const uint4 *>(rp + x);
            v[x] = t.x; v[x + 1] = t.y; v[x + 2] = t.z; v[x + 3] = t.w;
        }
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
            const float2 c = make_float2(lds_f32(sm, ia[tt] + OA), lds_f32(sm, ib[tt] + OB));
#pragma unroll
            for (int r = 0; r < QM; ++r)
                part[tt][r] = ffma2(make_float2(__uint_as_float(v[2 * r]), __uint_as_float(v[2 * r + 1])), c,
                                         part[tt][r]);
        }
    };
    // a run of cnt <= 4 pairs starting at pair record rp0 whose codes start at byte a of the
    // row (nibble run: pair b = byte b; byte run: pair b = bytes 2b, 2b+1).  slot: the nibble
    // run's 256-byte aligned lookup slot.
    auto nib_run = [&](uint32_t a, const uint32_t *rp0, uint32_t cnt, uint32_t slot) {
        const uint32_t al = a & ~3u, sh = (a & 3u) * 8u;
        uint32_t lo4[TPL], hi4[TPL];
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
            const uint32_t word = __funnelshift_r(lds_u32(sm, row[tt] + al), lds_u32(sm, row[tt] + al + 4), sh);
            lo4[tt] = (word << 2) & 0x3c3c3c3cu;   // even dims: low nibble x 4 per byte
            hi4[tt] = (word >> 2) & 0x3c3c3c3cu;   // odd dims: high nibble x 4 per byte
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            if ((uint32_t)p < cnt) {
                uint32_t ia[TPL], ib[TPL];
#pragma unroll
                for (int tt = 0; tt < TPL; ++tt) {
                    ia[tt] = __byte_perm(lo4[tt], slot, 0x7650u | p);  // slot + code * 4
                    ib[tt] = __byte_perm(hi4[tt], slot, 0x7650u | p);
                }
                pair(rp0 + p * RP, ia, ib, 64u * p, 256u + 64u * p);
            }
        }
    };
    auto byte_run = [&](uint32_t a, const uint32_t *rp0, uint32_t cnt) {
        const uint32_t al = a & ~3u, sh = (a & 3u) * 8u;
        uint32_t x4[TPL][4];
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
            const uint32_t w0 = lds_u32(sm, row[tt] + al), w1 = lds_u32(sm, row[tt] + al + 4),
                           w2 = lds_u32(sm, row[tt] + al + 8);
            const uint32_t x = __funnelshift_r(w0, w1, sh), y = __funnelshift_r(w1, w2, sh);
            x4[tt][0] = (x << 2) & 0x03fc03fcu;   // bytes 0, 2 of x (x 4)
            x4[tt][1] = (x >> 6) & 0x03fc03fcu;   // bytes 1, 3 of x
            x4[tt][2] = (y << 2) & 0x03fc03fcu;
            x4[tt][3] = (y >> 6) & 0x03fc03fcu;
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            if ((uint32_t)p < cnt) {
                const uint32_t *rp = rp0 + p * RP;
                const uint2 base = *reinterpret_cast<const uint2 *>(rp + 2 * QM);
                uint32_t ia[TPL], ib[TPL];
#pragma unroll
                for (int tt = 0; tt < TPL; ++tt) {
                    const uint32_t e = x4[tt][(p >> 1) * 2], o = x4[tt][(p >> 1) * 2 + 1];
                    // slots are aligned to their size: OR / add of code * 4 is the address
                    ia[tt] = (p & 1) ? base.x + (e >> 16) : base.x | (e & 0xffffu);
                    ib[tt] = (p & 1) ? base.y + (o >> 16) : base.y | (o & 0xffffu);
                }
                pair(rp, ia, ib, 0u, 0u);
            }
        }
    };
    // one group: its runs of four pairs, then the group-end scale step
    uint32_t rix = 0;  // first record of the current group
    auto group = [&](uint32_t g, uint32_t go, uint32_t gnext, uint32_t nsv, bool unrolled) {
        const uint32_t p0 = go / 2, np = gnext / 2 - p0;
        const uint32_t nfull = np / 4, rem = np & 3u;
        const uint32_t *rg = recs + rix * RP;
        if (go < nsv) {
            // run b of the head owns lookup slot b (512 bytes); the group's first run is rix / 4
            const uint32_t slot0 = cb_s + (rix >> 2) * 512u;
            if (unrolled) {
#pragma unroll
                for (uint32_t k = 0; k < nfull; ++k) nib_run(p0 + 4 * k, rg + 4 * k * RP, 4, slot0 + k * 512u);
            } else {
#pragma unroll 1
                for (uint32_t k = 0; k < nfull; ++k) nib_run(p0 + 4 * k, rg + 4 * k * RP, 4, slot0 + k * 512u);
            }
            if (rem) nib_run(p0 + 4 * nfull, rg + 4 * nfull * RP, rem, slot0 + nfull * 512u);
        } else {
            // byte group: dim 2*p0 sits at byte ns/2 + (2*p0 - ns)
            const uint32_t ob = 2 * p0 - nsv / 2;
            if (unrolled) {
#pragma unroll
                for (uint32_t k = 0; k < nfull; ++k) byte_run(ob + 8 * k, rg + 4 * k * RP, 4);
            } else {
#pragma unroll 1
                for (uint32_t k = 0; k < nfull; ++k) byte_run(ob + 8 * k, rg + 4 * k * RP, 4);
            }
            if (rem) byte_run(ob + 8 * nfull, rg + 4 * nfull * RP, rem);
        }
        const uint32_t nblk = nfull + (rem ? 1u : 0u);
        rix += 4 * nblk;
        // group end.  part holds the running (unscaled) sum over all groups so far, C_g;
        // sum_g s_g (C_g - C_{g-1}) = sum_g (s_g - s_{g+1}) C_g with s past the last group
        // = 0 (the scale rows are zero-padded), so no per-group reset is needed.
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
            float ds;
            if constexpr (LP::kStatic) {
                // g is a constant here: read s_g and s_{g+1} from their fixed halves
                const uint32_t w0 = sw[tt][(g >> 1) & 3u], w1 = g + 1 < 8u ? sw[tt][((g + 1) >> 1) & 3u] : 0u;
                ds = half_lo(w0 >> (16u * (g & 1u))) - half_lo(w1 >> (16u * ((g + 1) & 1u)));
            } else {
                ds = half_lo(sw[tt][0]) - half_lo(sw[tt][0] >> 16);
            }
            const float2 ds2 = make_float2(ds, ds);
#pragma unroll
            for (int r = 0; r < QM; ++r) acc2[tt][r] = ffma2(ds2, part[tt][r], acc2[tt][r]);
            if constexpr (!LP::kStatic) {
                sw[tt][0] = __funnelshift_r(sw[tt][0], sw[tt][1], 16);
                sw[tt][1] = __funnelshift_r(sw[tt][1], sw[tt][2], 16);
                sw[tt][2] = __funnelshift_r(sw[tt][2], sw[tt][3], 16);
                sw[tt][3] >>= 16;
            }
        }
    };
    if constexpr (LP::kStatic) {
#pragma unroll
        for (uint32_t g = 0; g < LP::kNG; ++g) group(g, LP::go(g), LP::go(g + 1), LP::kNS, true);
    } else {
#pragma unroll 1
        for (uint32_t g = 0; g < h.ng; ++g) group(g, h.group_off[g], h.group_off[g + 1], ns, false);
    }
#pragma unroll
    for (int tt = 0; tt < TPL; ++tt)
#pragma unroll
        for (int r = 0; r < QM; ++r) acc[tt][r] = acc2[tt][r].x + acc2[tt][r].y;
}

// Minimum resident CTAs per SM the register allocation must allow: the packed kernels of
// head dims up to 64 fit three CTAs in shared memory, and giving the compiler the
// registers of exactly three (up to 168 per thread) schedules the lookup loads deeper.
template <int D, int QM, KKind KK>
struct MinBlocks {
    static constexpr int value = (KK == KKind::Packed && D <= 64 && QM <= 4) ? 3 : 1;
};

// The head's codebook lookup table into shared memory with 16-byte loads, four in flight
// per thread (the table is 16-byte aligned in its blob), zero past its end: a few KB per CTA
// that a scalar loop would fetch one L2 round trip at a time.
__device__ __forceinline__ void stage_lookup(const AttnHead &h, const Plan &pl, float *cent_s, int tid) {
    const uint32_t n4 = pl.cent_alloc / 4u, nl = h.n_lookup;
    const float4 *src = reinterpret_cast<const float4 *>(h.lookup);
    float4 *dst = reinterpret_cast<float4 *>(cent_s);
#pragma unroll 4
    for (uint32_t q = tid; q < n4; q += kThreads) {
        float4 v;
        if (4u * q + 3u < nl) {
            v = __ldg(src + q);
        } else {
            v.x = 4u * q < nl ? h.lookup[4u * q] : 0.0f;
            v.y = 4u * q + 1u < nl ? h.lookup[4u * q + 1u] : 0.0f;
            v.z = 4u * q + 2u < nl ? h.lookup[4u * q + 2u] : 0.0f;
            v.w = 0.0f;
        }
        dst[q] = v;
    }
    for (uint32_t i = 4u * n4 + tid; i < pl.cent_alloc; i += kThreads) cent_s[i] = i < nl ? h.lookup[i] : 0.0f;
}

// A caller's work between the first tile copies and the query tables (NoPrologue: none).
struct NoPrologue {
    __device__ __forceinline__ void operator()() const {}
};

// One (sequence s, KV head hd) key range [t_lo, t_hi) into partial slot `slot` of nslots.
// A persistent caller may pass: len_known, the sequence's key length when it knows it (0:
// read the device length), lko_s, the head's lookup offsets in shared memory, and pro, work
// of its own that runs once this range's first tile copies are in flight and before the
// query tables are built (its query records, say), ending with a CTA barrier.
template <int D, int QM, KKind KK, bool VF32, class LP, class Pro = NoPrologue>
__device__ __forceinline__ void attn_pair(const AttnArgs &a, const Plan &pl, uint32_t d, uint32_t hd, uint32_t s,
                                          uint32_t t_lo, uint32_t t_hi, uint32_t slot, uint32_t nslots,
                                          uint32_t &phase, uint32_t &staged_hd, const float *qt_src = nullptr,
                                          bool defer_merge = false, uint32_t len_known = 0u,
                                          const uint16_t *lko_s = nullptr, const Pro &pro = Pro{}) {
    constexpr int TPL = Geo<D>::TPL, TT = Geo<D>::TT, QP = QPad<QM>::QP;
    constexpr bool MMA = UseMma<D, VF32>::value;
    constexpr int VSZ = VF32 ? 4 : 2, VEC = 16 / VSZ, LPT = D / VEC, TPS = 32 / LPT;
    static_assert(LPT >= 1 && LPT <= 32, "V slice layout");
    constexpr int KSZ = KK == KKind::F32 ? 4 : 2, KVEC = 16 / KSZ, LPTK = D / KVEC, TPSK = 32 / LPTK;
    static_assert(KK == KKind::Packed || (LPTK >= 1 && LPTK <= 32), "K slice layout");
    constexpr int NT = D / 8;  // MMA n-tiles (8 dims each)
    // Up to 4 query rows: P.V as O^T = V^T P^T, V^T in the 16-row A operand (16 dims per
    // tile) and P^T in the 8 B columns (high parts of rows 0-3 in columns 0-3, low parts in
    // 4-7): half the MMAs and accumulators of the P-as-A form, which up to 8 rows use.
    constexpr bool TMMA = MMA && QM <= 4;

    const AttnHead &h = a.head[hd];
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *rec = smem + pl.qrec;
    // the pair's query records: the query rotation's output, or the caller's copy (qt_src)
    const float *qt = qt_src ? qt_src : a.qt + ((uint64_t)s * a.heads + hd) * (uint64_t)(D * QP);
    auto query_tables = [&]() {
        if constexpr (KK == KKind::Packed) {
            build_tables<D, QM, QP>(h, qt, rec, d, pl.cent, tid, qt_src != nullptr, lko_s);
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(qt);
            float4 *dst = reinterpret_cast<float4 *>(rec);
            for (uint32_t i = tid; i < (uint32_t)(D * QP / 4); i += kThreads) dst[i] = qt_src ? src[i] : __ldg(src + i);
        }
    };
    const uint32_t seq = a.seq_first + s;
    // L2: a persistent caller's lengths change between phases
    const uint32_t len = len_known ? len_known : __ldcg(a.lengths + seq);
    const uint32_t R = a.rows;

    float *qrec_s = reinterpret_cast<float *>(rec);
    // P rows of TT floats at a stride of TT + 8: the P.V operand loads of four rows fall in
    // different banks
    constexpr int PS = TT + 8;
    float *pbuf = reinterpret_cast<float *>(smem + pl.pbuf) + w * PS * QM;  // [QM][PS]
    const uint32_t bar0 = smem_u32(smem + pl.bars) + (uint32_t)w * 32u, vbar = bar0 + 16u;
    __shared__ uint32_t s_last;

    uint32_t pos[QM];
    uint32_t tend = 0;
#pragma unroll
    for (int r = 0; r < QM; ++r) {
        uint32_t p = len ? len - 1 : 0;
        if (a.positions && (uint32_t)r < R) p = a.positions[s * R + r];
        pos[r] = p;
        if ((uint32_t)r < R) {
            const uint32_t e = a.causal ? min(p + 1, len) : len;
            tend = max(tend, e);
        }
    }
    if (a.logits) tend = len;
    uint32_t pmin = 0xffffffffu;
#pragma unroll
    for (int r = 0; r < QM; ++r)
        if ((uint32_t)r < R) pmin = min(pmin, pos[r]);
    const uint32_t t0 = t_lo;
    const uint32_t t1 = min(t_hi, tend);

    const uint32_t ntok = t1 > t0 ? t1 - t0 : 0u;
    const uint32_t ntiles = (ntok + TT - 1) / TT;
    unsigned char *vbuf = smem + pl.stage + (size_t)w * pl.warp_bytes;
    unsigned char *kstage0 = vbuf + align128(pl.vbytes);
    const bool two = pl.stages == 2;
    const unsigned char *kbase = h.k + (uint64_t)seq * h.k_seq_stride;
    const unsigned char *sbase =
        KK == KKind::Packed ? reinterpret_cast<const unsigned char *>(h.scales + (uint64_t)seq * h.s_seq_stride) : nullptr;
    const unsigned char *vbase = static_cast<const unsigned char *>(h.v) + (uint64_t)seq * h.v_seq_stride;
    const uint32_t krow = h.row_stride, vrow = D * VSZ, srow = h.scale_stride * 2u;
    const uint32_t soff = align16(pl.kbytes) + 16u;

    // whole tiles: rows past the sequence end exist (capacity padded to 64, zero filled)
    uint32_t pending = 0;  // bit st: K buffer st has a copy in flight; bit 2: the V buffer
    // this head's tile sizes: the plan's buffers fit the widest head of the launch
    const uint32_t kb_h = (uint32_t)TT * krow, sb_h = KK == KKind::Packed ? (uint32_t)TT * srow : 0u;
    auto issue_k = [&](uint32_t k, int st) {
        if (lane == 0) {
            const uint32_t at = t0 + k * TT;
            unsigned char *buf = kstage0 + (size_t)st * pl.kstage_bytes;
            const uint32_t bar = bar0 + (uint32_t)st * 8u;
            fence_proxy_async();
            mbar_expect_tx(bar, kb_h + sb_h);
            bulk_g2s(smem_u32(buf), kbase + (uint64_t)at * krow, kb_h, bar);
            if (KK == KKind::Packed) bulk_g2s(smem_u32(buf + soff), sbase + (uint64_t)at * srow, sb_h, bar);
        }
        pending |= 1u << st;
    };
    auto issue_v = [&](uint32_t k) {
        if (lane == 0) {
            fence_proxy_async();
            mbar_expect_tx(vbar, pl.vbytes);
            bulk_g2s(smem_u32(vbuf), vbase + (uint64_t)(t0 + k * TT) * vrow, pl.vbytes, vbar);
        }
        pending |= 4u;
    };

    bool ok = true;
    // phase (the caller's, carried across the pairs of one CTA): bit st = parity of K buffer
    // st; bit 2 = parity of the V buffer.  The first tiles are requested before the query
    // tables are built: the copies' latency overlaps the prologue.
    if ((uint32_t)w < ntiles) {
        issue_k(w, 0);
        issue_v(w);
    }
    if (KK == KKind::Packed && hd != staged_hd) {  // a later pair of another head
        __syncthreads();
        stage_lookup(h, pl, reinterpret_cast<float *>(smem + pl.cent), tid);
        staged_hd = hd;
    }
    pro();

    // ---- prologue: query tables ----
    query_tables();
    __syncthreads();

    // ---- per-warp flash-decoding over this range ----
    float m[QM], l[QM];
#pragma unroll
    for (int r = 0; r < QM; ++r) { m[r] = -INFINITY; l[r] = 0.0f; }
    constexpr int OS = TMMA ? (D / 16) * 4 : MMA ? NT * 4 : QM * VEC;  // output accumulators per lane
    float O[OS];
#pragma unroll
    for (int i = 0; i < OS; ++i) O[i] = 0.0f;
    float qreg[QM][KVEC];
    if constexpr (KK != KKind::Packed) {
        const int dl = (lane % LPTK) * KVEC;
#pragma unroll
        for (int r = 0; r < QM; ++r)
#pragma unroll
            for (int e = 0; e < KVEC; ++e) qreg[r][e] = qrec_s[(dl + e) * QP + r];
    }
    int it = 0;
    for (uint32_t k = w; k < ntiles; k += kWarps, ++it) {
        const int st = two ? (it & 1) : 0;
        const bool more = k + kWarps < ntiles;
        if (two && more) issue_k(k + kWarps, st ^ 1);
        if (!mbar_wait_bounded(bar0 + (uint32_t)st * 8u, (phase >> st) & 1u)) {
            ok = false;
            break;
        }
        phase ^= 1u << st;
        pending &= ~(1u << st);
        const uint32_t at = t0 + k * TT, n = min((uint32_t)TT, t1 - at);
        const unsigned char *kb = kstage0 + (size_t)st * pl.kstage_bytes;
        const uint16_t *sb = reinterpret_cast<const uint16_t *>(kb + soff);
        const unsigned char *vb = vbuf;

        // ---- logits for this lane's TPL tokens ----
        float acc[TPL][QM];
        if constexpr (KK == KKind::Packed) {
            packed_qk<D, QM, LP>(h, smem, (uint32_t)(kb - smem), sb, rec, pl.cent, lane, acc);
        } else {
            const uint32_t steps = (n + TPSK - 1) / TPSK;
            for (uint32_t st2 = 0; st2 < steps; ++st2) {
                const uint32_t tl = st2 * TPSK + lane / LPTK;
                float kv[KVEC];
                if (tl < n) {
                    const uint4 raw = *reinterpret_cast<const uint4 *>(kb + (size_t)tl * D * KSZ + (lane % LPTK) * 16);
                    if constexpr (KSZ == 2) {
                        const __half2 *hp = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(hp[e]);
                            kv[2 * e] = f.x; kv[2 * e + 1] = f.y;
                        }
                    } else {
                        kv[0] = __uint_as_float(raw.x); kv[1] = __uint_as_float(raw.y);
                        kv[2] = __uint_as_float(raw.z); kv[3] = __uint_as_float(raw.w);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < KVEC; ++e) kv[e] = 0.0f;
                }
#pragma unroll
                for (int r = 0; r < QM; ++r) {
                    float sum = 0.0f;
#pragma unroll
                    for (int e = 0; e < KVEC; ++e) sum = fmaf(qreg[r][e], kv[e], sum);
#pragma unroll
                    for (int o = 1; o < LPTK; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                    if ((lane % LPTK) == 0 && tl < n) pbuf[r * PS + tl] = sum;
                }
            }
            __syncwarp();
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const uint32_t tl = tt * 32 + lane;
#pragma unroll
                for (int r = 0; r < QM; ++r) acc[tt][r] = tl < n ? pbuf[r * PS + tl] : 0.0f;
            }
            __syncwarp();
        }

        // ---- masking, optional raw-logit capture, online softmax ----
        // A tile wholly inside the split and, when causal, at or before every row's position
        // needs no per-token mask.
        const bool full = n == (uint32_t)TT && (!a.causal || at + (uint32_t)TT - 1u <= pmin);
        float alpha[QM];
        bool rescale = false;
#pragma unroll
        for (int r = 0; r < QM; ++r) {
            const bool live = (uint32_t)r < R;
            float lg[TPL];
            bool up = false;
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const uint32_t tl = tt * 32 + lane, tok = at + tl;
                const bool valid = live && (full || (tl < n && (!a.causal || tok <= pos[r])));
                lg[tt] = valid ? acc[tt][r] : -INFINITY;
                up |= lg[tt] > m[r] + kLazy;
            }
            if (a.logits && live) {
#pragma unroll
                for (int tt = 0; tt < TPL; ++tt) {
                    const uint32_t tl = tt * 32 + lane, tok = at + tl;
                    if (tl < n) a.logits[(((uint64_t)s * a.heads + hd) * R + r) * a.logit_stride + tok] = lg[tt] * kLn2;
                }
            }
            alpha[r] = 1.0f;
            if (__any_sync(0xffffffffu, up)) {
                float tm = lg[0];
#pragma unroll
                for (int tt = 1; tt < TPL; ++tt) tm = fmaxf(tm, lg[tt]);
                const float mnew = fmaxf(m[r], warp_max(tm));
                alpha[r] = ex2(m[r] - mnew);  // 0 on the first live tile: l and O are still 0
                m[r] = mnew;
                rescale = true;
            }
            // no live score yet keeps m at -inf and every score at -inf: 2^(-inf - 0) = 0
            const float mref = m[r] == -INFINITY ? 0.0f : m[r] - kPShift;
            float ps = 0.0f;
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const float p = ex2(lg[tt] - mref);
                pbuf[r * PS + tt * 32 + lane] = p;
                ps += p;
            }
            l[r] = fmaf(l[r], alpha[r], ps);  // this lane's share; summed over lanes at the end
        }
        __syncwarp();
        if (!two && more) issue_k(k + kWarps, 0);
        if (!mbar_wait_bounded(vbar, (phase >> 2) & 1u)) {
            ok = false;
            break;
        }
        phase ^= 4u;
        pending &= ~4u;

        // ---- P.V ----
        if constexpr (TMMA) {
            // C fragment: row g / g + 8 = dim (16 per tile), column pair 2c / 2c + 1 = P column;
            // column j holds the high (j < 4) or low (j >= 4) part of query row j & 3
            const int g = lane >> 2, c = lane & 3;
            if (rescale) {
                // columns 2c, 2c + 1 hold rows 0, 1 (c even) or 2, 3 (c odd)
                float al[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) al[r] = r < QM ? alpha[r < QM ? r : 0] : 1.0f;
                const bool odd = c & 1;
                const float a0 = odd ? al[2] : al[0], a1 = odd ? al[3] : al[1];
#pragma unroll
                for (int i = 0; i < OS; i += 2) { O[i] *= a0; O[i + 1] *= a1; }
            }
            const uint32_t vb_s = smem_u32(vb);
            const int mi = lane >> 3, ri = lane & 7;
            const int qg = g & 3;
            const bool lo_col = g >= 4, live_col = qg < QM;
#pragma unroll
            for (int kb16 = 0; kb16 < TT / 16; ++kb16) {
                float2 pa = make_float2(0.0f, 0.0f), pb = make_float2(0.0f, 0.0f);
                if (live_col) {
                    pa = *reinterpret_cast<const float2 *>(pbuf + qg * PS + kb16 * 16 + 2 * c);
                    pb = *reinterpret_cast<const float2 *>(pbuf + qg * PS + kb16 * 16 + 2 * c + 8);
                }
                const __half2 ha = __floats2half2_rn(pa.x, pa.y), hb = __floats2half2_rn(pb.x, pb.y);
                const float2 fa = __half22float2(ha), fb = __half22float2(hb);
                const float2 m1 = make_float2(-1.0f, -1.0f);
                const float2 ra = ffma2(fa, m1, pa), rb = ffma2(fb, m1, pb);  // exact p - hi
                const __half2 la = __floats2half2_rn(ra.x, ra.y), lb = __floats2half2_rn(rb.x, rb.y);
                const uint32_t b0 = lo_col ? h2_bits(la) : h2_bits(ha), b1 = lo_col ? h2_bits(lb) : h2_bits(hb);
                // ldmatrix (transposed) row address of this lane: matrix mi = tokens +8*(mi>>1),
                // dims +8*(mi&1) of the 16-dim tile; row ri
                const uint32_t tok = (uint32_t)(kb16 * 16 + (mi >> 1) * 8 + ri);
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    const uint32_t chunk = (uint32_t)(2 * mt + (mi & 1));
                    const uint32_t pos_c = (chunk & ~7u) | ((chunk ^ tok) & 7u);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_trans(vb_s + tok * (D * 2) + pos_c * 16, a0, a1, a2, a3);
                    mma_16816(*reinterpret_cast<float(*)[4]>(&O[mt * 4]), a0, a1, a2, a3, b0, b1);
                }
            }
        } else if constexpr (MMA) {
            // fragment row g = query (high part of P), row g + 8 = the same query (low part);
            // column pair 2c/2c+1 (+8) = token (A) or dim (C)
            const int g = lane >> 2, c = lane & 3;
            if (rescale) {
                float ag = 1.0f;
#pragma unroll
                for (int r = 0; r < QM; ++r) ag = g == r ? alpha[r] : ag;
#pragma unroll
                for (int i = 0; i < NT * 4; ++i) O[i] *= ag;
            }
            const uint32_t vb_s = smem_u32(vb);
            const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
            for (int kb16 = 0; kb16 < TT / 16; ++kb16) {
                float2 pa = make_float2(0.0f, 0.0f), pb = make_float2(0.0f, 0.0f);
                if (g < QM) {
                    pa = *reinterpret_cast<const float2 *>(pbuf + g * PS + kb16 * 16 + 2 * c);
                    pb = *reinterpret_cast<const float2 *>(pbuf + g * PS + kb16 * 16 + 2 * c + 8);
                }
                const __half2 ha = __floats2half2_rn(pa.x, pa.y), hb = __floats2half2_rn(pb.x, pb.y);
                const float2 fa = __half22float2(ha), fb = __half22float2(hb);
                const float2 m1 = make_float2(-1.0f, -1.0f);
                const float2 ra = ffma2(fa, m1, pa), rb = ffma2(fb, m1, pb);  // exact p - hi
                const __half2 la = __floats2half2_rn(ra.x, ra.y), lb = __floats2half2_rn(rb.x, rb.y);
                const uint32_t ahi0 = h2_bits(ha), ahi2 = h2_bits(hb), alo0 = h2_bits(la), alo2 = h2_bits(lb);
                // ldmatrix row address of this lane: matrix mi (tokens +8*(mi&1), chunk +(mi>>1)), row ri
                const uint32_t tok = (uint32_t)(kb16 * 16 + (mi & 1) * 8 + ri);
#pragma unroll
                for (int np = 0; np < NT / 2; ++np) {
                    const uint32_t chunk = (uint32_t)(2 * np + (mi >> 1));
                    const uint32_t pos_c = (chunk & ~7u) | ((chunk ^ tok) & 7u);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_trans(vb_s + tok * (D * 2) + pos_c * 16, b0, b1, b2, b3);
                    float(&c0)[4] = *reinterpret_cast<float(*)[4]>(&O[(2 * np) * 4]);
                    float(&c1)[4] = *reinterpret_cast<float(*)[4]>(&O[(2 * np + 1) * 4]);
                    mma_16816(c0, ahi0, alo0, ahi2, alo2, b0, b1);
                    mma_16816(c1, ahi0, alo0, ahi2, alo2, b2, b3);
                }
            }
        } else {
            if (rescale) {
#pragma unroll
                for (int r = 0; r < QM; ++r)
#pragma unroll
                    for (int e = 0; e < VEC; ++e) O[r * VEC + e] *= alpha[r];
            }
            const int slot = lane / LPT, dl = (lane % LPT) * VEC;
            const uint32_t steps = (n + TPS - 1) / TPS;
#pragma unroll 4
            for (uint32_t st2 = 0; st2 < steps; ++st2) {
                const uint32_t tl = st2 * TPS + slot;
                if (tl < n) {
                    float vv[VEC];
                    const uint4 raw = *reinterpret_cast<const uint4 *>(vb + (size_t)tl * vrow + dl * VSZ);
                    if constexpr (VSZ == 2) {
                        const __half2 *hp = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(hp[e]);
                            vv[2 * e] = f.x; vv[2 * e + 1] = f.y;
                        }
                    } else {
                        vv[0] = __uint_as_float(raw.x); vv[1] = __uint_as_float(raw.y);
                        vv[2] = __uint_as_float(raw.z); vv[3] = __uint_as_float(raw.w);
                    }
#pragma unroll
                    for (int r = 0; r < QM; ++r) {
                        const float p = pbuf[r * PS + tl];
#pragma unroll
                        for (int e = 0; e < VEC; ++e) O[r * VEC + e] = fmaf(p, vv[e], O[r * VEC + e]);
                    }
                }
            }
        }
        __syncwarp();
        if (more) issue_v(k + kWarps);
    }
    if (!ok) {
        // report the timeout, then give the copies still in flight a bounded chance to land
        // before this shared memory is reused or released (a drained barrier moves on a phase,
        // as the next pair of a stream-K CTA expects)
        if (lane == 0) atomicOr(a.status, kStatusWaitTimeout);
        for (int b = 0; b < 3; ++b)
            if ((pending & (1u << b)) && mbar_wait_bounded(bar0 + (b == 2 ? 16u : 8u * b), (phase >> b) & 1u))
                phase ^= 1u << b;
    }

    // ---- merge the warps of this CTA ----
#pragma unroll
    for (int r = 0; r < QM; ++r) l[r] = warp_sum(l[r]);
    if constexpr (!MMA) {
#pragma unroll
        for (int i = 0; i < OS; ++i)
#pragma unroll
            for (int o = LPT; o < 32; o <<= 1) O[i] += __shfl_xor_sync(0xffffffffu, O[i], o);
    }
    __syncthreads();
    float *mO = reinterpret_cast<float *>(smem + pl.stage);  // [kWarps][QP][D]
    float *mm = mO + kWarps * QP * D;                        // [kWarps][QP]
    float *ml = mm + kWarps * QP;
    if constexpr (TMMA) {
        // add each low column into its high column (lane ^ 2 holds columns 2c ^ 4, 2c+1 ^ 4)
#pragma unroll
        for (int i = 0; i < OS; ++i) O[i] += __shfl_xor_sync(0xffffffffu, O[i], 2);
        const int g = lane >> 2, c = lane & 3;
        if (c < 2) {
            const int q0 = 2 * c, q1 = 2 * c + 1;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
                if (q0 < QM) {
                    mO[(w * QP + q0) * D + mt * 16 + g] = O[mt * 4 + 0];
                    mO[(w * QP + q0) * D + mt * 16 + g + 8] = O[mt * 4 + 2];
                }
                if (q1 < QM) {
                    mO[(w * QP + q1) * D + mt * 16 + g] = O[mt * 4 + 1];
                    mO[(w * QP + q1) * D + mt * 16 + g + 8] = O[mt * 4 + 3];
                }
            }
        }
    } else if constexpr (MMA) {
        const int g = lane >> 2, c = lane & 3;
        if (g < QM) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                mO[(w * QP + g) * D + nt * 8 + 2 * c] = O[nt * 4 + 0] + O[nt * 4 + 2];
                mO[(w * QP + g) * D + nt * 8 + 2 * c + 1] = O[nt * 4 + 1] + O[nt * 4 + 3];
            }
        }
    } else {
        if (lane < LPT) {
#pragma unroll
            for (int r = 0; r < QM; ++r)
#pragma unroll
                for (int e = 0; e < VEC; ++e) mO[(w * QP + r) * D + (lane % LPT) * VEC + e] = O[r * VEC + e];
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < QM; ++r) { mm[w * QP + r] = m[r]; ml[w * QP + r] = l[r]; }
    }
    __syncthreads();
    const uint32_t rows_live = min(R, (uint32_t)QM);
    const uint64_t obase = ((uint64_t)s * a.heads + hd) * R;
    for (uint32_t idx = tid; idx < rows_live * d; idx += kThreads) {
        const uint32_t r = idx / d, dd = idx % d;
        float M = -INFINITY;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) M = fmaxf(M, mm[ww * QP + r]);
        float L = 0.0f, Ov = 0.0f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) {
            const float mw = mm[ww * QP + r];
            const float f = mw == -INFINITY ? 0.0f : ex2(mw - M);
            L = fmaf(ml[ww * QP + r], f, L);
            Ov = fmaf(mO[(ww * QP + r) * D + dd], f, Ov);
        }
        if (nslots == 1) {
            a.out[(obase + r) * d + dd] = Ov / L;
            if (dd == 0 && a.lse) a.lse[obase + r] = (M + log2f(L) - kPShift) * kLn2;
        } else {
            float *pp = a.part + ((((uint64_t)slot * a.seq_count + s) * a.heads + hd) * R + r) * (uint64_t)(d + 2);
            pp[dd] = Ov;
            if (dd == 0) { pp[d] = M; pp[d + 1] = L; }
        }
    }
    // defer_merge: the caller merges the partials itself after a grid-wide barrier
    if (nslots > 1 && !defer_merge) {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t ticket = atomicAdd(&a.counters[s * a.heads + hd], 1u);
            s_last = ticket == nslots - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            const uint64_t sstride = (uint64_t)a.seq_count * a.heads * R * (d + 2);
            const float *pbase = a.part + ((uint64_t)s * a.heads + hd) * R * (uint64_t)(d + 2);
            // every slot's (maximum, sum) of every row in one round of independent loads, the
            // per-row maximum, weights and sum from shared memory, then the weighted outputs
            // eight slots of loads at a time: the same arithmetic in the same order as a
            // per-element pass over the slots, without one L2 round trip per slot
            float *ms = reinterpret_cast<float *>(smem + pl.stage);  // [nslots][QP] maxima, then weights
            float *ls = ms + nslots * QP;                             // [nslots][QP] sums
            float *rs = ls + nslots * QP;                             // [QP] (maximum, sum) per row
            for (uint32_t idx = tid; idx < rows_live * nslots; idx += kThreads) {
                const uint32_t r = idx / nslots, sp = idx % nslots;
                const float *pp = pbase + (uint64_t)r * (d + 2) + sp * sstride;
                ms[sp * QP + r] = __ldcg(pp + d);
                ls[sp * QP + r] = __ldcg(pp + d + 1);
            }
            __syncthreads();
            if ((uint32_t)tid < rows_live) {
                const uint32_t r = tid;
                float M = -INFINITY;
                for (uint32_t sp = 0; sp < nslots; ++sp) M = fmaxf(M, ms[sp * QP + r]);
                float L = 0.0f;
                for (uint32_t sp = 0; sp < nslots; ++sp) {
                    const float m = ms[sp * QP + r];
                    const float f = m == -INFINITY ? 0.0f : ex2(m - M);
                    L = fmaf(ls[sp * QP + r], f, L);
                    ms[sp * QP + r] = f;
                }
                rs[2 * r] = M;
                rs[2 * r + 1] = L;
            }
            __syncthreads();
            for (uint32_t idx = tid; idx < rows_live * d; idx += kThreads) {
                const uint32_t r = idx / d, dd = idx % d;
                const float *pp = pbase + (uint64_t)r * (d + 2) + dd;
                float Ov = 0.0f;
                for (uint32_t sp0 = 0; sp0 < nslots; sp0 += 8) {
                    float v[8];
#pragma unroll
                    for (uint32_t k = 0; k < 8; ++k) v[k] = sp0 + k < nslots ? __ldcg(pp + (sp0 + k) * sstride) : 0.0f;
#pragma unroll
                    for (uint32_t k = 0; k < 8; ++k)
                        if (sp0 + k < nslots) Ov = fmaf(v[k], ms[(sp0 + k) * QP + r], Ov);
                }
                const float M = rs[2 * r], L = rs[2 * r + 1];
                a.out[(obase + r) * d + dd] = Ov / L;
                if (dd == 0 && a.lse) a.lse[obase + r] = (M + log2f(L) - kPShift) * kLn2;
            }
            if (tid == 0) a.counters[s * a.heads + hd] = 0u;
        }
    }
    __syncthreads();  // the merge scratch and tile buffers are free for the next pair
}

// Element j of query row q after split-half RoPE at position pos (src/model/kernels.wgsl:
// 49-54) with the table inv[d/2], rounded like separate multiplies and adds; without a
// table the element itself.
__device__ __forceinline__ float rope_elem(const float *q, uint32_t j, uint32_t d, uint32_t pos, const float *inv) {
    if (!inv) return q[j];
    const uint32_t pairs = d / 2, p = j < pairs ? j : j - pairs;
    const float ang = __fmul_rn((float)pos, inv[p]);
    const float c = cosf(ang), sn = sinf(ang), x = q[p], y = q[p + pairs];
    return j < pairs ? __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn)) : __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
}

// The CTA's own query records for (sequence s, KV head hd), with the query rotation
// kernel's arithmetic (qrot_kernel, below): for launches of one partial wave, where a
// separate rotation launch on the critical path costs more than every CTA rotating its
// pair's few query rows.  rot_s: the head's rotation already in shared memory (head dims
// up to 64), transposed: R[j][i] at rot_t[i * (D + 1) + j], so lanes over consecutive j
// read 32 banks (the padded row stride; rows 64 floats apart would share one); pg_s: its
// permutation [D] then group of each dim [D], in shared memory too; qraw: R * d floats of
// scratch; qt: [D][QP] output, shared memory, which first holds the raw query rows (read in
// the same round trip as the length).  Every output is one ascending FMA chain over its
// group, as in qrot_kernel.  Returns the sequence's key length.
template <int D, int QP>
__device__ __forceinline__ uint32_t own_query_records(const AttnArgs &a, uint32_t d, uint32_t hd, uint32_t s,
                                                      const float *rot_t, const uint8_t *pg_s, float *qraw,
                                                      float *qt) {
    const AttnHead &h = a.head[hd];
    const uint32_t R = a.rows, tid = threadIdx.x;
    const float *qg = a.q + ((uint64_t)s * a.heads + hd) * (uint64_t)R * d;
    const uint32_t len = __ldcg(a.lengths + a.seq_first + s);
    for (uint32_t idx = tid; idx < R * d; idx += kThreads) qt[idx] = __ldcg(qg + idx);
    __syncthreads();
    for (uint32_t idx = tid; idx < R * d; idx += kThreads) {
        const uint32_t r = idx / d, i = idx % d;
        const uint32_t pos = a.positions ? a.positions[s * R + r] : (len ? len - 1 : 0);
        qraw[idx] = rope_elem(qt + r * d, pg_s[i], d, pos, a.rope);
    }
    __syncthreads();
    const float qscale = kLog2e / sqrtf((float)d);
    for (uint32_t idx = tid; idx < (uint32_t)(D * QP); idx += kThreads) {
        const uint32_t j = idx % D, r = idx / D;
        float v = 0.0f;
        if (r < R && j < d) {
            const uint32_t g = pg_s[D + j], lo = h.group_off[g], hi = h.group_off[g + 1];
            for (uint32_t i = lo; i < hi; ++i) v = fmaf(rot_t[i * (D + 1) + j], qraw[r * d + i], v);
            v *= qscale;
        }
        qt[j * QP + r] = v;
    }
    __syncthreads();
    return len;
}

// One CTA of the decode attention.  Split-KV (a.sk_units == 0): the CTA owns split `split`
// of the pair (sequence s, KV head hd).  Stream-K (a.sk_units CTAs): the pairs' token tiles
// (a.sk_pair_tiles of kWarps * TT tokens per pair, pairs in head-major order) are dealt to
// the CTAs as equal contiguous ranges of a.sk_tiles, so one wave of CTAs covers the whole
// launch with the same work each; a range crossing pairs runs one segment per pair, and the
// segments of a pair are merged like splits by the last to finish.
template <int D, int QM, KKind KK, bool VF32, class LP>
__device__ __forceinline__ void attn_body(const AttnArgs &a, const Plan &pl, uint32_t d, uint32_t split, uint32_t hd,
                                          uint32_t s) {
    constexpr int TT = Geo<D>::TT;
    constexpr uint32_t CT = kWarps * TT;  // tokens per tile of the whole CTA
    const int tid = threadIdx.x;
    extern __shared__ __align__(128) unsigned char smem[];
    const uint32_t P = a.heads * a.seq_count, nt = a.sk_pair_tiles, K = a.sk_tiles;
    const uint64_t g0 = (uint64_t)split * K, total = (uint64_t)P * nt;
    if (a.sk_units && g0 < total) {
        const uint32_t p0 = (uint32_t)(g0 / nt);
        hd = p0 / a.seq_count;
        s = p0 % a.seq_count;
    }
    // the codebooks are the store's own tables: staged while the kernel before this one (the
    // query rotation) finishes; lengths, query records and cache rows only after the wait
    if constexpr (KK == KKind::Packed) stage_lookup(a.head[hd], pl, reinterpret_cast<float *>(smem + pl.cent), tid);
    // a.fuse_q: this CTA rotates its pair's queries itself (no rotation launch before it);
    // the rotation, a table of the store, comes into the tile buffers before the wait
    constexpr int QP = QPad<QM>::QP;
    const bool fq = KK == KKind::Packed && a.fuse_q && !a.sk_units;
    float *rot_s = reinterpret_cast<float *>(smem + pl.stage);  // transposed, rows of D + 1 floats
    // with it the permutation and group of each dim (after the raw query scratch), and the
    // lookup offsets after the query records in the P buffers (the query tables read them
    // once the first tile copies have taken over the tile buffers)
    float *qraw_s = rot_s + D * (D + 1);
    uint8_t *pg_s = reinterpret_cast<uint8_t *>(qraw_s + kMaxRows * D);
    float *qt_s = reinterpret_cast<float *>(smem + pl.pbuf);
    uint16_t *lko_s = reinterpret_cast<uint16_t *>(qt_s + D * QP);
    if (fq) {
        const AttnHead &fh = a.head[hd];
#pragma unroll 8
        for (uint32_t e = tid; e < d * d; e += kThreads) rot_s[(e % d) * (D + 1) + e / d] = __ldg(fh.rot + e);
        for (uint32_t i = tid; i < d; i += kThreads) {
            pg_s[i] = fh.perm[i];
            pg_s[D + i] = fh.group_of[i];
            lko_s[i] = fh.lookup_off[i];
        }
    }
    pdl_wait();
    // the kernel after this one may launch once every CTA of this grid has started: it then
    // takes only the slots this grid's last wave frees, fetches its constant tables and waits
    pdl_trigger();
    if (tid < kWarps * 4) mbar_init(smem_u32(smem + pl.bars) + tid * 8u, 1u);
    fence_barrier_init();
    __syncthreads();
    uint32_t phase = 0, staged_hd = hd;
    if (!a.sk_units) {
        // fused rotation: query records into the P buffers (free until the tile loop), rotated
        // query rows after the rotation in the tile buffers (free until the first copies)
        const uint32_t len = fq ? own_query_records<D, QP>(a, d, hd, s, rot_s, pg_s, qraw_s, qt_s) : 0u;
        attn_pair<D, QM, KK, VF32, LP>(a, pl, d, hd, s, split * a.tokens_per_split,
                                       split * a.tokens_per_split + a.tokens_per_split, split, a.splits, phase,
                                       staged_hd, fq ? qt_s : nullptr, false, len, fq ? lko_s : nullptr);
        return;
    }
    const uint64_t g1 = g0 + K < total ? g0 + K : total;
    for (uint64_t g = g0; g < g1;) {
        const uint32_t p = (uint32_t)(g / nt);
        const uint64_t pstart = (uint64_t)p * nt;
        const uint32_t lo = (uint32_t)(g - pstart), hi = (uint32_t)((g1 < pstart + nt ? g1 : pstart + nt) - pstart);
        const uint32_t first = (uint32_t)(pstart / K), last = (uint32_t)((pstart + nt - 1) / K);
        attn_pair<D, QM, KK, VF32, LP>(a, pl, d, p / a.seq_count, p % a.seq_count, lo * CT, hi * CT, split - first,
                                       last - first + 1, phase, staged_hd);
        g = pstart + nt;
    }
}

template <int D, int QM, KKind KK, bool VF32>
__global__ void __launch_bounds__(kThreads, MinBlocks<D, QM, KK>::value)
    attn_kernel(const __grid_constant__ AttnArgs a, const Plan pl, uint32_t d) {
    attn_body<D, QM, KK, VF32, RuntimeGroups>(a, pl, d, blockIdx.x, blockIdx.y, blockIdx.z);
}

// Query records for one (sequence, KV head): qt[j][r] = sum_{i in group(j)} R[j][i] *
// q_r[perm[i]] / sqrt(d) for packed keys (the query rotated into the code domain), or
// q_r[j] / sqrt(d) for dense keys; zero for j >= d and r >= rows.  One CTA per
// (head, sequence), computed once instead of once per split.
static __global__ void __launch_bounds__(128) qrot_kernel(const __grid_constant__ AttnArgs a, uint32_t d, uint32_t D,
                                                   uint32_t QP, int packed) {
    constexpr uint32_t RS = 64 + 1;      // row stride of the transposed rotation (padded)
    __shared__ float qin[kMaxRows * kMaxDim];         // the raw query rows
    __shared__ float qraw[kMaxRows * (kMaxDim + 1)];  // RoPE'd and permuted, rows of d + 1
    __shared__ float rot_s[64 * RS];   // the head's rotation transposed, head dims up to 64
    __shared__ uint8_t pg_s[2 * 64];   // its permutation, then the group of each dim
    const uint32_t hd = blockIdx.x, s = blockIdx.y, R = a.rows, RQ = d + 1;
    const AttnHead &h = a.head[hd];
    // the rotation is read by every output: one copy into shared memory instead of a chain of
    // dependent L2 reads per output, transposed (R[j][i] at rot_s[i * RS + j]) so that the
    // outputs of one warp (consecutive j) read consecutive banks, where rows 64 floats apart
    // would share one; with it the permutation and groups.  They are the store's own tables,
    // so the copies run before the wait for the kernel ahead (programmatic launch)
    const bool staged = packed && d <= 64;
    if (staged) {
#pragma unroll 8
        for (uint32_t e = threadIdx.x; e < d * d; e += blockDim.x) rot_s[(e % d) * RS + e / d] = __ldg(h.rot + e);
        for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
            pg_s[i] = h.perm[i];
            pg_s[64 + i] = h.group_of[i];
        }
    }
    pdl_wait();
    pdl_trigger();
    const float *qg = a.q + ((uint64_t)s * a.heads + hd) * (uint64_t)R * d;
    // the raw rows in the same round trip as the length (no load waits on the permutation)
    const uint32_t len = a.lengths[a.seq_first + s];
    for (uint32_t idx = threadIdx.x; idx < R * d; idx += blockDim.x) qin[idx] = __ldcg(qg + idx);
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < R * d; idx += blockDim.x) {
        const uint32_t r = idx / d, i = idx % d;
        // a query sits at its position (default: the last appended row)
        const uint32_t pos = a.positions ? a.positions[s * R + r] : (len ? len - 1 : 0);
        const uint32_t src = packed ? (staged ? pg_s[i] : h.perm[i]) : i;
        qraw[r * RQ + i] = rope_elem(qin + r * d, src, d, pos, a.rope);
    }
    __syncthreads();
    const float qscale = kLog2e / sqrtf((float)d);  // scores in log2 units
    float *out = a.qt + ((uint64_t)s * a.heads + hd) * (uint64_t)(D * QP);
    for (uint32_t idx = threadIdx.x; idx < D * QP; idx += blockDim.x) {
        const uint32_t j = idx / QP, r = idx % QP;
        float v = 0.0f;
        if (r < R && j < d) {
            const float *qr = qraw + r * RQ;
            if (packed) {
                const uint32_t g = staged ? pg_s[64 + j] : h.group_of[j], lo = h.group_off[g], hi = h.group_off[g + 1];
                if (staged) {
                    for (uint32_t i = lo; i < hi; ++i) v = fmaf(rot_s[i * RS + j], qr[i], v);
                } else {
                    const float *rj = h.rot + (uint64_t)j * d;
                    for (uint32_t i = lo; i < hi; ++i) v = fmaf(rj[i], qr[i], v);
                }
            } else {
                v = qr[j];
            }
            v *= qscale;
        }
        out[idx] = v;
    }
}

#ifndef __CUDACC_RTC__
// Host-side dispatch helper for one (D, QM, KK, VF32) instantiation.
template <int D, int QM, KKind KK, bool VF32>
cudaError_t run(const AttnArgs &a, const Plan &pl, uint32_t d, dim3 grid, cudaStream_t s) {
    auto kern = attn_kernel<D, QM, KK, VF32>;
    static int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || (int)pl.total > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.total);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = (int)pl.total;
    }
    return launch_pdl(kern, grid, dim3(kThreads), pl.total, s, a, pl, d);
}

// Resident CTAs per SM for a plan; remembered per (device, shared-memory size), so launches
// after the first make no attribute calls (nothing but the launch itself while a stream is
// being captured).
template <int D, int QM, KKind KK, bool VF32>
int occupancy(const Plan &pl) {
    auto kern = attn_kernel<D, QM, KK, VF32>;
    static int cached_dev[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
    static uint32_t cached_smem[8] = {};
    static int cached_n[8] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = dev & 7;
    if (cached_dev[slot] == dev && cached_smem[slot] == pl.total) return cached_n[slot];
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.total);
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, pl.total);
    cached_dev[slot] = dev;
    cached_smem[slot] = pl.total;
    cached_n[slot] = n;
    return n;
}
#endif  // __CUDACC_RTC__

}  // namespace attn
}  // namespace bgtq
