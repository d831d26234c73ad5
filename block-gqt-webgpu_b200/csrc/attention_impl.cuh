// Flash-decoding attention over the Block-GTQ key cache (sm_100a).
//
// Replaces the reference's three-pass WGSL attention - fused packed-K dot
// (src/attention/fused-dot.wgsl:15-37), parallel softmax and weighted sum
// (src/attention/parallel-tail.wgsl:10-33), the model's compressed_dot / softmax /
// weighted kernels (src/model/compressed-dot.wgsl:14-31, src/model/attention.wgsl:13-39)
// and the baseline FP16/FP32-K passes (src/attention/attention.wgsl:17-43) - with one
// kernel per (split, KV head, sequence) plus a last-CTA split combine.  Semantics follow
// src/reference/attention.py:5-22: logits = q.k/sqrt(d), positions t > pos masked when
// causal, softmax, P.V, all accumulated in FP32.
//
// Packed keys are never reconstructed.  The query is rotated once into the code domain,
//   qt_i = sum_{j in group(i)} R[i][j] q[perm[j]] / sqrt(d),
// so that q.k = sum_g s_g sum_{i in g} qt_i cent[i][code_i] (k = reconstruct(codes) of
// src/reference/production_math.py:27-31, R block-diagonal as PackedKeys enforces).
//
// Data movement: each warp owns a two-stage ring of shared-memory tiles (packed rows,
// FP16 scales, V rows) filled by cp.async.bulk (TMA bulk copies, no multicast) that
// complete on an mbarrier; every mbarrier wait is bounded and reports a timeout through
// the device status word instead of spinning forever.
// Compute layout: lane = token for dequantisation + QK (codes in registers, codebooks in
// shared memory, query records broadcast), lane = 16-byte slice of V for P.V.
#pragma once

#include <cuda_fp16.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace attn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kWaitLimit = 1u << 22;

template <int D>
struct Geo {
    static constexpr int TPL = D <= 64 ? 2 : 1;  // tokens per lane in the lane=token phase
    static constexpr int TT = 32 * TPL;          // tokens per warp tile
    static constexpr int RW = D / 4;             // max 32-bit words of a packed row
};
template <int QM>
struct QPad {
    static constexpr int QP = QM <= 1 ? 1 : QM <= 2 ? 2 : QM <= 4 ? 4 : 8;
};

struct Plan {
    uint32_t cent, qrec, stage, pbuf, bars, total;
    uint32_t kbytes, sbytes, vbytes, stage_bytes, cent_alloc;
    uint32_t stages;  // 2: prefetch the next tile while computing; 1 when two do not fit
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

inline Plan make_plan(KKind kk, int v_f32, uint32_t D, uint32_t QP, uint32_t TT, uint32_t row_stride,
                      uint32_t scale_stride, uint32_t n_cent, uint32_t smem_limit = 227u * 1024u,
                      uint32_t stages = 2) {
    Plan p{};
    p.stages = stages;
    uint32_t off = 0;
    p.cent = off;
    p.cent_alloc = kk == KKind::Packed ? n_cent + 256u : 0u;
    off = align16(off + 4u * p.cent_alloc);
    p.qrec = off;
    off = align16(off + 4u * D * QP);
    p.kbytes = TT * row_stride;
    p.sbytes = kk == KKind::Packed ? TT * scale_stride * 2u : 0u;
    p.vbytes = TT * D * (v_f32 ? 4u : 2u);
    p.stage_bytes = align16(p.kbytes) + align16(p.sbytes) + align16(p.vbytes);
    off = (off + 127u) & ~127u;
    p.stage = off;
    off += kWarps * stages * p.stage_bytes;
    p.pbuf = off;
    off = align16(off + kWarps * TT * QP * 4u);
    p.bars = off;
    off += kWarps * 2u * 8u;
    p.total = align16(off);
    if (p.total > smem_limit && stages == 2)
        return make_plan(kk, v_f32, D, QP, TT, row_stride, scale_stride, n_cent, smem_limit, 1);
    return p;
}

// ---- PTX helpers: mbarrier + bulk async copies (sm_90+, no multicast) ----
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

// Dequantise + QK for the TPL tokens of this lane.  The packed rows sit in registers.
// Pass 1 walks the nibble region two dimensions (one byte) at a time at compile-time bit
// positions; the row is then realigned in place by ns/2 bytes so that pass 2 finds the
// byte-region code of dimension j at byte j, again at a compile-time position.  Both
// passes keep per-group partial sums and scale them once per group (groups are whole
// pairs and the nibble/byte split is a group boundary, as parse_layout enforces).
template <int D, int QM, int QP>
__device__ __forceinline__ void packed_qk(const AttnHead &h, const unsigned char *kb, const uint16_t *sb,
                                          const float *cent_s, const float *qrec_s, const uint32_t (&bm)[4],
                                          int lane, float (&acc)[Geo<D>::TPL][QM]) {
    constexpr int TPL = Geo<D>::TPL, RW = Geo<D>::RW;
    const uint32_t row_stride = h.row_stride, ns = h.ns;
    uint32_t W[TPL][RW], sw[TPL][4];
    float part[TPL][QM];
#pragma unroll
    for (int tt = 0; tt < TPL; ++tt) {
        const int tl = tt * 32 + lane;
        const uint4 *rp = reinterpret_cast<const uint4 *>(kb + (size_t)tl * row_stride);
#pragma unroll
        for (int q4 = 0; q4 < RW / 4; ++q4) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if ((uint32_t)q4 * 16u < row_stride) v = rp[q4];
            W[tt][4 * q4 + 0] = v.x; W[tt][4 * q4 + 1] = v.y; W[tt][4 * q4 + 2] = v.z; W[tt][4 * q4 + 3] = v.w;
        }
        if (h.scale_stride == 4) {
            const uint2 v = *reinterpret_cast<const uint2 *>(sb + (size_t)tl * 4);
            sw[tt][0] = v.x; sw[tt][1] = v.y; sw[tt][2] = 0u; sw[tt][3] = 0u;
        } else {
            const uint4 v = *reinterpret_cast<const uint4 *>(sb + (size_t)tl * 8);
            sw[tt][0] = v.x; sw[tt][1] = v.y; sw[tt][2] = v.z; sw[tt][3] = v.w;
        }
#pragma unroll
        for (int r = 0; r < QM; ++r) { acc[tt][r] = 0.0f; part[tt][r] = 0.0f; }
    }
    auto flush = [&]() {
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
            const float sc = half_lo(sw[tt][0]);
#pragma unroll
            for (int r = 0; r < QM; ++r) { acc[tt][r] = fmaf(sc, part[tt][r], acc[tt][r]); part[tt][r] = 0.0f; }
            sw[tt][0] = __funnelshift_r(sw[tt][0], sw[tt][1], 16);
            sw[tt][1] = __funnelshift_r(sw[tt][1], sw[tt][2], 16);
            sw[tt][2] = __funnelshift_r(sw[tt][2], sw[tt][3], 16);
            sw[tt][3] >>= 16;
        }
    };
    // ---- pass 1: nibble region, dimensions (j, j+1) share byte j/2 ----
#pragma unroll
    for (int j = 0; j < D; j += 2) {
        if ((uint32_t)j < ns) {
            float q0[QP], q1[QP];
            load_q<QP>(qrec_s + j * QP, q0);
            load_q<QP>(qrec_s + (j + 1) * QP, q1);
            const float *cb0 = cent_s + h.cb_base[j], *cb1 = cent_s + h.cb_base[j + 1];
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const uint32_t byte = W[tt][j >> 3] >> (((j >> 1) & 3) * 8);
                const float c0 = cb0[byte & 15u], c1 = cb1[(byte >> 4) & 15u];
#pragma unroll
                for (int r = 0; r < QM; ++r) part[tt][r] = fmaf(q1[r], c1, fmaf(q0[r], c0, part[tt][r]));
            }
            if (j + 2 < D && ((bm[(j + 2) >> 5] >> ((j + 2) & 31)) & 1u)) flush();
        }
    }
    // ---- realign: byte-region code of dimension j (>= ns) moves to byte j ----
    if (ns < (uint32_t)D) {
        const uint32_t sbytes = ns >> 1, aw = sbytes >> 2, c8 = (sbytes & 3u) * 8u;
#pragma unroll
        for (int tt = 0; tt < TPL; ++tt) {
#pragma unroll
            for (int b = 1; b < RW; b <<= 1) {
                if (aw & (uint32_t)b) {
#pragma unroll
                    for (int k = RW - 1; k >= 0; --k) W[tt][k] = k >= b ? W[tt][k - b] : 0u;
                }
            }
#pragma unroll
            for (int k = RW - 1; k >= 0; --k) W[tt][k] = __funnelshift_l(k > 0 ? W[tt][k - 1] : 0u, W[tt][k], c8);
        }
    }
    // ---- pass 2: byte region ----
#pragma unroll
    for (int j = 0; j < D; j += 2) {
        if ((uint32_t)j >= ns) {
            float q0[QP], q1[QP];
            load_q<QP>(qrec_s + j * QP, q0);
            load_q<QP>(qrec_s + (j + 1) * QP, q1);
            const float *cb0 = cent_s + h.cb_base[j], *cb1 = cent_s + h.cb_base[j + 1];
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const float c0 = cb0[(W[tt][j >> 2] >> ((j & 3) * 8)) & 255u];
                const float c1 = cb1[(W[tt][(j + 1) >> 2] >> (((j + 1) & 3) * 8)) & 255u];
#pragma unroll
                for (int r = 0; r < QM; ++r) part[tt][r] = fmaf(q1[r], c1, fmaf(q0[r], c0, part[tt][r]));
            }
            if (j + 2 < D && ((bm[(j + 2) >> 5] >> ((j + 2) & 31)) & 1u)) flush();
        }
    }
#pragma unroll
    for (int tt = 0; tt < TPL; ++tt) {
        const float sc = half_lo(sw[tt][0]);
#pragma unroll
        for (int r = 0; r < QM; ++r) acc[tt][r] = fmaf(sc, part[tt][r], acc[tt][r]);
    }
}

template <int D, int QM, KKind KK, bool VF32>
__global__ void __launch_bounds__(kThreads) attn_kernel(const __grid_constant__ AttnArgs a, const Plan pl, uint32_t d) {
    constexpr int TPL = Geo<D>::TPL, TT = Geo<D>::TT, QP = QPad<QM>::QP;
    constexpr int VSZ = VF32 ? 4 : 2, VEC = 16 / VSZ, LPT = D / VEC, TPS = 32 / LPT;
    static_assert(LPT >= 1 && LPT <= 32, "V slice layout");
    constexpr int KSZ = KK == KKind::F32 ? 4 : 2, KVEC = 16 / KSZ, LPTK = D / KVEC, TPSK = 32 / LPTK;
    static_assert(KK == KKind::Packed || (LPTK >= 1 && LPTK <= 32), "K slice layout");

    const uint32_t split = blockIdx.x, hd = blockIdx.y, s = blockIdx.z;
    const AttnHead &h = a.head[hd];
    const uint32_t seq = a.seq_first + s;
    const uint32_t len = a.lengths[seq];
    const uint32_t R = a.rows;
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;

    extern __shared__ __align__(128) unsigned char smem[];
    float *cent_s = reinterpret_cast<float *>(smem + pl.cent);
    float *qrec_s = reinterpret_cast<float *>(smem + pl.qrec);
    float *pbuf = reinterpret_cast<float *>(smem + pl.pbuf) + w * TT * QP;
    const uint32_t bar0 = smem_u32(smem + pl.bars) + (uint32_t)w * 16u;
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
    const uint32_t t0 = split * a.tokens_per_split;
    const uint32_t t1 = min(t0 + a.tokens_per_split, tend);

    // ---- prologue: codebooks, query records, barriers ----
    if constexpr (KK == KKind::Packed) {
        for (uint32_t i = tid; i < pl.cent_alloc; i += kThreads) cent_s[i] = i < h.n_cent ? h.cent[i] : 0.0f;
    }
    // query records (rotated into code order and scaled by 1/sqrt(d) by qrot_kernel)
    {
        const float4 *src = reinterpret_cast<const float4 *>(a.qt + ((uint64_t)s * a.heads + hd) * (uint64_t)(D * QP));
        float4 *dst = reinterpret_cast<float4 *>(qrec_s);
        for (uint32_t i = tid; i < (uint32_t)(D * QP / 4); i += kThreads) dst[i] = __ldg(src + i);
    }
    if (tid < kWarps * 2) mbar_init(smem_u32(smem + pl.bars) + tid * 8u, 1u);
    fence_barrier_init();
    uint32_t bm[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) bm[i] = h.bound_mask[i];
    __syncthreads();

    // ---- per-warp flash-decoding over this split ----
    float m[QM], l[QM], O[QM][VEC];
#pragma unroll
    for (int r = 0; r < QM; ++r) {
        m[r] = -INFINITY; l[r] = 0.0f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) O[r][e] = 0.0f;
    }
    float qreg[QM][KVEC];
    if constexpr (KK != KKind::Packed) {
        const int dl = (lane % LPTK) * KVEC;
#pragma unroll
        for (int r = 0; r < QM; ++r)
#pragma unroll
            for (int e = 0; e < KVEC; ++e) qreg[r][e] = qrec_s[(dl + e) * QP + r];
    }
    const uint32_t ntok = t1 > t0 ? t1 - t0 : 0u;
    const uint32_t ntiles = (ntok + TT - 1) / TT;
    unsigned char *stage0 = smem + pl.stage + (size_t)w * pl.stages * pl.stage_bytes;
    const bool two = pl.stages == 2;
    const unsigned char *kbase = h.k + (uint64_t)seq * h.k_seq_stride;
    const unsigned char *sbase =
        KK == KKind::Packed ? reinterpret_cast<const unsigned char *>(h.scales + (uint64_t)seq * h.s_seq_stride) : nullptr;
    const unsigned char *vbase = static_cast<const unsigned char *>(h.v) + (uint64_t)seq * h.v_seq_stride;
    const uint32_t krow = h.row_stride, vrow = D * VSZ, srow = h.scale_stride * 2u;

    auto issue = [&](uint32_t k, int st) {
        if (lane == 0) {
            const uint32_t at = t0 + k * TT, n = min((uint32_t)TT, t1 - at);
            unsigned char *buf = stage0 + (size_t)st * pl.stage_bytes;
            const uint32_t kb = n * krow, vb = n * vrow;
            const uint32_t sb = KK == KKind::Packed ? ((n + 1u) & ~1u) * srow : 0u;
            const uint32_t bar = bar0 + (uint32_t)st * 8u;
            fence_proxy_async();
            mbar_expect_tx(bar, kb + sb + vb);
            bulk_g2s(smem_u32(buf), kbase + (uint64_t)at * krow, kb, bar);
            if (KK == KKind::Packed)
                bulk_g2s(smem_u32(buf + align16(pl.kbytes)), sbase + (uint64_t)at * srow, sb, bar);
            bulk_g2s(smem_u32(buf + align16(pl.kbytes) + align16(pl.sbytes)), vbase + (uint64_t)at * vrow, vb, bar);
        }
    };

    bool ok = true;
    uint32_t phase = 0;
    if ((uint32_t)w < ntiles) issue(w, 0);
    int it = 0;
    for (uint32_t k = w; k < ntiles; k += kWarps, ++it) {
        const int st = two ? (it & 1) : 0;
        if (two && k + kWarps < ntiles) issue(k + kWarps, st ^ 1);
        if (!mbar_wait_bounded(bar0 + (uint32_t)st * 8u, (phase >> st) & 1u)) {
            ok = false;
            break;
        }
        phase ^= 1u << st;
        const uint32_t at = t0 + k * TT, n = min((uint32_t)TT, t1 - at);
        const unsigned char *kb = stage0 + (size_t)st * pl.stage_bytes;
        const uint16_t *sb = reinterpret_cast<const uint16_t *>(kb + align16(pl.kbytes));
        const unsigned char *vb = kb + align16(pl.kbytes) + align16(pl.sbytes);

        // ---- logits for this lane's TPL tokens ----
        float acc[TPL][QM];
        if constexpr (KK == KKind::Packed) {
            packed_qk<D, QM, QP>(h, kb, sb, cent_s, qrec_s, bm, lane, acc);
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
                    if ((lane % LPTK) == 0 && tl < n) pbuf[tl * QP + r] = sum;
                }
            }
            __syncwarp();
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const uint32_t tl = tt * 32 + lane;
#pragma unroll
                for (int r = 0; r < QM; ++r) acc[tt][r] = tl < n ? pbuf[tl * QP + r] : 0.0f;
            }
            __syncwarp();
        }

        // ---- masking, optional raw-logit capture, online softmax ----
        float alpha[QM];
#pragma unroll
        for (int r = 0; r < QM; ++r) {
            float lg[TPL];
            float tm = -INFINITY;
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const uint32_t tl = tt * 32 + lane, tok = at + tl;
                const bool valid = tl < n && (uint32_t)r < R && (!a.causal || tok <= pos[r]);
                lg[tt] = valid ? acc[tt][r] : -INFINITY;
                if (a.logits && tl < n && (uint32_t)r < R)
                    a.logits[(((uint64_t)s * a.heads + hd) * R + r) * a.logit_stride + tok] = lg[tt];
                tm = fmaxf(tm, lg[tt]);
            }
            tm = warp_max(tm);
            const float mnew = fmaxf(m[r], tm);
            alpha[r] = mnew == -INFINITY ? 1.0f : exp2f((m[r] - mnew) * kLog2e);
            float ps = 0.0f;
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt) {
                const float p = lg[tt] == -INFINITY ? 0.0f : exp2f((lg[tt] - mnew) * kLog2e);
                pbuf[(tt * 32 + lane) * QP + r] = p;
                ps += p;
            }
            ps = warp_sum(ps);
            l[r] = l[r] * alpha[r] + ps;
            m[r] = mnew;
        }
        if constexpr (QP > QM) {
#pragma unroll
            for (int tt = 0; tt < TPL; ++tt)
#pragma unroll
                for (int r = QM; r < QP; ++r) pbuf[(tt * 32 + lane) * QP + r] = 0.0f;
        }
#pragma unroll
        for (int r = 0; r < QM; ++r)
#pragma unroll
            for (int e = 0; e < VEC; ++e) O[r][e] *= alpha[r];
        __syncwarp();

        // ---- P.V: lane = 16-byte slice of a V row ----
        {
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
                    float p[QP];
                    load_q<QP>(pbuf + tl * QP, p);
#pragma unroll
                    for (int r = 0; r < QM; ++r)
#pragma unroll
                        for (int e = 0; e < VEC; ++e) O[r][e] = fmaf(p[r], vv[e], O[r][e]);
                }
            }
        }
        __syncwarp();
        if (!two && k + kWarps < ntiles) issue(k + kWarps, 0);
    }
    if (!ok) atomicOr(a.status, kStatusWaitTimeout);

    // ---- reduce P.V partial sums across token slots of the warp ----
#pragma unroll
    for (int r = 0; r < QM; ++r)
#pragma unroll
        for (int e = 0; e < VEC; ++e)
#pragma unroll
            for (int o = LPT; o < 32; o <<= 1) O[r][e] += __shfl_xor_sync(0xffffffffu, O[r][e], o);

    // ---- merge the warps of this CTA ----
    __syncthreads();
    float *mO = reinterpret_cast<float *>(smem + pl.stage);  // [kWarps][QP][D]
    float *mm = mO + kWarps * QP * D;                        // [kWarps][QP]
    float *ml = mm + kWarps * QP;
    if (lane < LPT) {
#pragma unroll
        for (int r = 0; r < QM; ++r)
#pragma unroll
            for (int e = 0; e < VEC; ++e) mO[(w * QP + r) * D + (lane % LPT) * VEC + e] = O[r][e];
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
            const float f = mw == -INFINITY ? 0.0f : exp2f((mw - M) * kLog2e);
            L = fmaf(ml[ww * QP + r], f, L);
            Ov = fmaf(mO[(ww * QP + r) * D + dd], f, Ov);
        }
        if (a.splits == 1) {
            a.out[(obase + r) * d + dd] = Ov / L;
            if (dd == 0 && a.lse) a.lse[obase + r] = M + logf(L);
        } else {
            float *pp = a.part + ((((uint64_t)split * a.seq_count + s) * a.heads + hd) * R + r) * (uint64_t)(d + 2);
            pp[dd] = Ov;
            if (dd == 0) { pp[d] = M; pp[d + 1] = L; }
        }
    }
    if (a.splits > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t ticket = atomicAdd(&a.counters[s * a.heads + hd], 1u);
            s_last = ticket == a.splits - 1 ? 1u : 0u;
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            const uint64_t sstride = (uint64_t)a.seq_count * a.heads * R * (d + 2);
            for (uint32_t idx = tid; idx < rows_live * d; idx += kThreads) {
                const uint32_t r = idx / d, dd = idx % d;
                const float *pp = a.part + (((uint64_t)s * a.heads + hd) * R + r) * (uint64_t)(d + 2);
                float M = -INFINITY;
                for (uint32_t sp = 0; sp < a.splits; ++sp) M = fmaxf(M, __ldcg(pp + sp * sstride + d));
                float L = 0.0f, Ov = 0.0f;
                for (uint32_t sp = 0; sp < a.splits; ++sp) {
                    const float ms = __ldcg(pp + sp * sstride + d);
                    const float f = ms == -INFINITY ? 0.0f : exp2f((ms - M) * kLog2e);
                    L = fmaf(__ldcg(pp + sp * sstride + d + 1), f, L);
                    Ov = fmaf(__ldcg(pp + sp * sstride + dd), f, Ov);
                }
                a.out[(obase + r) * d + dd] = Ov / L;
                if (dd == 0 && a.lse) a.lse[obase + r] = M + logf(L);
            }
            if (tid == 0) a.counters[s * a.heads + hd] = 0u;
        }
    }
}

// Query records for one (sequence, KV head): qt[j][r] = sum_{i in group(j)} R[j][i] *
// q_r[perm[i]] / sqrt(d) for packed keys (the query rotated into the code domain), or
// q_r[j] / sqrt(d) for dense keys; zero for j >= d and r >= rows.  One CTA per
// (head, sequence), computed once instead of once per split.
__global__ void __launch_bounds__(128) qrot_kernel(const __grid_constant__ AttnArgs a, uint32_t d, uint32_t D,
                                                   uint32_t QP, int packed) {
    __shared__ float qraw[kMaxRows * kMaxDim];
    const uint32_t hd = blockIdx.x, s = blockIdx.y, R = a.rows;
    const AttnHead &h = a.head[hd];
    const float *qg = a.q + ((uint64_t)s * a.heads + hd) * (uint64_t)R * d;
    for (uint32_t idx = threadIdx.x; idx < R * d; idx += blockDim.x) {
        const uint32_t r = idx / d, i = idx % d;
        qraw[idx] = packed ? qg[r * d + h.perm[i]] : qg[r * d + i];
    }
    __syncthreads();
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
    float *out = a.qt + ((uint64_t)s * a.heads + hd) * (uint64_t)(D * QP);
    for (uint32_t idx = threadIdx.x; idx < D * QP; idx += blockDim.x) {
        const uint32_t j = idx / QP, r = idx % QP;
        float v = 0.0f;
        if (r < R && j < d) {
            if (packed) {
                const uint32_t g = h.group_of[j], lo = h.group_off[g], hi = h.group_off[g + 1];
                const float *rj = h.rot + (uint64_t)j * d;
                for (uint32_t i = lo; i < hi; ++i) v = fmaf(rj[i], qraw[r * d + i], v);
            } else {
                v = qraw[r * d + j];
            }
            v *= inv_sqrt_d;
        }
        out[idx] = v;
    }
}

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
    kern<<<grid, kThreads, pl.total, s>>>(a, pl, d);
    return cudaGetLastError();
}

template <int D, int QM, KKind KK, bool VF32>
int occupancy(const Plan &pl) {
    auto kern = attn_kernel<D, QM, KK, VF32>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.total);
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, pl.total);
    return n;
}

}  // namespace attn
}  // namespace bgtq
