// Causal prefill attention over the Block-GTQ key cache on the 5th-generation tensor cores
// (tcgen05 UMMA with TMEM accumulators, sm_100a).
//
// Same computation as prefill.cu (src/model/decoder.ts:30-81 model prefill; semantics of
// src/reference/attention.py:5-22 over k = reconstruct(codes)), restructured for UMMA:
// one CTA of 256 threads owns M = 128 query rows - floor(128 / G) positions x the G query
// heads of one KV head; a row = a TMEM lane, served by two threads (warps w and w + 4)
// that take key columns / output dims 0-31 and 32-63 - and walks 64-key tiles:
//   1. the packed tile (rows + FP16 scales) and the V tile arrive by cp.async.bulk (TMA
//      bulk copies, no multicast) on mbarriers, two tiles in flight;
//   2. all threads dequantise the packed tile into shared memory as code-domain values
//      s_g * cent split into FP16 high / low halves (K-major, 128-byte swizzle), a thread per
//      key and eight dimension pairs, decoded from a per-pair table;
//   3. one thread issues S = Q_hi C_hi + Q_hi C_lo + Q_lo C_hi as 12 UMMAs (M 128, N 64,
//      K 16) into three TMEM accumulators - the large high x high term over dims 0-31 and
//      32-63 separately, the two small cross terms together - so the tensor cores' running
//      sums stay short; tcgen05.commit signals an mbarrier;
//   4. each thread loads its half row (tcgen05.ld), adds the three parts in FP32, masks,
//      and the two halves of a row agree on the running maximum through shared memory; an
//      online softmax in log2 units writes P_hi / P_lo (probabilities scaled by 2^12);
//   5. one thread issues the tile's O = P_hi V + P_lo V as 8 UMMAs (V MN-major, the value
//      store's swizzled rows copied verbatim) into a fresh TMEM accumulator, and each
//      thread folds it into its FP32 output row: o = alpha o + O_tile.
// Every mbarrier wait is bounded; on a timeout the CTA reports it in the device status
// word, waits (bounded) for its copies and tensor-core work in flight, frees its TMEM and
// stops.  TMEM: 256 columns per CTA; shared memory keeps at most two CTAs on an SM, so
// allocations never wait on each other.
#include <cuda_fp16.h>

#include "attention_impl.cuh"

namespace bgtq {
namespace tc {

using attn::bulk_g2s;
using attn::fence_barrier_init;
using attn::fence_proxy_async;
using attn::kLog2e;
using attn::kPShift;
using attn::mbar_expect_tx;
using attn::mbar_init;
using attn::mbar_wait_bounded;
using attn::smem_u32;

constexpr int D = 64, BN = 64, M = 128, NTH = 256;  // two threads per row: column halves
constexpr uint32_t kRow = D * 2;                // bytes of one FP16 row (128-byte swizzle row)
constexpr uint32_t kQTile = M * kRow;           // 16 KB
constexpr uint32_t kCTile = BN * kRow;          // 8 KB
constexpr uint32_t kTmemCols = 256;
// TMEM columns: S_hh over dims 0-31, S_hh over dims 32-63, S cross terms, O tile
constexpr uint32_t kColHH0 = 0, kColHH1 = 64, kColX = 128, kColO = 192;
// Per dimension pair decode word (x): byte of the codes in the packed row, bit 8: the pair
// is two raw bytes (else the low / high nibbles of one byte), bits 16-18: group; (y): the
// compact codebook offsets of the two dimensions.  Pairs past the head dim decode zeros.
constexpr uint32_t kPairByte = 1u << 8;

struct Plan {
    uint32_t qhi, qlo, chi, clo, phi, plo, vst, kst, cent, meta, bars, slot, red, total;
    uint32_t kstage, cent_alloc;
};

inline Plan make_plan(uint32_t row_stride, uint32_t scale_stride, uint32_t n_cent) {
    Plan p{};
    uint32_t off = 0;  // relative to a 1024-byte aligned base
    p.qhi = off; off += kQTile;
    p.qlo = off; off += kQTile;
    p.chi = off; off += kCTile;
    p.clo = off; off += kCTile;
    p.phi = off; off += kQTile;
    p.plo = off; off += kQTile;
    p.vst = off; off += 2 * kCTile;
    p.kstage = attn::align128(attn::align16(BN * row_stride) + attn::align16(BN * scale_stride * 2u));
    p.kst = off; off += 2 * p.kstage;
    p.cent_alloc = n_cent + 16u;
    p.cent = off; off = attn::align16(off + 4u * p.cent_alloc);
    p.meta = off; off += 4u * D;
    p.bars = off; off += 8u * 8u;   // K0, K1, V0, V1, S, O
    p.slot = off; off += 16u;
    p.red = off; off += 2u * M * 4u;  // per-half row maxima, then row sums
    p.total = attn::align16(off) + 1024u;  // slack to align the base
    return p;
}

// UMMA shared-memory descriptor: 128-byte swizzle, SBO = 1024 bytes (8-row atoms),
// LBO as given, SM100 version 1 (CUTLASS UMMA::SmemDescriptor bit layout).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3fffu);
    d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
    d |= (uint64_t)((1024u >> 4) & 0x3fffu) << 32;
    d |= (uint64_t)1 << 46;        // version
    d |= (uint64_t)2 << 61;        // SWIZZLE_128B
    return d;
}
// Instruction descriptor, kind::f16: F32 accumulate, F16 A and B, A K-major, B K- or
// MN-major, N = 64, M = 128 (CUTLASS UMMA::InstrDescriptor bit layout).
__host__ __device__ constexpr uint32_t idesc(uint32_t b_mn_major) {
    return (1u << 4) | (b_mn_major << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive FP32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void split2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 f = __half22float2(h);
    const float2 r = __ffma2_rn(f, make_float2(-1.0f, -1.0f), make_float2(x, y));  // exact x - f
    const __half2 l = __floats2half2_rn(r.x, r.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Write 8 FP32 values as FP16 high / low halves into chunk `ch` of swizzled row `row`.
__device__ __forceinline__ void put8(unsigned char *hi_tile, unsigned char *lo_tile, uint32_t row, uint32_t ch,
                                     const float (&v)[8]) {
    uint4 h, l;
    split2(v[0], v[1], h.x, l.x);
    split2(v[2], v[3], h.y, l.y);
    split2(v[4], v[5], h.z, l.z);
    split2(v[6], v[7], h.w, l.w);
    const uint32_t at = row * kRow + ((ch ^ (row & 7u)) << 4);
    *reinterpret_cast<uint4 *>(hi_tile + at) = h;
    *reinterpret_cast<uint4 *>(lo_tile + at) = l;
}

template <int G>
__global__ void __launch_bounds__(NTH, 2) prefill_tc_kernel(const __grid_constant__ PrefillArgs a, const Plan pl) {
    constexpr uint32_t PB = M / G;  // positions per CTA
    const uint32_t qb = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const AttnHead &hd = a.head[h];
    const uint32_t seq = a.seq_first + s;
    const uint32_t tid = threadIdx.x, warp = tid >> 5;
    const uint32_t row = tid & (M - 1), hf = tid >> 7;  // row (TMEM lane) and column half
    const uint32_t pi = row / G, gq = row % G;
    const uint32_t q0 = qb * PB, qi = q0 + pi;
    const bool live = pi < PB && qi < a.n;
    const uint32_t pos = a.pos_first + qi;
    const uint32_t nq = min(PB, a.n - q0);
    const uint32_t last_pos = a.pos_first + q0 + nq - 1;
    const uint32_t len = a.lengths[seq];
    const uint32_t kend = min(last_pos + 1, len);
    const uint32_t ntiles = (kend + BN - 1) / BN;

    extern __shared__ unsigned char smem_raw[];
    unsigned char *sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(sm);
    float *cent_s = reinterpret_cast<float *>(sm + pl.cent);
    uint2 *pair_s = reinterpret_cast<uint2 *>(sm + pl.meta);
    const uint32_t bars = sbase + pl.bars;
    const uint32_t bar_s = bars + 32u, bar_o = bars + 40u;
    volatile uint32_t *slot = reinterpret_cast<volatile uint32_t *>(sm + pl.slot);
    float *red = reinterpret_cast<float *>(sm + pl.red);  // [2][M]

    // ---- prologue: TMEM, codebooks, decode words, query tile, barriers ----
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + pl.slot),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    for (uint32_t i = tid; i < pl.cent_alloc; i += NTH) cent_s[i] = i < hd.n_cent ? hd.cent[i] : 0.0f;
    if (tid < (uint32_t)D / 2) {
        const uint32_t j0 = 2 * tid;
        // zero pair: nibble byte 0 against the zero tail of the codebooks (codes <= 15)
        uint2 pw = make_uint2(0u, hd.n_cent | hd.n_cent << 16);
        if (j0 < a.d) {
            const bool nib = j0 < hd.ns;
            pw.x = (nib ? tid : hd.ns / 2 + (j0 - hd.ns)) | (nib ? 0u : kPairByte) | (uint32_t)hd.group_of[j0] << 16;
            pw.y = (uint32_t)hd.cb_base[j0] | (uint32_t)hd.cb_base[j0 + 1] << 16;
        }
        pair_s[tid] = pw;
    }
    {
        // this thread's query row (code domain, log2 units) as FP16 high / low halves
        const uint64_t HQ = (uint64_t)a.heads * G;
        const float *qr = a.qt + (((uint64_t)s * a.n + (live ? qi : 0u)) * HQ + (uint64_t)h * G + gq) * D;
#pragma unroll
        for (uint32_t c4 = 0; c4 < 4; ++c4) {
            const uint32_t ch = 4 * hf + c4;
            float v[8];
            if (live) {
                const float4 x0 = *reinterpret_cast<const float4 *>(qr + ch * 8);
                const float4 x1 = *reinterpret_cast<const float4 *>(qr + ch * 8 + 4);
                v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
                v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = 0.0f;
            }
            put8(sm + pl.qhi, sm + pl.qlo, row, ch, v);
        }
    }
    if (tid < 6) mbar_init(bars + 8u * tid, 1u);
    fence_barrier_init();
    fence_proxy_async();
    tc_before_sync();
    __syncthreads();
    tc_after_sync();
    const uint32_t tmem = *slot;
    const uint32_t tlane = ((warp & 3u) * 32u) << 16;  // this warp's TMEM lanes
    const uint32_t c0 = 32u * hf;                        // this thread's first column

    const unsigned char *kbase = hd.k + (uint64_t)seq * hd.k_seq_stride;
    const unsigned char *sgl = reinterpret_cast<const unsigned char *>(hd.scales + (uint64_t)seq * hd.s_seq_stride);
    const unsigned char *vbase = static_cast<const unsigned char *>(hd.v) + (uint64_t)seq * hd.v_seq_stride;
    const uint32_t row_stride = hd.row_stride, srow = hd.scale_stride * 2u;
    const uint32_t kb_h = BN * row_stride, sb_h = BN * srow, soff = attn::align16(BN * row_stride);
    auto issue_k = [&](uint32_t j, uint32_t st) {
        const uint32_t bar = bars + 8u * st, dst = sbase + pl.kst + st * pl.kstage;
        fence_proxy_async();
        mbar_expect_tx(bar, kb_h + sb_h);
        bulk_g2s(dst, kbase + (uint64_t)j * BN * row_stride, kb_h, bar);
        bulk_g2s(dst + soff, sgl + (uint64_t)j * BN * srow, sb_h, bar);
    };
    auto issue_v = [&](uint32_t j, uint32_t st) {
        const uint32_t bar = bars + 16u + 8u * st;
        fence_proxy_async();
        mbar_expect_tx(bar, kCTile);
        bulk_g2s(sbase + pl.vst + st * kCTile, vbase + (uint64_t)j * BN * kRow, kCTile, bar);
    };
    uint32_t pending = 0;  // bits 0,1: K stages; 2,3: V stages; 4: S commit; 5: O commit
    for (uint32_t j = 0; j < 2 && j < ntiles; ++j) {
        if (tid == 0) {
            issue_k(j, j);
            issue_v(j, j);
        }
        pending |= (1u << j) | (4u << j);
    }

    constexpr uint32_t ID_QK = idesc(0), ID_PV = idesc(1);
    const uint64_t dq_hi = sdesc(sbase + pl.qhi, 0), dq_lo = sdesc(sbase + pl.qlo, 0);
    const uint64_t dc_hi = sdesc(sbase + pl.chi, 0), dc_lo = sdesc(sbase + pl.clo, 0);
    const uint64_t dp_hi = sdesc(sbase + pl.phi, 0), dp_lo = sdesc(sbase + pl.plo, 0);

    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    uint32_t phase = 0;  // bit b: parity of barrier b (K0, K1, V0, V1, S, O)
    bool err = false;    // this thread saw a wait time out; CTA-wide decisions use __syncthreads_or

    // packed tile t (stage t & 1) -> code-domain FP16 high / low halves in the C tile
    auto dequant = [&](uint32_t t) {
        const uint32_t st = t & 1u;
        if (!mbar_wait_bounded(bars + 8u * st, (phase >> st) & 1u)) err = true;
        phase ^= 1u << st;
        pending &= ~(1u << st);
        const unsigned char *kt = sm + pl.kst + st * pl.kstage;
        // thread = key (lanes: consecutive keys, one codebook per instruction) x pairs
        // 8r .. 8r+7 (chunks 2r, 2r+1); the pair's kind is uniform over the warp
        const uint32_t key = tid & (BN - 1), r = tid >> 6;
        const unsigned char *krow = kt + key * row_stride;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(kt + soff + key * srow);
        float v0[8], v1[8];
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
            const uint2 pw = pair_s[8 * r + q];
            const uint32_t boff = pw.x & 0xffu;
            uint32_t c0, c1;
            if (pw.x & kPairByte) {
                c0 = krow[boff];
                c1 = krow[boff + 1];
            } else {
                const uint32_t b = krow[boff];
                c0 = b & 15u;
                c1 = b >> 4;
            }
            const float scale = __half2float(__ushort_as_half(sc[pw.x >> 16]));
            float &x0 = q < 4 ? v0[2 * q] : v1[2 * q - 8], &x1 = q < 4 ? v0[2 * q + 1] : v1[2 * q - 7];
            x0 = cent_s[(pw.y & 0xffffu) + c0] * scale;
            x1 = cent_s[(pw.y >> 16) + c1] * scale;
        }
        put8(sm + pl.chi, sm + pl.clo, key, 2 * r, v0);
        put8(sm + pl.chi, sm + pl.clo, key, 2 * r + 1, v1);
    };
    // S = Q C^T of the tile in the C tile (issued by thread 0; the caller tracks the commit)
    auto issue_s = [&]() {
#pragma unroll
        for (uint32_t ks = 0; ks < 4; ++ks) {
            const uint64_t ko = (ks * 32u) >> 4;  // 16 dims = 32 bytes along the swizzled row
            umma(tmem + kColX, dq_lo + ko, dc_hi + ko, ID_QK, ks > 0 ? 1u : 0u);
            umma(tmem + kColX, dq_hi + ko, dc_lo + ko, ID_QK, 1u);
            umma(tmem + (ks < 2 ? kColHH0 : kColHH1), dq_hi + ko, dc_hi + ko, ID_QK, (ks & 1u) ? 1u : 0u);
        }
        umma_commit(bar_s);
    };

    // Software pipeline: tile j + 1 is dequantised while the tensor cores run tile j's P.V,
    // and its S is issued before tile j's output fold, so each tile takes three CTA barriers.
    if (ntiles > 0) {
        dequant(0);
        fence_proxy_async();
        tc_before_sync();
        __syncthreads();
        tc_after_sync();
        if (tid == 0) {
            if (2 < ntiles) issue_k(2, 0);
            issue_s();
        }
        if (2 < ntiles) pending |= 1u;
        pending |= 16u;
    }
    for (uint32_t j = 0; j < ntiles; ++j) {
        const uint32_t st = j & 1u;
        if (!mbar_wait_bounded(bar_s, (phase >> 4) & 1u)) err = true;
        phase ^= 16u;
        pending &= ~16u;
        tc_after_sync();
        // ---- this half row's scores, mask, online softmax, P halves ----
        float sv[32];
        {
            // the two high x high parts in one round trip, then the cross terms (added in the
            // same order as before: hh0 + hh1, then + x)
            float t[32];
            tmem_ld32(tmem + tlane + kColHH0 + c0, sv);
            tmem_ld32(tmem + tlane + kColHH1 + c0, t);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[i] += t[i];
            tmem_ld32(tmem + tlane + kColX + c0, t);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[i] += t[i];
        }
        const uint32_t k0 = j * BN + c0;
        if (!live || k0 + 31u > pos || k0 + 32u > len) {  // keys past the row's position or the length
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t key = k0 + i;
                sv[i] = live && key <= pos && key < len ? sv[i] : -INFINITY;
            }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, sv[i]);
        red[hf * M + row] = mx;
        tc_before_sync();
        __syncthreads();
        mx = fmaxf(red[row], red[M + row]);
        const float mnew = fmaxf(m_run, mx);
        const float alpha = mnew == -INFINITY ? 1.0f : attn::ex2(m_run - mnew);
        m_run = mnew;
        const float mref = mnew == -INFINITY ? 0.0f : mnew - kPShift;
        float ps = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float p = attn::ex2(sv[i] - mref);  // masked: 2^-inf = 0
            sv[i] = p;
            ps += p;
        }
        l_run = fmaf(l_run, alpha, ps);  // this half's share of the row sum
#pragma unroll
        for (uint32_t c4 = 0; c4 < 4; ++c4) {
            float w8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) w8[e] = sv[c4 * 8 + e];
            put8(sm + pl.phi, sm + pl.plo, row, 4 * hf + c4, w8);
        }
        fence_proxy_async();
        tc_before_sync();
        if (__syncthreads_or(err)) break;
        tc_after_sync();
        // ---- O tile = P_hi V + P_lo V on the tensor cores ----
        if (tid == 0) {
            if (!mbar_wait_bounded(bars + 16u + 8u * st, (phase >> (2 + st)) & 1u)) {
                err = true;
            } else {
                const uint64_t dv = sdesc(sbase + pl.vst + st * kCTile, kCTile);
#pragma unroll
                for (uint32_t ks = 0; ks < 4; ++ks) {
                    const uint64_t pk = (ks * 32u) >> 4;          // 16 keys along the P row
                    const uint64_t vk = (ks * 16u * kRow) >> 4;    // 16 key rows of V
                    umma(tmem + kColO, dp_lo + pk, dv + vk, ID_PV, ks > 0 ? 1u : 0u);
                    umma(tmem + kColO, dp_hi + pk, dv + vk, ID_PV, 1u);
                }
                umma_commit(bar_o);
            }
        }
        phase ^= 4u << st;
        pending &= ~(4u << st);
        pending |= 32u;  // on a failed V wait nothing commits: the error path's wait times out
        // ---- meanwhile: dequantise tile j + 1 (the C tile is free: S of tile j is done) ----
        if (j + 1 < ntiles) dequant(j + 1);
        fence_proxy_async();
        tc_before_sync();
        if (__syncthreads_or(err)) break;
        tc_after_sync();
        if (j + 1 < ntiles) {
            if (tid == 0) {
                if (j + 3 < ntiles) issue_k(j + 3, st ^ 1u);
                issue_s();
            }
            if (j + 3 < ntiles) pending |= 1u << (st ^ 1u);
            pending |= 16u;
        }
        // ---- fold tile j's output while the tensor cores compute S of tile j + 1 ----
        if (!mbar_wait_bounded(bar_o, (phase >> 5) & 1u)) err = true;
        phase ^= 32u;
        pending &= ~32u;
        tc_after_sync();
        {
            float t[32];
            tmem_ld32(tmem + tlane + kColO + c0, t);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], alpha, t[i]);
        }
        // the V stage is free once P.V is done (read by the tensor cores only)
        if (tid == 0 && j + 2 < ntiles && !err) issue_v(j + 2, st);
        if (j + 2 < ntiles) pending |= 4u << st;
    }

    red[hf * M + row] = l_run;
    tc_before_sync();
    if (__syncthreads_or(err)) {
        // report, then give copies and tensor-core work in flight a bounded chance to finish
        if (tid == 0) atomicOr(a.status, kStatusWaitTimeout);
        for (uint32_t b = 0; b < 6; ++b)
            if (pending & (1u << b)) mbar_wait_bounded(bars + 8u * b, (phase >> b) & 1u);
    } else if (live) {
        const float inv = 1.0f / (red[row] + red[M + row]);
        const uint64_t HQ = (uint64_t)a.heads * G;
        float *dst = a.out + (((uint64_t)s * a.n + qi) * HQ + (uint64_t)h * G + gq) * a.d;
#pragma unroll
        for (uint32_t i = 0; i < 32; ++i)
            if (c0 + i < a.d) dst[c0 + i] = o[i] * inv;
    }
    tc_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

template <int G>
cudaError_t run(const PrefillArgs &a, const Plan &pl, cudaStream_t s) {
    auto kern = prefill_tc_kernel<G>;
    static int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || (int)pl.total > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.total);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = (int)pl.total;
    }
    constexpr uint32_t PB = M / G;
    const dim3 grid((a.n + PB - 1) / PB, a.heads, a.seq_count);
    kern<<<grid, NTH, pl.total, s>>>(a, pl);
    return cudaGetLastError();
}

}  // namespace tc

// The UMMA prefill's shared-memory plan keeps at most two CTAs per SM (each holds 256 of
// the SM's 512 TMEM columns); larger tiles than that are rejected here.
cudaError_t launch_prefill_tc(const PrefillArgs &a, uint32_t max_cent, cudaStream_t s) {
    uint32_t row_stride = 0, scale_stride = 0;
    for (uint32_t h = 0; h < a.heads; ++h) {
        row_stride = row_stride > a.head[h].row_stride ? row_stride : a.head[h].row_stride;
        scale_stride = scale_stride > a.head[h].scale_stride ? scale_stride : a.head[h].scale_stride;
    }
    const tc::Plan pl = tc::make_plan(row_stride, scale_stride, max_cent);
    if (pl.total <= 228u * 1024u / 3u) return cudaErrorInvalidConfiguration;  // would allow 3 CTAs per SM
    switch (a.gqa) {
        case 1: return tc::run<1>(a, pl, s);
        case 2: return tc::run<2>(a, pl, s);
        case 3: return tc::run<3>(a, pl, s);
        case 4: return tc::run<4>(a, pl, s);
        case 5: return tc::run<5>(a, pl, s);
        case 6: return tc::run<6>(a, pl, s);
        case 7: return tc::run<7>(a, pl, s);
        case 8: return tc::run<8>(a, pl, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bgtq
