// Causal prefill attention over the Block-GTQ key cache on tensor cores (sm_100a).
//
// The model path's chunked prefill (src/model/decoder.ts:30-81: compressed_dot, softmax and
// weighted of src/model/compressed-dot.wgsl:14-31 and src/model/attention.wgsl:13-39) for n
// query positions pos_first .. pos_first + n - 1 of every sequence, every query head of every
// KV head: logits = q.k/sqrt(d) with k = reconstruct(codes) (src/reference/production_math.py:
// 27-31), keys after a row's position masked, softmax, P.V (src/reference/attention.py:5-22).
//
// As in decode, keys are never reconstructed: the queries are rotated into the code domain
// (prefill_qrot_kernel), so a key contributes s_g * cent[i][code_i] per code position i.
// One CTA takes BM = 16 * MB positions of one sequence and all G query heads of one KV head
// (warp = 16 positions of one query head) and walks the key tiles up to its last position:
//   - a 64-key tile of packed rows + FP16 scales and the matching FP16 V tile arrive by
//     cp.async.bulk (TMA bulk copies, no multicast) on mbarriers, two tiles in flight;
//   - all threads dequantise the packed tile into shared memory as code-domain values split
//     into FP16 high and low halves (about 22 significant bits), rows chunk-swizzled;
//   - each warp computes S = Q C^T on the tensor cores (mma.sync m16n8k16, FP32 accumulate)
//     as Q_hi C_hi + Q_hi C_lo + Q_lo C_hi, keeps an online softmax in registers (scores in
//     log2 units, probabilities scaled by 2^12) and accumulates O += P_hi V + P_lo V with V
//     fragments from ldmatrix.trans on the swizzled V tile.
// Every mbarrier wait is bounded; a timeout sets a bit of the device status word and the
// CTA stops after waiting (again bounded) for its copies in flight.
#include <cuda_fp16.h>

#include "attention_impl.cuh"

namespace bgtq {
namespace pre {

using attn::bulk_g2s;
using attn::fence_barrier_init;
using attn::fence_proxy_async;
using attn::kLog2e;
using attn::kPShift;
using attn::mbar_expect_tx;
using attn::mbar_init;
using attn::mbar_wait_bounded;
using attn::mma_16816;
using attn::smem_u32;

constexpr int D = 64;                  // head dim of the prefill kernel (code positions)
constexpr int BN = 64;                 // keys per tile
constexpr uint32_t kTileHalfRow = D * 2;  // bytes of one FP16 row of a C or V tile
constexpr uint32_t kCTile = BN * kTileHalfRow;

// Per-code-position decode word: bits 0-7 byte of the code in the packed row, bit 8 high
// nibble, bit 9 whole byte, bit 10 position past the head dim (value 0), bits 12-14 group,
// bits 16-31 first entry of the position's compact codebook.
constexpr uint32_t kMetaHigh = 1u << 8, kMetaByte = 1u << 9, kMetaZero = 1u << 10;

template <int G>
struct Shape {
    static constexpr int MB = G >= 8 ? 1 : 8 / G;  // 16-position blocks per CTA
    static constexpr int W = G * MB;               // warps
    static constexpr int BM = 16 * MB;             // positions per CTA
};

struct Plan {
    uint32_t cent, meta, chi, clo, kst, vst, bars, total;
    uint32_t kbytes, sbytes, kstage, cent_alloc;
};

inline Plan make_plan(uint32_t row_stride, uint32_t scale_stride, uint32_t n_cent) {
    Plan p{};
    uint32_t off = 0;
    p.cent = off;
    p.cent_alloc = n_cent + 16u;
    off = attn::align16(off + 4u * p.cent_alloc);
    p.meta = off;
    off = attn::align128(off + 4u * D);
    p.chi = off;
    off += kCTile;
    p.clo = off;
    off += kCTile;
    p.kbytes = BN * row_stride;
    p.sbytes = BN * scale_stride * 2u;
    p.kstage = attn::align128(attn::align16(p.kbytes) + attn::align16(p.sbytes));
    p.kst = off;
    off += 2u * p.kstage;
    p.vst = off;
    off += 2u * kCTile;
    p.bars = off;
    off += 4u * 8u;  // K barriers 0, 1; V barriers 0, 1
    p.total = attn::align16(off);
    return p;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// FP32 pair -> FP16 high halves and FP16 low halves (the rounding residual).
__device__ __forceinline__ void split2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 f = __half22float2(h);
    const float2 r = __ffma2_rn(f, make_float2(-1.0f, -1.0f), make_float2(x, y));  // exact x - f
    const __half2 l = __floats2half2_rn(r.x, r.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Code-domain queries: qt[s][t][hq][i] = sum_{j in group(i)} R[i][j] q[perm[j]] * log2(e)/sqrt(d)
// (after split-half RoPE at the query's position when a table is given).  One CTA rotates
// kQrotTokens positions x G query heads of KV head blockIdx.y of sequence blockIdx.z: the
// head's rotation (transposed) and the query rows (row-major, odd stride: conflict-free
// stores and reads) are staged in shared memory, and each thread accumulates 4 outputs x 8
// rows over all j in ascending order.  R[i][j] is exactly 0 outside group(i) (the layout
// check enforces it), so the dense sum rounds exactly like the sum over the group alone.
constexpr uint32_t kQrotTokens = 16, kQrotThreads = 256, kQrotRowsMax = kQrotTokens * kMaxRows;  // 128 rows
constexpr uint32_t kQrotStride = D + 1;  // floats per staged query row

__global__ void __launch_bounds__(kQrotThreads) prefill_qrot_kernel(const __grid_constant__ PrefillArgs a) {
    extern __shared__ __align__(16) float qsm[];
    const uint32_t t0 = blockIdx.x * kQrotTokens, h = blockIdx.y, s = blockIdx.z, G = a.gqa, d = a.d;
    const AttnHead &hd = a.head[h];
    const uint64_t HQ = (uint64_t)a.heads * G;
    const uint32_t nt = min(kQrotTokens, a.n - t0), rows = nt * G;
    const uint32_t tid = threadIdx.x;
    float *rt = qsm;                                            // [D][D]: rt[j][i] = R[i][j] (0 past d)
    float *qs = qsm + D * D;                                    // [kQrotRowsMax][kQrotStride] query rows
    uint32_t *perm = reinterpret_cast<uint32_t *>(qs + kQrotRowsMax * kQrotStride);  // [D]
    for (uint32_t idx = tid; idx < (uint32_t)(D * D); idx += kQrotThreads) {
        const uint32_t j = idx / D, i = idx % D;
        rt[idx] = (i < d && j < d) ? hd.rot[(uint64_t)i * d + j] : 0.0f;
    }
    if (tid < (uint32_t)D) perm[tid] = tid < d ? hd.perm[tid] : 0u;
    {
        const float *qg = a.q + (((uint64_t)s * a.n + t0) * HQ + (uint64_t)h * G) * d;
#pragma unroll 8
        for (uint32_t idx = tid; idx < kQrotRowsMax * D; idx += kQrotThreads) {
            const uint32_t row = idx / D, i = idx % D;
            float v = 0.0f;
            if (row < rows && i < d) {
                const uint32_t t = row / G, g = row - t * G;
                v = attn::rope_elem(qg + ((uint64_t)t * HQ + g) * d, i, d, a.pos_first + t0 + t, a.rope);
            }
            qs[row * kQrotStride + i] = v;
        }
    }
    __syncthreads();
    // thread tile: outputs 4*ib .. 4*ib+3, rows 8*rb .. 8*rb+7
    const uint32_t ib = tid % 16, rb = tid / 16;
    float acc[4][8];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[x][r] = 0.0f;
    if (8 * rb < rows) {
        const float *qr = qs + 8 * rb * kQrotStride;
        for (uint32_t j = 0; j < d; ++j) {
            const float4 rv = *reinterpret_cast<const float4 *>(rt + j * D + 4 * ib);
            const uint32_t pj = perm[j];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float qv = qr[r * kQrotStride + pj];
                acc[0][r] = fmaf(rv.x, qv, acc[0][r]);
                acc[1][r] = fmaf(rv.y, qv, acc[1][r]);
                acc[2][r] = fmaf(rv.z, qv, acc[2][r]);
                acc[3][r] = fmaf(rv.w, qv, acc[3][r]);
            }
        }
    }
    const float qscale = kLog2e / sqrtf((float)d);
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const uint32_t row = 8 * rb + r;
        if (row < rows) {
            const uint32_t t = row / G, g = row - t * G;
            float4 o;
            o.x = 4 * ib + 0 < d ? acc[0][r] * qscale : 0.0f;
            o.y = 4 * ib + 1 < d ? acc[1][r] * qscale : 0.0f;
            o.z = 4 * ib + 2 < d ? acc[2][r] * qscale : 0.0f;
            o.w = 4 * ib + 3 < d ? acc[3][r] * qscale : 0.0f;
            *reinterpret_cast<float4 *>(a.qt + (((uint64_t)s * a.n + t0 + t) * HQ + (uint64_t)h * G + g) * D + 4 * ib) = o;
        }
    }
}

template <int G>
__global__ void __launch_bounds__(Shape<G>::W * 32, 2) prefill_kernel(const __grid_constant__ PrefillArgs a,
                                                                   const Plan pl) {
    constexpr int MB = Shape<G>::MB, NTH = Shape<G>::W * 32, BM = Shape<G>::BM;
    const uint32_t qb = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const AttnHead &hd = a.head[h];
    const uint32_t seq = a.seq_first + s;
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    const int gq = w % G, mb = w / G;
    const int g = lane >> 2, c = lane & 3;
    (void)MB;

    const uint32_t q0 = qb * BM;                               // first query of the CTA
    const uint32_t nq = min((uint32_t)BM, a.n - q0);
    const uint32_t len = a.lengths[seq];
    const uint32_t last_pos = a.pos_first + q0 + nq - 1;
    const uint32_t kend = min(last_pos + 1, len);              // keys [0, kend) are visible
    const uint32_t ntiles = (kend + BN - 1) / BN;
    const uint32_t wq0 = q0 + 16u * mb;                        // first query of this warp
    const uint32_t wpos0 = a.pos_first + wq0;                  // its position
    const bool wlive = wq0 < a.n;
    const uint32_t wlast = min(wpos0 + 15u, last_pos);         // last live position of the warp

    extern __shared__ __align__(128) unsigned char smem[];
    float *cent_s = reinterpret_cast<float *>(smem + pl.cent);
    uint32_t *meta_s = reinterpret_cast<uint32_t *>(smem + pl.meta);
    const uint32_t chi = smem_u32(smem + pl.chi), clo = smem_u32(smem + pl.clo);
    const uint32_t bars = smem_u32(smem + pl.bars);

    // ---- prologue: codebooks, decode words, barriers ----
    for (uint32_t i = tid; i < pl.cent_alloc; i += NTH) cent_s[i] = i < hd.n_cent ? hd.cent[i] : 0.0f;
    if (tid < D) {
        const uint32_t i = tid;
        uint32_t m = kMetaZero;
        if (i < a.d) {
            const uint32_t grp = hd.group_of[i];
            if (i < hd.ns) m = (i >> 1) | ((i & 1u) ? kMetaHigh : 0u);
            else m = (hd.ns / 2 + (i - hd.ns)) | kMetaByte;
            m |= grp << 12 | (uint32_t)hd.cb_base[i] << 16;
        }
        meta_s[i] = m;
    }
    if (tid < 4) mbar_init(bars + 8u * tid, 1u);
    fence_barrier_init();
    __syncthreads();

    const unsigned char *kbase = hd.k + (uint64_t)seq * hd.k_seq_stride;
    const unsigned char *sbase = reinterpret_cast<const unsigned char *>(hd.scales + (uint64_t)seq * hd.s_seq_stride);
    const unsigned char *vbase = static_cast<const unsigned char *>(hd.v) + (uint64_t)seq * hd.v_seq_stride;
    const uint32_t row_stride = hd.row_stride, srow = hd.scale_stride * 2u;
    const uint32_t soff = attn::align16(pl.kbytes);
    // whole tiles: capacity is padded to 64 rows and zero-filled
    // this head's tile sizes: the plan's buffers fit the widest head of the launch
    const uint32_t kb_h = BN * row_stride, sb_h = BN * srow;
    auto issue_k = [&](uint32_t j, uint32_t st) {
        const uint32_t bar = bars + 8u * st, dst = smem_u32(smem + pl.kst + st * pl.kstage);
        fence_proxy_async();
        mbar_expect_tx(bar, kb_h + sb_h);
        bulk_g2s(dst, kbase + (uint64_t)j * BN * row_stride, kb_h, bar);
        bulk_g2s(dst + soff, sbase + (uint64_t)j * BN * srow, sb_h, bar);
    };
    auto issue_v = [&](uint32_t j, uint32_t st) {
        const uint32_t bar = bars + 16u + 8u * st, dst = smem_u32(smem + pl.vst + st * kCTile);
        fence_proxy_async();
        mbar_expect_tx(bar, kCTile);
        bulk_g2s(dst, vbase + (uint64_t)j * BN * kTileHalfRow, kCTile, bar);
    };
    uint32_t pending = 0;  // bit st: K stage st in flight; bit 2 + st: V stage st in flight
    for (uint32_t j = 0; j < 2 && j < ntiles; ++j) {
        if (tid == 0) {
            issue_k(j, j);
            issue_v(j, j);
        }
        pending |= (1u << j) | (4u << j);
    }

    // ---- this warp's queries as FP16 high / low A fragments ----
    uint32_t qh[4][4], ql[4][4];
    {
        const uint64_t HQ = (uint64_t)a.heads * G;
        auto qrow = [&](uint32_t r) -> const float * {
            return a.qt + (((uint64_t)s * a.n + wq0 + r) * HQ + (uint64_t)h * G + gq) * D;
        };
        const bool r0 = wq0 + g < a.n, r1 = wq0 + g + 8 < a.n;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const int c0 = 16 * ks + 2 * c;
            const float2 z = make_float2(0.0f, 0.0f);
            const float2 v0 = r0 ? *reinterpret_cast<const float2 *>(qrow(g) + c0) : z;
            const float2 v1 = r1 ? *reinterpret_cast<const float2 *>(qrow(g + 8) + c0) : z;
            const float2 v2 = r0 ? *reinterpret_cast<const float2 *>(qrow(g) + c0 + 8) : z;
            const float2 v3 = r1 ? *reinterpret_cast<const float2 *>(qrow(g + 8) + c0 + 8) : z;
            split2(v0.x, v0.y, qh[ks][0], ql[ks][0]);
            split2(v1.x, v1.y, qh[ks][1], ql[ks][1]);
            split2(v2.x, v2.y, qh[ks][2], ql[ks][2]);
            split2(v3.x, v3.y, qh[ks][3], ql[ks][3]);
        }
    }

    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    const int mi = lane >> 3, ri = lane & 7;
    uint32_t phase = 0;
    bool err = false;  // this thread saw a wait time out; CTA-wide decisions use __syncthreads_or

    for (uint32_t j = 0; j < ntiles; ++j) {
        const uint32_t st = j & 1u;
        // ---- dequantise packed tile j into FP16 high / low code-domain values ----
        if (!mbar_wait_bounded(bars + 8u * st, (phase >> st) & 1u)) err = true;
        phase ^= 1u << st;
        pending &= ~(1u << st);
        const unsigned char *kt = smem + pl.kst + st * pl.kstage;
        for (uint32_t it = tid; it < BN * 8u; it += NTH) {
            const uint32_t key = it & (BN - 1), ch = it >> 6;
            const unsigned char *row = kt + key * row_stride;
            const uint16_t *sc = reinterpret_cast<const uint16_t *>(kt + soff + key * srow);
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t mt = meta_s[ch * 8 + e];
                const uint32_t byte = row[mt & 0xffu];
                const uint32_t code = (mt & kMetaByte) ? byte : ((mt & kMetaHigh) ? byte >> 4 : byte & 15u);
                const float scale = __half2float(__ushort_as_half(sc[(mt >> 12) & 7u]));
                v[e] = (mt & kMetaZero) ? 0.0f : cent_s[(mt >> 16) + code] * scale;
            }
            uint4 hi, lo;
            split2(v[0], v[1], hi.x, lo.x);
            split2(v[2], v[3], hi.y, lo.y);
            split2(v[4], v[5], hi.z, lo.z);
            split2(v[6], v[7], hi.w, lo.w);
            const uint32_t at = key * kTileHalfRow + ((ch ^ (key & 7u)) << 4);
            *reinterpret_cast<uint4 *>(smem + pl.chi + at) = hi;
            *reinterpret_cast<uint4 *>(smem + pl.clo + at) = lo;
        }
        if (__syncthreads_or(err)) break;
        if (tid == 0 && j + 2 < ntiles) issue_k(j + 2, st);
        if (j + 2 < ntiles) pending |= 1u << st;

        const uint32_t k0 = j * BN;
        const bool active = wlive && k0 <= wlast;
        if (active) {
            // ---- S = Q_hi C_hi + Q_hi C_lo + Q_lo C_hi ----
            // Each 16-dim step starts from zero with the two small cross terms, adds the
            // large term last, and is summed into S in FP32 (round to nearest), so the
            // tensor cores' accumulation rounding acts once per step on a partial sum
            // rather than on the running logit.
            float sf[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) sf[nt][0] = sf[nt][1] = sf[nt][2] = sf[nt][3] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                float tp[8][4];
#pragma unroll
                for (int nt = 0; nt < 8; ++nt) tp[nt][0] = tp[nt][1] = tp[nt][2] = tp[nt][3] = 0.0f;
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    const uint32_t key = (uint32_t)((2 * np + (mi >> 1)) * 8 + ri);
                    const uint32_t ch = (uint32_t)(2 * ks + (mi & 1));
                    const uint32_t off = key * kTileHalfRow + ((ch ^ (key & 7u)) << 4);
                    uint32_t b0, b1, b2, b3, e0, e1, e2, e3;
                    ldsm_x4(chi + off, b0, b1, b2, b3);
                    ldsm_x4(clo + off, e0, e1, e2, e3);
                    mma_16816(tp[2 * np], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b0, b1);
                    mma_16816(tp[2 * np], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], e0, e1);
                    mma_16816(tp[2 * np], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b0, b1);
                    mma_16816(tp[2 * np + 1], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b2, b3);
                    mma_16816(tp[2 * np + 1], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], e2, e3);
                    mma_16816(tp[2 * np + 1], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b2, b3);
                }
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sf[nt][e] += tp[nt][e];
            }
            // ---- mask: keys after a row's position, past the length, rows past n ----
            if (k0 + BN - 1 > wpos0 || k0 + BN > len || wq0 + 16 > a.n) {
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t r = (uint32_t)(g + (e >> 1) * 8);
                        const uint32_t key = k0 + nt * 8 + 2 * c + (e & 1);
                        const bool ok = wq0 + r < a.n && key <= wpos0 + r && key < len;
                        sf[nt][e] = ok ? sf[nt][e] : -INFINITY;
                    }
            }
            // ---- online softmax per row (rows g and g + 8 of this lane) ----
            float alpha[2];
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                float mx = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(sf[nt][2 * hr], sf[nt][2 * hr + 1]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mnew = fmaxf(m[hr], mx);
                alpha[hr] = mnew == -INFINITY ? 1.0f : attn::ex2(m[hr] - mnew);
                m[hr] = mnew;
                const float mref = mnew == -INFINITY ? 0.0f : mnew - kPShift;
                float ps = 0.0f;
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float x = sf[nt][2 * hr + e];
                        const float p = attn::ex2(x - mref);  // masked: 2^-inf = 0
                        sf[nt][2 * hr + e] = p;
                        ps += p;
                    }
                l[hr] = fmaf(l[hr], alpha[hr], ps);
            }
            // ---- O = alpha O + (P_hi V + P_lo V), the tile's product summed from zero ----
            float tv[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) tv[nt][0] = tv[nt][1] = tv[nt][2] = tv[nt][3] = 0.0f;
            if (!mbar_wait_bounded(bars + 16u + 8u * st, (phase >> (2 + st)) & 1u)) err = true;
            const uint32_t vs = smem_u32(smem + pl.vst + st * kCTile);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t ph[4], plo[4];
                split2(sf[2 * ks][0], sf[2 * ks][1], ph[0], plo[0]);
                split2(sf[2 * ks][2], sf[2 * ks][3], ph[1], plo[1]);
                split2(sf[2 * ks + 1][0], sf[2 * ks + 1][1], ph[2], plo[2]);
                split2(sf[2 * ks + 1][2], sf[2 * ks + 1][3], ph[3], plo[3]);
                const uint32_t tok = (uint32_t)(ks * 16 + (mi & 1) * 8 + ri);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    const uint32_t ch = (uint32_t)(2 * np + (mi >> 1));
                    uint32_t b0, b1, b2, b3;
                    attn::ldsm_x4_trans(vs + tok * kTileHalfRow + ((ch ^ (tok & 7u)) << 4), b0, b1, b2, b3);
                    mma_16816(tv[2 * np], plo[0], plo[1], plo[2], plo[3], b0, b1);
                    mma_16816(tv[2 * np], ph[0], ph[1], ph[2], ph[3], b0, b1);
                    mma_16816(tv[2 * np + 1], plo[0], plo[1], plo[2], plo[3], b2, b3);
                    mma_16816(tv[2 * np + 1], ph[0], ph[1], ph[2], ph[3], b2, b3);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                o[nt][0] = fmaf(o[nt][0], alpha[0], tv[nt][0]);
                o[nt][1] = fmaf(o[nt][1], alpha[0], tv[nt][1]);
                o[nt][2] = fmaf(o[nt][2], alpha[1], tv[nt][2]);
                o[nt][3] = fmaf(o[nt][3], alpha[1], tv[nt][3]);
            }
        }
        phase ^= 4u << st;
        pending &= ~(4u << st);
        if (__syncthreads_or(err)) break;
        if (tid == 0 && j + 2 < ntiles) issue_v(j + 2, st);
        if (j + 2 < ntiles) pending |= 4u << st;
    }
    if (__syncthreads_or(err)) {
        // report, then give the copies still in flight a bounded chance to land
        if (tid == 0) atomicOr(a.status, kStatusWaitTimeout);
        for (uint32_t b = 0; b < 4; ++b)
            if (pending & (1u << b)) mbar_wait_bounded(bars + 8u * b, (phase >> b) & 1u);
        return;
    }

    // ---- normalise and store ----
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
        l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
    }
    if (!wlive) return;
    const uint64_t HQ = (uint64_t)a.heads * G;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const uint32_t q = wq0 + g + 8 * hr;
        if (q >= a.n) continue;
        const float inv = 1.0f / l[hr];
        float *dst = a.out + (((uint64_t)s * a.n + q) * HQ + (uint64_t)h * G + gq) * a.d;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const uint32_t col = nt * 8 + 2 * c;
            if (col < a.d) dst[col] = o[nt][2 * hr] * inv;
            if (col + 1 < a.d) dst[col + 1] = o[nt][2 * hr + 1] * inv;
        }
    }
}

template <int G>
cudaError_t run(const PrefillArgs &a, const Plan &pl, cudaStream_t s) {
    auto kern = prefill_kernel<G>;
    static int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || (int)pl.total > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.total);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = (int)pl.total;
    }
    const dim3 grid((a.n + Shape<G>::BM - 1) / Shape<G>::BM, a.heads, a.seq_count);
    kern<<<grid, Shape<G>::W * 32, pl.total, s>>>(a, pl);
    return cudaGetLastError();
}

}  // namespace pre

cudaError_t launch_prefill(const PrefillArgs &a, uint32_t max_cent, int umma, cudaStream_t s) {
    if (!a.n || !a.seq_count) return cudaSuccess;
    uint32_t row_stride = 0, scale_stride = 0;
    for (uint32_t h = 0; h < a.heads; ++h) {
        row_stride = row_stride > a.head[h].row_stride ? row_stride : a.head[h].row_stride;
        scale_stride = scale_stride > a.head[h].scale_stride ? scale_stride : a.head[h].scale_stride;
    }
    // one plan for all heads, sized for the widest; each head copies its own tile sizes
    const pre::Plan pl = pre::make_plan(row_stride, scale_stride, max_cent);
    {
        const size_t qsmem = sizeof(float) * ((size_t)pre::D * pre::D + (size_t)pre::kQrotRowsMax * pre::kQrotStride + pre::D);
        static int configured[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64 || (int)qsmem > configured[dev]) {
            cudaError_t e = cudaFuncSetAttribute(pre::prefill_qrot_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)qsmem);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) configured[dev] = (int)qsmem;
        }
        pre::prefill_qrot_kernel<<<dim3((a.n + pre::kQrotTokens - 1) / pre::kQrotTokens, a.heads, a.seq_count),
                                   pre::kQrotThreads, qsmem, s>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (umma) return launch_prefill_tc(a, max_cent, s);
    switch (a.gqa) {
        case 1: return pre::run<1>(a, pl, s);
        case 2: return pre::run<2>(a, pl, s);
        case 3: return pre::run<3>(a, pl, s);
        case 4: return pre::run<4>(a, pl, s);
        case 5: return pre::run<5>(a, pl, s);
        case 6: return pre::run<6>(a, pl, s);
        case 7: return pre::run<7>(a, pl, s);
        case 8: return pre::run<8>(a, pl, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bgtq
