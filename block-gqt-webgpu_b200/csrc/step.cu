// Persistent decode step of the model path: one token per sequence through every layer of a
// decoder (src/model/decoder.ts:31-81 decode, shaders of src/model/kernels.wgsl:11-54 and
// the compressed-K attention) in ONE cooperative launch.
//
// Per layer, phases separated by grid-wide barriers (every CTA is resident: cooperative
// launch), each spread over all CTAs:
//   1. RMSNorm + Q/K/V projection (+ bias)            GEMV over the residual stream h
//   2. K/V append: split-half RoPE on K at the token's row, Block-GTQ encode into the packed
//      store (bit for bit the append kernels' arithmetic: this file is compiled with
//      -fmad=false like encode.cu), V to the FP16 store, lengths moved on; the appending
//      warp then scores its new key against the pair's query rows itself (the key
//      reconstructed from its codes and scales) and leaves the new row's partial.  In the
//      same phase the other CTAs rotate each (sequence, KV head)'s queries into the code
//      domain (RoPE at the new row, block rotation: the query rotation kernel's arithmetic)
//      and run the attention tasks: (KV head, sequence, range of the keys stored before this
//      step), each the decode-attention body over its range leaving a partial.  No task
//      reads a row this phase writes, so none waits for the append.
//   3. every CTA merges the pairs' partials (the attention kernel's split-KV merge), then
//      o_proj + residual add into h
//   4. RMSNorm + gate/up + SiLU gating
//   5. down_proj + residual add into h
// then the final RMSNorm + lm_head.  The stand-alone path runs the same work as seven
// launches per layer; a decode step of a small model is a chain of microsecond kernels, and
// here each kernel boundary becomes a grid barrier (one atomic per CTA and a poll of one L2
// word) with the next phase's weights already requested into L2 (bulk L2 prefetch) while
// the phase before runs.
//
// Coherence: data produced inside the launch (activations, lengths, K/V rows, partials)
// is read through L2 (ld.global.cg) or by bulk copies after a generic-to-async proxy fence;
// weights and tables, never written, through the read-only path.  Every barrier wait is
// bounded: a CTA whose wait runs out sets the device status word and an abort word that
// every other CTA polls, so the launch ends with an error status instead of hanging; the
// abort word stays set, and the decoder object then refuses further steps.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "attention_impl.cuh"
#include "encode_impl.cuh"
#include "objects.h"

namespace bgtq {
namespace step {

constexpr int kThreads = attn::kThreads;  // the attention body's CTA: 4 warps
constexpr int kWarps = kThreads / 32;
constexpr int kChunks = 4;                  // 16-byte weight chunks per lane and row in flight
constexpr uint32_t kSpinLimit = 1u << 22;   // barrier polls (32 ns sleeps after the first 64): about a second
constexpr int D = 64;                       // head dim of the step kernel
constexpr uint32_t kQrawFloats = kMaxRows * D;
constexpr uint32_t kQtFloats = D * 8;
constexpr uint32_t kBarriersPerLayer = 5;

// Weights and stores of one layer (device resident, written once at decoder creation).
struct Layer {
    const float *ln1, *qkv_b, *ln2;
    const __half *w_qkv, *w_o, *w_gu, *w_down;
    alignas(16) KvRopeArgs kv;  // append: K/V sources in the Q/K/V buffer, stores, RoPE table
    alignas(16) AttnArgs att;   // attention over the layer's stores, output into the attention buffer
    unsigned char pad[16];      // the copies of kv / att round up to 16 bytes
};
constexpr uint32_t kKvBytes = (sizeof(KvRopeArgs) + 15) & ~15u;
constexpr uint32_t kAttBytes = (sizeof(AttnArgs) + 15) & ~15u;

struct Args {
    const Layer *layers;
    uint32_t n_layers, batch, hidden, q_heads, kv_heads, gqa, d, inter, vocab, qkv_row;
    float eps;
    const int64_t *tokens;   // [B] token ids (null: h already holds the embeddings)
    const float *emb;        // [vocab][hidden] FP32 embedding rows
    float *h;                // [B][hidden] residual stream
    float *qkv;              // [B][qkv_row]
    float *att;              // [B][q_heads * d]
    float *act;              // [B][inter]
    float *logits;           // [B][vocab]
    const float *final_norm;
    const __half *lm_head;   // [vocab][hidden]
    attn::Plan pl;           // attention shared-memory plan (offsets from the dynamic base)
    uint32_t task_tokens;    // tokens per attention task (a multiple of the CTA tile)
    uint32_t enc_stage;      // bytes of staged encode tables (0: read from global memory)
    uint32_t off_e, off_r, off_q;  // dynamic shared memory: encode tables, rotation, query scratch
    uint32_t off_part;             // the attention partials' copy in the GEMV region (0: read through L2)
    uint32_t off_lk;               // the first attention pair's codebooks (lookup layout, 1024-aligned)
    uint32_t *bar;           // grid barrier: 64-bit arrival counter, abort word
    unsigned long long bar_base;  // the arrival counter at launch
    uint32_t *status;
    uint32_t len_new[kMaxRows];  // per sequence: its length once this step's token is appended
    unsigned long long *trace;   // optional: global-timer stamps of CTA 0 at each phase end
};

// CTA 0's global-timer stamp k (the phase breakdown of bgtq_decoder_trace).
__device__ __forceinline__ void stamp(const Args &A, uint32_t k) {
    if (A.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        A.trace[k] = t;
    }
}

// ---- coherent (L2) loads of data written earlier in the launch ----
__device__ __forceinline__ float ldcg(const float *p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ldcg(const uint32_t *p) { return __ldcg(p); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// An mbarrier's shared memory is repurposed (the phases share regions) or initialised again
// (once per layer) only after it is invalidated.
__device__ __forceinline__ void mbar_inval(uint32_t bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// Generic-proxy global writes of this thread before / async-proxy (bulk copy) reads after.
__device__ __forceinline__ void fence_proxy_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Grid-wide barrier over the launch's CTAs (all resident): bar[0..1] is a 64-bit arrival
// counter that only grows (the host passes the value it has at launch, bar_base), bar[2]
// the abort word.  Barrier k of the launch completes when the counter reaches
// bar_base + (k + 1) * CTAs: one atomic per CTA, then polls of one L2 word, no reset.
// Returns false when this CTA's wait ran out or another CTA aborted: the caller returns.
__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool grid_barrier(uint32_t *bar, unsigned long long target, uint32_t *status) {
    __shared__ uint32_t s_ok;
    unsigned long long *count = reinterpret_cast<unsigned long long *>(bar);
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t ok = 1;
        // the arrival releases this CTA's writes (ordered before it by the CTA barrier); no
        // return value, so no round trip before the polls start
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(count) : "memory");
        uint32_t it = 0;
        while (ld_acquire64(count) < target) {
            if (++it > kSpinLimit || ((it & 63u) == 0 && ld_acquire(bar + 2))) {
                ok = 0;
                break;
            }
            if (it > 64u) __nanosleep(32);
        }
        if (ok && ld_acquire(bar + 2)) ok = 0;
        if (!ok) {
            atomicOr(status, kStatusWaitTimeout);
            atomicExch(bar + 2, 1u);
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// Asks L2 for share `part` of `parts` of `bytes` (a multiple of 16) at p (16-byte aligned):
// bulk prefetches issued by thread `issuer`, so a matrix a later phase streams is on chip when
// it starts.  By default every CTA takes its share.
__device__ __forceinline__ void prefetch_l2(const void *p, uint64_t bytes, uint32_t issuer = 0,
                                            uint32_t part = ~0u, uint32_t parts = 0) {
    if (threadIdx.x != issuer || !p || !bytes) return;
    if (!parts) {
        part = blockIdx.x;
        parts = gridDim.x;
    }
    const uint64_t per = ((bytes + parts - 1) / parts + 15u) & ~15ull;
    const uint64_t b0 = (uint64_t)part * per;
    if (b0 >= bytes) return;
    uint64_t n = bytes - b0 < per ? bytes - b0 : per;
    const unsigned char *q = static_cast<const unsigned char *>(p) + b0;
    while (n) {  // pieces below 2^20 bytes
        const uint32_t c = (uint32_t)(n < (1u << 20) ? n : (1u << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(c) : "memory");
        q += c;
        n -= c;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// FP16 x 8 (one 16-byte chunk) dotted with 8 FP32 activations (explicit FMAs).
__device__ __forceinline__ float dot8(const uint4 w, const float *x) {
    const __half2 *hh = reinterpret_cast<const __half2 *>(&w);
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(hh[k]);
        acc = fmaf(f.x, x[2 * k], acc);
        acc = fmaf(f.y, x[2 * k + 1], acc);
    }
    return acc;
}

// One GEMV phase over the whole grid (the stand-alone gemv_kernel's arithmetic):
//   MODE 0  y[b][r]  = W[r] . rmsnorm(x[b]) (+ bias[r])
//   MODE 1  y[b][r] += W[r] . x[b]
//   MODE 2  y[b][r]  = silu(W[r] . n) * (W[out + r] . n),  n = rmsnorm(x[b])
// Each CTA stages the B activation rows (normalised for MODES 0 and 2) in shared memory xs;
// each warp owns RPW output rows at a time, all of their weight chunks of a pass loaded
// before the first FMA.  tok != null: x[b] is the embedding row of token tok[b], and CTA 0
// also writes it to h (the residual stream's start).
// One pass of a warp's weights: RPW rows (gate and up rows for MODE 2) x KC 16-byte chunks per
// lane.  The first pass of a GEMV phase is loaded before the grid barrier that opens it
// (weights never change), so its latency overlaps the barrier.
template <int MODE, int RPW, int KC>
struct Pass {
    static constexpr int NW = MODE == 2 ? 2 : 1;
    uint4 v[RPW][NW][KC];
    __device__ __forceinline__ void load(const __half *w, uint32_t in, uint32_t out, uint32_t r0, uint32_t base) {
        const uint32_t chunks = in / 8, lane = threadIdx.x & 31u;
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int u = 0; u < NW; ++u)
#pragma unroll
                for (int c = 0; c < KC; ++c) {
                    const uint32_t row = r0 + r, ch = base + lane + 32u * c;
                    v[r][u][c] = row < out && ch < chunks
                                     ? __ldg(reinterpret_cast<const uint4 *>(w + (uint64_t)(row + u * out) * in) + ch)
                                     : make_uint4(0, 0, 0, 0);
                }
    }
    // the first pass of this warp's first rows
    __device__ __forceinline__ void preload(const __half *w, uint32_t in, uint32_t out) {
        load(w, in, out, (blockIdx.x * kWarps + (threadIdx.x >> 5)) * RPW, 0);
    }
};

// The attention output rows of every (sequence, query head) into xs [B][heads * gqa * d],
// merged from the attention tasks' partials (nt ranges per pair): per row the maximum, the
// weights 2^(m_i - M) and the sum, then the weighted outputs - the attention kernel's
// split merge, same arithmetic and order, done by every CTA of the phase that consumes it
// instead of by the last task of each pair (whose serial L2 round trips would sit on the
// attention phase's critical path).  The partials (nt slots, contiguous) come into shared
// memory with one bulk copy when part_s is given, so the merge itself reads shared memory.
// wts: shared scratch of B * heads * gqa * (2 nt + 2) floats.
struct Merge {
    const AttnArgs *a;  // null: no merge (the activations are read as they are)
    uint32_t nt;
    float *part_s;      // shared copy of the partials, or null (read through L2)
    uint64_t *bar;
};

__device__ __forceinline__ void merge_rows(const Args &A, const Merge &m, float *xs, float *wts) {
    const AttnArgs &a = *m.a;
    const uint32_t B = A.batch, H = a.heads, R = a.rows, d = A.d, tid = threadIdx.x, nt = m.nt;
    const uint32_t rows = B * H * R, W = 2 * nt + 2;  // per row: nt weights, nt sums, maximum, sum
    const uint32_t sstride = a.seq_count * H * R * (d + 2), n = nt * sstride;
    const float *src = a.part;
    bool shared_copy = false;
    if (m.part_s) {
        const uint32_t bulk = (n * 4u) & ~15u, bar = attn::smem_u32(m.bar);
        if (tid == 0) {
            fence_proxy_global();  // written by other CTAs' generic stores, read by a bulk copy
            attn::mbar_init(bar, 1u);
            attn::fence_barrier_init();
            attn::fence_proxy_async();
            attn::mbar_expect_tx(bar, bulk);
            attn::bulk_g2s(attn::smem_u32(m.part_s), a.part, bulk, bar);
        }
        for (uint32_t i = bulk / 4u + tid; i < n; i += kThreads) m.part_s[i] = ldcg(a.part + i);
        __syncthreads();
        shared_copy = __syncthreads_and(attn::mbar_wait_bounded(bar, 0u));
        if (!shared_copy && tid == 0) atomicOr(A.status, kStatusWaitTimeout);
        if (shared_copy && tid == 0) mbar_inval(bar);
        if (shared_copy) src = m.part_s;
    }
    auto ld = [&](uint32_t i) { return shared_copy ? src[i] : ldcg(src + i); };
    for (uint32_t idx = tid; idx < rows * nt; idx += kThreads) {
        const uint32_t row = idx / nt, sp = idx % nt;  // row = (b * H + hd) * R + r
        const uint32_t at = sp * sstride + row * (d + 2) + d;
        wts[row * W + sp] = ld(at);
        wts[row * W + nt + sp] = ld(at + 1);
    }
    __syncthreads();
    for (uint32_t row = tid; row < rows; row += kThreads) {
        float *wr = wts + row * W;
        float M = -INFINITY;
        for (uint32_t sp = 0; sp < nt; ++sp) M = fmaxf(M, wr[sp]);
        float L = 0.0f;
        for (uint32_t sp = 0; sp < nt; ++sp) {
            const float mv = wr[sp];
            const float f = mv == -INFINITY ? 0.0f : attn::ex2(mv - M);
            L = fmaf(wr[nt + sp], f, L);
            wr[sp] = f;
        }
        wr[2 * nt] = M;
        wr[2 * nt + 1] = L;
    }
    __syncthreads();
    for (uint32_t idx = tid; idx < rows * d; idx += kThreads) {
        const uint32_t row = idx / d, dd = idx % d, base = row * (d + 2) + dd;
        const float *wr = wts + row * W;
        float Ov = 0.0f;
        for (uint32_t sp0 = 0; sp0 < nt; sp0 += 8) {
            float v[8];
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) v[k] = sp0 + k < nt ? ld(base + (sp0 + k) * sstride) : 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
                if (sp0 + k < nt) Ov = fmaf(v[k], wr[sp0 + k], Ov);
        }
        xs[idx] = Ov / wr[2 * nt + 1];  // row-major [b][hd][r][d] = [b][query head][d]
    }
    __syncthreads();
}

template <int MODE, int BT, int RPW, int KC>
__device__ __forceinline__ void gemv(const Args &A, const float *x, uint32_t x_stride, const int64_t *tok, uint32_t in,
                                     const float *norm_w, const __half *w, const float *bias, uint32_t out, float *y,
                                     uint32_t y_stride, float *xs, Pass<MODE, RPW, KC> &wp,
                                     const Merge *merge = nullptr) {
    // the RMSNorm sums in the stand-alone GEMV's order (256 threads: per thread a strided
    // sum, per warp a butterfly, then warps 0..7 in order), so both paths normalise alike
    constexpr int kNormThreads = 256, kNormWarps = kNormThreads / 32, kSub = kNormThreads / kThreads;
    __shared__ float red[kNormWarps][BT];
    constexpr int NW = MODE == 2 ? 2 : 1;
    const uint32_t B = A.batch;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (merge) merge_rows(A, *merge, xs, xs + B * in);
    else for (uint32_t e = tid; e < B * in; e += kThreads) {
        const uint32_t b = e / in, i = e - b * in;
        float v;
        if (tok) {
            v = __ldg(A.emb + (uint64_t)tok[b] * in + i);
            if (blockIdx.x == 0) A.h[(uint64_t)b * A.hidden + i] = v;
        } else {
            v = ldcg(x + (uint64_t)b * x_stride + i);
        }
        xs[e] = v;
    }
    __syncthreads();
    if (MODE != 1) {
        float ss[BT];
#pragma unroll
        for (int b = 0; b < BT; ++b) {
#pragma unroll
            for (int k = 0; k < kSub; ++k) {  // virtual thread tid + k * kThreads
                float s = 0.0f;
                if ((uint32_t)b < B)
                    for (uint32_t i = tid + k * kThreads; i < in; i += kNormThreads) s = fmaf(xs[b * in + i], xs[b * in + i], s);
                s = warp_sum(s);
                if (lane == 0) red[warp + k * kWarps][b] = s;
            }
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < BT; ++b) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kNormWarps; ++k) s += red[k][b];
            ss[b] = rsqrtf(s / (float)in + A.eps);
        }
#pragma unroll
        for (int b = 0; b < BT; ++b)
            if ((uint32_t)b < B)
                for (uint32_t i = tid; i < in; i += kThreads) xs[b * in + i] = xs[b * in + i] * ss[b] * __ldg(norm_w + i);
        __syncthreads();
    }
    const uint32_t chunks = in / 8;
    bool first = true;  // wp holds the first pass of the first rows already
    for (uint32_t r0 = (blockIdx.x * kWarps + warp) * RPW; r0 < out; r0 += gridDim.x * kWarps * RPW) {
        float acc[RPW][NW][BT];
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int u = 0; u < NW; ++u)
#pragma unroll
                for (int b = 0; b < BT; ++b) acc[r][u][b] = 0.0f;
        for (uint32_t base = 0; base < chunks; base += 32u * KC) {
            if (!first) wp.load(w, in, out, r0, base);
            first = false;
            const auto &wv = wp.v;
#pragma unroll
            for (int c = 0; c < KC; ++c) {
                const uint32_t ch = base + lane + 32u * c;
                if (ch < chunks) {
#pragma unroll
                    for (int r = 0; r < RPW; ++r)
#pragma unroll
                        for (int u = 0; u < NW; ++u)
#pragma unroll
                            for (int b = 0; b < BT; ++b)
                                if ((uint32_t)b < B) acc[r][u][b] += dot8(wv[r][u][c], xs + b * in + 8u * ch);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const uint32_t row = r0 + r;
#pragma unroll
            for (int u = 0; u < NW; ++u)
#pragma unroll
                for (int b = 0; b < BT; ++b) acc[r][u][b] = warp_sum(acc[r][u][b]);
            if (lane == 0 && row < out) {
#pragma unroll
                for (int b = 0; b < BT; ++b) {
                    if ((uint32_t)b >= B) continue;
                    const float v = acc[r][0][b];
                    float *dst = y + (uint64_t)b * y_stride + row;
                    if constexpr (MODE == 0) {
                        *dst = bias ? v + __ldg(bias + row) : v;
                    } else if constexpr (MODE == 1) {
                        *dst = ldcg(dst) + v;
                    } else {
                        *dst = v / (1.0f + expf(-v)) * acc[r][NW - 1][b];
                    }
                }
            }
        }
    }
}

// K/V append of sequence b, KV head hd at row pos (kv_rope_append_kernel's arithmetic for
// one token, FP32 sources): RoPE'd K rounded to FP16, encoded into the packed store; V to
// the FP16 store; then the head's key and value lengths moved to pos + 1.  One warp; d = 64
// (lane p holds dim pair p), cs: the row's RoPE angles.  vv returns the lane's V elements
// (lane, lane + 32) as read from the source.
template <bool kStaged>
__device__ void append_one(const Args &A, const KvRopeArgs &a, const EncodeHead &h, uint32_t hd, uint32_t b,
                           uint32_t pos, const float2 *cs, WarpKey &wk, float *kr, int lane, float (&vv)[2]) {
    const uint32_t d = A.d, pairs = d / 2, seq = a.seq_first + b;
    vv[0] = vv[1] = 0.0f;
    if (pos >= a.capacity) {  // the host checked the capacity: refuse, report
        if (lane == 0) atomicOr(A.status, kStatusBadLength);
        return;
    }
    const uint64_t at = (uint64_t)b * a.seq_stride + (uint64_t)hd * d;
    const float *ks = static_cast<const float *>(a.k_src), *vs = static_cast<const float *>(a.v_src);
    // the row's K pair and V elements of this lane in one round trip
    const float x = ldcg(ks + at + lane), y = ldcg(ks + at + lane + pairs);
    vv[0] = ldcg(vs + at + lane);
    vv[1] = ldcg(vs + at + lane + 32u);
    {
        const float c = cs[lane].x, sn = cs[lane].y;
        kr[lane] = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn));
        kr[lane + pairs] = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
    }
    __syncwarp();
    for (uint32_t i = lane; i < d; i += 32) wk.xs[i] = __half2float(__float2half_rn(kr[h.t.perm[i]]));
    warp_encode<kStaged>(h, d, wk, seq, pos, lane);
    __half *vrow = reinterpret_cast<__half *>(a.v[hd]) + (uint64_t)seq * a.v_seq_stride[hd] + (uint64_t)pos * a.vD;
#pragma unroll
    for (uint32_t u = 0; u < 2; ++u) {
        const uint32_t e = lane + 32u * u;
        uint32_t de = e;
        if (a.v_swizzle) {
            const uint32_t c = e >> 3;
            de = (((c & ~7u) | ((c ^ pos) & 7u)) << 3) | (e & 7u);
        }
        vrow[de] = __float2half_rn(vv[u]);
    }
    __syncwarp();
    if (lane == 0) {
        a.head[hd].lengths[seq] = pos + 1;
        a.v_lengths[hd][seq] = pos + 1;
    }
    fence_proxy_global();  // the rows are read next by bulk copies (async proxy)
}

// The attention partial of the row append_one just stored (sequence b, KV head hd), written
// by the same warp into partial slot `slot`: the key reconstructed from the warp's codebook
// values and FP16 scales (src/reference/production_math.py:27-31: per group s_g R^T c, in
// the permuted order), each of the pair's query rows RoPE'd at the row (cs: its angles),
// their dot product in log2 units (the query records' log2(e) / sqrt(d)); then, as the
// attention body leaves a range of one key: maximum = the logit, sum = 2^kPShift, output =
// 2^kPShift * V, V the FP16 row (vv: the lane's source elements).  kr (the warp's RoPE
// scratch) holds the reconstructed key.  The query elements of every row are loaded in one
// batch.  d = 64; QM bounds the rows.
template <bool kStaged, int QM>
__device__ void new_row_partial(const Args &A, const AttnArgs &a, const EncodeHead &h, uint32_t hd, uint32_t b,
                                uint32_t slot, const float2 *cs, const float (&vv)[2], const WarpKey &wk, float *kr,
                                int lane) {
    const uint32_t d = A.d, pairs = d / 2, R = a.rows;
    const float *qg = A.qkv + (uint64_t)b * A.qkv_row + (uint64_t)hd * R * d;
    uint32_t pj[2];
    bool first[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const uint32_t j = h.t.perm[lane + 32u * u];
        pj[u] = j < pairs ? j : j - pairs;
        first[u] = j < pairs;
    }
    float qx[QM][2], qy[QM][2];
#pragma unroll
    for (uint32_t r = 0; r < (uint32_t)QM; ++r)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            qx[r][u] = r < R ? ldcg(qg + r * d + pj[u]) : 0.0f;
            qy[r][u] = r < R ? ldcg(qg + r * d + pj[u] + pairs) : 0.0f;
        }
    for (uint32_t i = lane; i < d; i += 32) {
        const uint32_t g = h.t.group_of[i], lo = h.group_off[g], hi = h.group_off[g + 1];
        float x = 0.0f;
#pragma unroll 8
        for (uint32_t j = lo; j < hi; ++j) x = fmaf(table_load<kStaged>(h.t.rot + (uint64_t)j * d + i), wk.cv[j], x);
        kr[i] = __fmul_rn(x, __half2float(__ushort_as_half(wk.srow[g])));
    }
    __syncwarp();
    float kv_i[2];
    float2 cu[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        kv_i[u] = kr[lane + 32u * u];
        cu[u] = cs[pj[u]];
    }
    const float qscale = attn::kLog2e / sqrtf((float)d), one = (float)(1u << (int)attn::kPShift);
    const float o0 = __fmul_rn(one, __half2float(__float2half_rn(vv[0])));
    const float o1 = __fmul_rn(one, __half2float(__float2half_rn(vv[1])));
#pragma unroll
    for (uint32_t r = 0; r < (uint32_t)QM; ++r) {
        if (r >= R) break;
        float dot = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float x = qx[r][u], y = qy[r][u], c = cu[u].x, sn = cu[u].y;
            const float q = first[u] ? __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn))
                                     : __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
            dot = fmaf(q, kv_i[u], dot);
        }
        const float lg = __fmul_rn(warp_sum(dot), qscale);
        float *pp = a.part + ((((uint64_t)slot * a.seq_count + b) * a.heads + hd) * R + r) * (uint64_t)(d + 2);
        pp[lane] = o0;
        pp[lane + 32] = o1;
        if (lane == 0) {
            pp[d] = lg;
            pp[d + 1] = one;
        }
    }
}

// Split-half RoPE of element j of a raw row q (d = 2 * pairs) with the angle's cosine and
// sine cs[j mod pairs]: attn::rope_elem's arithmetic, the angle computed once per launch.
__device__ __forceinline__ float rope_cs(const float *q, uint32_t j, uint32_t pairs, const float2 *cs) {
    const uint32_t p = j < pairs ? j : j - pairs;
    const float c = cs[p].x, sn = cs[p].y, x = q[p], y = q[p + pairs];
    return j < pairs ? __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, sn)) : __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, sn));
}

// Query records of (sequence s, KV head hd) into shared memory qt [D][QP] (qrot_kernel's
// arithmetic): the gqa query rows of the head, split-half RoPE at the sequence's new row
// (cs: that row's angles), permuted and rotated into the code domain, scaled to log2 units;
// zero past the rows.  rot, perm, grp: the head's rotation, permutation and group of each
// dim (shared-memory copies, or the tables in global memory); the permutation and group
// entries a thread needs are fetched together with the query rows, so the chain holds one
// round trip.  One CTA; qraw (kMaxRows * D floats) is its scratch.  Ends with a CTA barrier.
template <int QM>
__device__ void query_records(const Args &A, const AttnArgs &a, uint32_t hd, uint32_t s, const float2 *cs,
                              const float *rot, const uint8_t *perm, const uint8_t *grp, float *qraw, float *qt) {
    constexpr uint32_t QP = attn::QPad<QM>::QP;
    constexpr uint32_t kE2 = (kMaxRows * D + kThreads - 1) / kThreads, kE3 = (D * QP + kThreads - 1) / kThreads;
    const AttnHead &h = a.head[hd];
    const uint32_t R = a.rows, d = A.d, tid = threadIdx.x;
    const float *qg = A.qkv + (uint64_t)s * A.qkv_row + (uint64_t)hd * R * d;
    uint32_t pm[kE2], gq[kE3];
#pragma unroll
    for (uint32_t u = 0; u < kE2; ++u) {
        const uint32_t idx = tid + u * kThreads;
        pm[u] = idx < R * d ? perm[idx % d] : 0u;
    }
#pragma unroll
    for (uint32_t u = 0; u < kE3; ++u) {
        const uint32_t j = (tid + u * kThreads) / QP;
        gq[u] = j < d ? grp[j] : 0u;
    }
    for (uint32_t idx = tid; idx < R * d; idx += kThreads) qt[idx] = ldcg(qg + idx);  // raw rows, then RoPE
    __syncthreads();
#pragma unroll
    for (uint32_t u = 0; u < kE2; ++u) {
        const uint32_t idx = tid + u * kThreads;
        if (idx < R * d) qraw[idx] = rope_cs(qt + (idx / d) * d, pm[u], d / 2, cs);
    }
    __syncthreads();
    const float qscale = attn::kLog2e / sqrtf((float)d);
#pragma unroll
    for (uint32_t u = 0; u < kE3; ++u) {
        const uint32_t idx = tid + u * kThreads;
        if (idx >= D * QP) break;
        const uint32_t j = idx / QP, r = idx % QP;
        float v = 0.0f;
        if (r < R && j < d) {
            const uint32_t g = gq[u], lo = h.group_off[g], hi = h.group_off[g + 1];
            const float *rj = rot + (uint64_t)j * d;
            for (uint32_t i = lo; i < hi; ++i) v = fmaf(rj[i], qraw[r * d + i], v);
            v *= qscale;
        }
        qt[idx] = v;
    }
    __syncthreads();
}


// Attention tasks: nt ranges of task_tokens per pair over the keys stored before this step
// (partial slots 0 .. nt-1; slot nt is the new row's), pairs in head-major order; task t
// runs on CTA (t + n_app) mod grid, so the K/V append CTAs take tasks last.
struct Tasks {
    uint32_t nt, total, first;  // ranges per pair, tasks, this CTA's first task (>= total: none)
};
__device__ __forceinline__ Tasks tasks(const Args &A, uint32_t n_app) {
    uint32_t lmax = 2;
    for (uint32_t b = 0; b < A.batch; ++b) lmax = max(lmax, A.len_new[b]);
    Tasks t;
    t.nt = (lmax - 1u + A.task_tokens - 1) / A.task_tokens;
    t.total = A.kv_heads * A.batch * t.nt;
    t.first = (blockIdx.x + gridDim.x - n_app % gridDim.x) % gridDim.x;
    return t;
}

// Shared-memory copies of the head tables of a CTA's first attention pair, made during the
// Q/K/V phase: rotation [d][d], permutation, group of each dim, lookup offsets (rot null:
// none, every pair reads the tables in global memory).
struct HeadCopy {
    const float *rot;
    const uint8_t *perm, *grp;
    const uint16_t *lko;
    uint32_t hd;
};

// The attention phase of one layer: the CTA's tasks, each attn::attn_pair over its range.  A
// task that starts a pair builds the pair's query records (and stages a new head's
// codebooks) as the body's prologue, after the range's first tile copies are issued, so the
// copies land meanwhile.  The head of hc (the CTA's first pair) has its codebooks in their
// own region (A.off_lk, copied during the Q/K/V phase); other heads are staged into the
// plan's.  cs: the new rows' RoPE angles, [batch][d / 2].
template <int QM>
__device__ void attention_phase(const Args &A, const AttnArgs &a, const Tasks &tk, const float2 *cs, float *qraw_s,
                                float *qt_s, const HeadCopy &hc) {
    extern __shared__ __align__(128) unsigned char smem[];
    const uint32_t B = A.batch, T = A.task_tokens, tid = threadIdx.x;
    if (tk.first >= tk.total) return;
    // the body's mbarriers (their shared memory held GEMV activations in between)
    if (tid < kWarps * 4) attn::mbar_init(attn::smem_u32(smem + A.pl.bars) + tid * 8u, 1u);
    attn::fence_barrier_init();
    __syncthreads();
    float *cent_s = reinterpret_cast<float *>(smem + A.pl.cent);
    attn::Plan pl_own = A.pl;
    pl_own.cent = A.off_lk;
    uint32_t phase = 0, q_pair = ~0u, staged_hd = ~0u;
    for (uint32_t t = tk.first; t < tk.total; t += gridDim.x) {
        const uint32_t p = t / tk.nt, i = t % tk.nt, hd = p / B, s = p % B;
        const AttnHead &h = a.head[hd];
        const bool own = hc.rot && hd == hc.hd, fresh = p != q_pair, restage = !own && hd != staged_hd;
        auto prologue = [&]() {
            if (restage) attn::stage_lookup(h, A.pl, cent_s, (int)tid);
            if (fresh)
                query_records<QM>(A, a, hd, s, cs + s * (D / 2), own ? hc.rot : h.rot, own ? hc.perm : h.perm,
                                  own ? hc.grp : h.group_of, qraw_s, qt_s);
        };
        if (!own) staged_hd = hd;
        q_pair = p;
        uint32_t body_hd = hd;  // codebooks in place: the body stages none
        // the range ends before the row this step appends, and its length is known: the
        // keys stored before this step
        attn::attn_pair<D, QM, KKind::Packed, false, attn::RuntimeGroups>(
            a, own ? pl_own : A.pl, A.d, hd, s, i * T, min((i + 1) * T, A.len_new[s] - 1u), i, tk.nt + 1, phase,
            body_hd, qt_s, true, A.len_new[s] - 1u, own ? hc.lko : nullptr, prologue);
    }
    // every copy has landed (each pair ends with its waits and a CTA barrier): the region
    // goes back to the GEMV phases
    if (tid < kWarps * 4) mbar_inval(attn::smem_u32(smem + A.pl.bars) + tid * 8u);
    __syncthreads();
}

// The decode step.  QM: query rows per KV head of the attention body (gqa <= QM); BT: the
// batch bound of the GEMV accumulators (batch <= BT).
template <int QM, int BT>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ Args A) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) unsigned char hs_raw[sizeof(EncodeHead)];
    __shared__ __align__(8) uint64_t stage_bar, rot_bar, args_bar, mrg_bar;
    // the layer's append / attention arguments, copied into shared memory during the Q/K/V
    // phase: the bodies read their fields in dependent chains, which global memory would
    // turn into L2 round trips
    __shared__ __align__(16) unsigned char kv_raw[kKvBytes], att_raw[kAttBytes];
    __shared__ WarpKey wks[kWarps];
    __shared__ float kr[kWarps][kMaxDim];
    EncodeHead &hs = *reinterpret_cast<EncodeHead *>(hs_raw);
    float *xs = reinterpret_cast<float *>(smem);  // GEMV activations (the attention plan's region)
    unsigned char *enc_s = smem + A.off_e;
    float *rot_s = reinterpret_cast<float *>(smem + A.off_r);
    const uint8_t *tab_s = smem + A.off_r + 4u * D * D;  // permutation, group of each dim, lookup offsets
    float *qraw_s = reinterpret_cast<float *>(smem + A.off_q), *qt_s = qraw_s + kQrawFloats;
    // cosine and sine of every sequence's new-row RoPE angles (the same in every layer)
    __shared__ float2 cs_s[kMaxRows * (D / 2)];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t B = A.batch, H = A.kv_heads, d = A.d;
    for (uint32_t idx = tid; idx < B * (D / 2); idx += kThreads) {
        const uint32_t b = idx / (D / 2), p = idx % (D / 2);
        const float ang = __fmul_rn((float)(A.len_new[b] - 1u), A.layers[0].kv.inv_freq[p]);
        cs_s[idx] = make_float2(cosf(ang), sinf(ang));
    }
    const uint32_t n_app = H * ((B + kWarps - 1) / kWarps);  // CTAs of the K/V append: a warp per key
    const bool app_cta = blockIdx.x < n_app;
    const uint32_t app_hd = blockIdx.x % H;
    const Tasks tk = tasks(A, n_app);
    const bool has_task = tk.first < tk.total;
    const uint32_t first_p = has_task ? tk.first / tk.nt : 0u, first_hd = first_p / B;
    // CTAs with an attention task and no append copy their first pair's head tables into
    // shared memory during the Q/K/V phase
    const bool early_q = has_task && !app_cta;
    const uint32_t rot_bytes = d * d * 4u, rbar = attn::smem_u32(&rot_bar), abar = attn::smem_u32(&args_bar);
    const uint32_t args_bytes = (has_task ? kAttBytes : 0u) + (app_cta ? kKvBytes : 0u);
    const uint32_t qkv_bytes = A.qkv_row * A.hidden * 2u;
    prefetch_l2(A.layers[0].w_qkv, qkv_bytes);
    stamp(A, 0);
    uint32_t nb = 0;  // barriers passed
    Pass<0, 2, kChunks> pq;  // 2 rows x 128 chunks of 8 inputs per warp and pass
    pq.preload(A.layers[0].w_qkv, A.hidden, A.qkv_row);

    for (uint32_t l = 0; l < A.n_layers; ++l) {
        const Layer &L = A.layers[l];
        // ---- 1. RMSNorm + Q/K/V; meanwhile the append CTAs' encode tables and the attention
        //      CTAs' rotation are copied into shared memory ----
        const bool staging = A.enc_stage && app_cta;
        if (staging) stage_head_tables(L.kv.head[app_hd], enc_s, hs, &stage_bar);
        if (args_bytes && tid == 0) {
            attn::mbar_init(abar, 1u);
            attn::fence_barrier_init();
            attn::fence_proxy_async();
            attn::mbar_expect_tx(abar, args_bytes);
            if (has_task) attn::bulk_g2s(attn::smem_u32(att_raw), &L.att, kAttBytes, abar);
            if (app_cta) attn::bulk_g2s(attn::smem_u32(kv_raw), &L.kv, kKvBytes, abar);
        }
        if (early_q && tid == 0) {
            // rotation, permutation, group of each dim and lookup offsets of the first pair's
            // head (16-byte aligned in the table blob; d = 64, so whole 16-byte units)
            const AttnHead &fh = L.att.head[first_hd];
            attn::mbar_init(rbar, 1u);
            attn::fence_barrier_init();
            attn::fence_proxy_async();
            const uint32_t lk_bytes = attn::align16(4u * fh.n_lookup);  // the blob pads with zeros
            attn::mbar_expect_tx(rbar, rot_bytes + 4u * d + lk_bytes);
            attn::bulk_g2s(attn::smem_u32(rot_s), fh.rot, rot_bytes, rbar);
            attn::bulk_g2s(attn::smem_u32(smem + A.off_lk), fh.lookup, lk_bytes, rbar);
            attn::bulk_g2s(attn::smem_u32(tab_s), fh.perm, d, rbar);
            attn::bulk_g2s(attn::smem_u32(tab_s + d), fh.group_of, d, rbar);
            attn::bulk_g2s(attn::smem_u32(tab_s + 2 * d), fh.lookup_off, 2 * d, rbar);
        }
        if (early_q) {
            // the zero tail after the copied codebooks (lookups of padding records land there)
            const uint32_t n0 = attn::align16(4u * L.att.head[first_hd].n_lookup) / 4u;
            float *lk = reinterpret_cast<float *>(smem + A.off_lk);
            for (uint32_t i = n0 + tid; i < min(n0 + 256u, A.pl.cent_alloc); i += kThreads) lk[i] = 0.0f;
        }
        gemv<0, BT, 2, kChunks>(A, A.h, A.hidden, l == 0 ? A.tokens : nullptr, A.hidden, L.ln1, L.w_qkv, L.qkv_b,
                                A.qkv_row, A.qkv, A.qkv_row, xs, pq);
        if (!grid_barrier(A.bar, A.bar_base + (unsigned long long)(++nb) * gridDim.x, A.status)) {
            if (staging) staged_tables_drain(&stage_bar, false);
            if (early_q) attn::mbar_wait_bounded(rbar, 0u);
            if (args_bytes) attn::mbar_wait_bounded(abar, 0u);
            return;
        }
        stamp(A, 1 + 5 * l);
        // ---- 2. K/V append | attention tasks.  The later phases' matrices are requested into
        //      L2 by the CTAs with neither (every CTA its share when few are idle) ----
        {
            const uint32_t busy = n_app + tk.total, n_idle = busy < gridDim.x ? gridDim.x - busy : 0u;
            const bool by_idle = n_idle >= 16u;
            if (!by_idle || blockIdx.x >= busy) {
                const uint32_t part = by_idle ? blockIdx.x - busy : ~0u, parts = by_idle ? n_idle : 0u;
                prefetch_l2(L.w_o, (uint64_t)A.hidden * A.q_heads * d * 2u, 0, part, parts);
                prefetch_l2(L.w_gu, (uint64_t)2u * A.inter * A.hidden * 2u, 32, part, parts);
                prefetch_l2(L.w_down, (uint64_t)A.hidden * A.inter * 2u, 64, part, parts);
                if (l + 1 < A.n_layers) prefetch_l2(A.layers[l + 1].w_qkv, qkv_bytes, 96, part, parts);
                else prefetch_l2(A.lm_head, (uint64_t)A.vocab * A.hidden * 2u, 96, part, parts);
            }
        }
        bool args_landed = false;
        if (args_bytes) {
            args_landed = __syncthreads_and(attn::mbar_wait_bounded(abar, 0u));
            if (!args_landed && tid == 0) atomicOr(A.status, kStatusWaitTimeout);
            if (args_landed && tid == 0) mbar_inval(abar);  // initialised again next layer
        }
        // the copies this CTA made (an append CTA copies the append arguments, a CTA with an
        // attention task the attention arguments), else the global originals
        const KvRopeArgs &kv = args_landed && app_cta ? *reinterpret_cast<const KvRopeArgs *>(kv_raw) : L.kv;
        const AttnArgs &att = args_landed && has_task ? *reinterpret_cast<const AttnArgs *>(att_raw) : L.att;
        if (app_cta) {
            const bool staged = staging && staged_tables_ready(&stage_bar, A.status);
            const uint32_t b = (blockIdx.x / H) * kWarps + warp;
            if (b < B) {
                const uint32_t pos = A.len_new[b] - 1u;
                const float2 *csb = cs_s + b * (D / 2);
                float vv[2];
                if (staged) {
                    append_one<true>(A, kv, hs, app_hd, b, pos, csb, wks[warp], kr[warp], lane, vv);
                    new_row_partial<true, QM>(A, att, hs, app_hd, b, tk.nt, csb, vv, wks[warp], kr[warp], lane);
                } else {
                    append_one<false>(A, kv, kv.head[app_hd], app_hd, b, pos, csb, wks[warp], kr[warp], lane, vv);
                    new_row_partial<false, QM>(A, att, kv.head[app_hd], app_hd, b, tk.nt, csb, vv, wks[warp], kr[warp],
                                           lane);
                }
            }
            if (staging) {
                staged_tables_drain(&stage_bar, staged);
                __syncthreads();
                if (tid == 0) mbar_inval(smem_addr(&stage_bar));  // initialised again next layer
            }
        }
        HeadCopy hc{};
        if (early_q) {
            const bool landed = __syncthreads_and(attn::mbar_wait_bounded(rbar, 0u));
            if (!landed && tid == 0) atomicOr(A.status, kStatusWaitTimeout);
            if (landed) hc = HeadCopy{rot_s, tab_s, tab_s + d, reinterpret_cast<const uint16_t *>(tab_s + 2 * d), first_hd};
            if (landed && tid == 0) mbar_inval(rbar);  // initialised again next layer
        }
        // ---- attention over the keys stored before this step, in the same phase (no range
        //      reads a row the appends write) ----
        attention_phase<QM>(A, att, tk, cs_s, qraw_s, qt_s, hc);
        Pass<1, 1, kChunks> po;
        po.preload(L.w_o, A.q_heads * d, A.hidden);
        if (!grid_barrier(A.bar, A.bar_base + (unsigned long long)(++nb) * gridDim.x, A.status)) return;
        stamp(A, 2 + 5 * l);
        // ---- 4. o_proj + residual ----
        const Merge mg{&att, tk.nt + 1, A.off_part ? reinterpret_cast<float *>(smem + A.off_part) : nullptr,
                       &mrg_bar};
        gemv<1, BT, 1, kChunks>(A, A.att, A.q_heads * d, nullptr, A.q_heads * d, nullptr, L.w_o, nullptr, A.hidden,
                                A.h, A.hidden, xs, po, &mg);
        Pass<2, 2, kChunks> pg;
        pg.preload(L.w_gu, A.hidden, A.inter);
        if (!grid_barrier(A.bar, A.bar_base + (unsigned long long)(++nb) * gridDim.x, A.status)) return;
        stamp(A, 3 + 5 * l);
        // ---- 5. RMSNorm + gate/up + SiLU ----
        gemv<2, BT, 2, kChunks>(A, A.h, A.hidden, nullptr, A.hidden, L.ln2, L.w_gu, nullptr, A.inter, A.act, A.inter,
                                xs, pg);
        Pass<1, 1, kChunks> pd;
        pd.preload(L.w_down, A.inter, A.hidden);
        if (!grid_barrier(A.bar, A.bar_base + (unsigned long long)(++nb) * gridDim.x, A.status)) return;
        stamp(A, 4 + 5 * l);
        // ---- 6. down_proj + residual ----
        gemv<1, BT, 1, kChunks>(A, A.act, A.inter, nullptr, A.inter, nullptr, L.w_down, nullptr, A.hidden, A.h,
                                A.hidden, xs, pd);
        if (l + 1 < A.n_layers) pq.preload(A.layers[l + 1].w_qkv, A.hidden, A.qkv_row);
        if (!grid_barrier(A.bar, A.bar_base + (unsigned long long)(++nb) * gridDim.x, A.status)) return;
        stamp(A, 5 + 5 * l);
    }
    // ---- final RMSNorm + lm_head: eight rows per warp in flight ----
    Pass<0, 8, 3> plm;
    plm.preload(A.lm_head, A.hidden, A.vocab);
    gemv<0, BT, 8, 3>(A, A.h, A.hidden, nullptr, A.hidden, A.final_norm, A.lm_head, nullptr, A.vocab, A.logits, A.vocab,
                      xs, plm);
    stamp(A, 1 + 5 * A.n_layers);
}

}  // namespace step
}  // namespace bgtq

// ---------------------------------------------------------------------------------------
// Host side: the decoder object and its entry points.
// ---------------------------------------------------------------------------------------
struct bgtq_decoder {
    int device = 0;
    bgtq_decoder_desc desc{};
    std::vector<bgtq_attention *> att;
    const void *kernel = nullptr;
    uint32_t ctas = 0, smem = 0, qkv_row = 0, gqa = 0;
    bgtq::step::Args args{};      // everything but the per-step fields
    bgtq::DevBuf layers, scratch, bar, rope, trace;
    unsigned long long bar_epoch = 0;  // the device arrival counter after the last step
    bool tracing = false;
};

namespace {

using namespace bgtq;

bgtq_status dfail(bgtq_status s, const std::string &m) {
    set_last_error(m);
    return s;
}

struct Guard {
    int prev = -1;
    bool ok = true;
    explicit Guard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~Guard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

const void *pick_kernel(uint32_t gqa, uint32_t batch) {
    if (gqa <= 3) return batch == 1 ? (const void *)step::step_kernel<3, 1> : (const void *)step::step_kernel<3, 4>;
    return batch == 1 ? (const void *)step::step_kernel<8, 1> : (const void *)step::step_kernel<8, 4>;
}

bool aligned16(const void *p) { return p && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

bgtq_status bgtq_decoder_create(const bgtq_decoder_desc *dp, bgtq_decoder **out) {
    using step::Layer;
    if (!dp || !out) return dfail(BGTQ_EINVAL, "null argument");
    *out = nullptr;
    const bgtq_decoder_desc &d = *dp;
    const uint32_t L = d.layers, B = d.batch;
    if (!L || B < 1 || B > 4 || d.head_dim != 64 || !d.kv_heads || d.kv_heads > (uint32_t)kMaxHeads ||
        !d.q_heads || d.q_heads % d.kv_heads || d.q_heads / d.kv_heads > (uint32_t)kMaxRows || !d.hidden ||
        d.hidden % 8 || !d.intermediate || d.intermediate % 8 || !d.vocab || !d.inv_freq || !d.ln1 || !d.ln2 ||
        !d.w_qkv || !d.w_o || !d.w_gate_up || !d.w_down || !d.final_norm || !aligned16(d.lm_head) || !d.attention)
        return dfail(BGTQ_EINVAL, "decoder: unsupported shape or missing weights");
    const uint32_t gqa = d.q_heads / d.kv_heads, hd_dim = d.head_dim;
    const uint32_t qkv_row = (d.q_heads + 2 * d.kv_heads) * hd_dim, att_w = d.q_heads * hd_dim;
    const int dev = d.attention[0] ? d.attention[0]->device : 0;
    for (uint32_t l = 0; l < L; ++l) {
        const bgtq_attention *a = d.attention[l];
        if (!a || a->heads != d.kv_heads || a->rows < gqa || a->dim != hd_dim || a->sequences < B || a->device != dev ||
            !d.ln1[l] || !d.ln2[l] || !aligned16(d.w_qkv[l]) || !aligned16(d.w_o[l]) || !aligned16(d.w_gate_up[l]) ||
            !aligned16(d.w_down[l]))
            return dfail(BGTQ_EINVAL, "decoder: layer " + std::to_string(l) + " weights or attention object");
        for (uint32_t h = 0; h < a->heads; ++h)
            if (a->keys[h]->kind != BGTQ_KEYS_PACKED || a->values[h]->dtype != BGTQ_F16)
                return dfail(BGTQ_EINVAL, "decoder: packed keys and FP16 values required");
    }
    Guard g(dev);
    if (!g.ok) return dfail(BGTQ_ECUDA, "cannot select device");
    uint32_t *status = device_status_word(dev);
    if (!status) return dfail(BGTQ_ECUDA, "no status word");
    bgtq_decoder *dec = new bgtq_decoder;
    dec->device = dev;
    dec->desc = d;
    dec->att.assign(d.attention, d.attention + L);
    dec->qkv_row = qkv_row;
    dec->gqa = gqa;
    auto bail = [&](bgtq_status s, const std::string &m) {
        bgtq_decoder_destroy(dec);
        return dfail(s, m);
    };
    auto ck = [&](cudaError_t e) { return e == cudaSuccess; };
    // scratch: Q/K/V rows, attention output, gate/up activations; RoPE table; barrier words
    const size_t n_qkv = (size_t)B * qkv_row, n_att = (size_t)B * att_w, n_act = (size_t)B * d.intermediate;
    if (!ck(dec->scratch.ensure(4 * (n_qkv + n_att + n_act))) || !ck(dec->rope.ensure(4 * (hd_dim / 2))) ||
        !ck(dec->bar.ensure(16)) || !ck(dec->layers.ensure(sizeof(Layer) * L)))
        return bail(BGTQ_ECUDA, "decoder: device allocation");
    float *qkv = static_cast<float *>(dec->scratch.p), *attn_out = qkv + n_qkv, *act = attn_out + n_att;
    if (!ck(cudaMemcpy(dec->rope.p, d.inv_freq, 4 * (hd_dim / 2), cudaMemcpyHostToDevice)) ||
        !ck(cudaMemset(dec->bar.p, 0, 16)))
        return bail(BGTQ_ECUDA, "decoder: upload");
    // per-layer arguments
    std::vector<Layer> hl(L);
    uint32_t row_stride = 0, scale_stride = 4, max_cent = 0, enc_stage = ~0u, cap = ~0u, max_splits = 64;
    for (uint32_t l = 0; l < L; ++l) {
        Layer &ly = hl[l];
        std::memset(&ly, 0, sizeof(ly));
        bgtq_attention *at = d.attention[l];
        ly.ln1 = d.ln1[l];
        ly.ln2 = d.ln2[l];
        ly.qkv_b = d.qkv_bias ? d.qkv_bias[l] : nullptr;
        ly.w_qkv = reinterpret_cast<const __half *>(d.w_qkv[l]);
        ly.w_o = reinterpret_cast<const __half *>(d.w_o[l]);
        ly.w_gu = reinterpret_cast<const __half *>(d.w_gate_up[l]);
        ly.w_down = reinterpret_cast<const __half *>(d.w_down[l]);
        KvRopeArgs &kv = ly.kv;
        AttnArgs &a = ly.att;
        kv.capacity = ~0u;
        for (uint32_t h = 0; h < d.kv_heads; ++h) {
            bgtq_keys *k = at->keys[h];
            bgtq_values *v = at->values[h];
            if (v->D != hd_dim) return bail(BGTQ_EINVAL, "decoder: value rows must have the head dim");
            fill_encode_head(k, kv.head[h]);
            kv.v[h] = v->data;
            kv.v_lengths[h] = v->d_lengths;
            kv.v_seq_stride[h] = (uint64_t)v->cap_alloc * v->D;
            fill_packed_head(a.head[h], k, v);
            row_stride = std::max(row_stride, k->row_stride);
            scale_stride = std::max(scale_stride, k->scale_stride);
            max_cent = std::max(max_cent, a.head[h].n_lookup);
            cap = std::min(cap, std::min(k->capacity, v->capacity));
            kv.capacity = std::min(kv.capacity, std::min(k->capacity, v->capacity));
        }
        // staged encode tables only when every layer's heads fit the staging window
        const uint32_t es = encode_stage_bytes(kv.head, d.kv_heads);
        enc_stage = enc_stage == ~0u ? es : (es && enc_stage ? std::max(enc_stage, es) : 0u);
        kv.k_src = qkv + att_w;
        kv.v_src = qkv + att_w + d.kv_heads * hd_dim;
        kv.start = at->keys[0]->d_lengths;
        kv.row_stride = qkv_row;
        kv.seq_stride = qkv_row;
        kv.rope = 1;
        kv.count = 1;
        kv.seq_count = B;
        kv.heads = d.kv_heads;
        kv.vD = at->values[0]->D;
        kv.v_swizzle = values_swizzled(0, kv.vD) ? 1u : 0u;
        kv.status = status;
        for (uint32_t p = 0; p < hd_dim / 2; ++p) kv.inv_freq[p] = d.inv_freq[p];
        a.qt = at->qt;
        a.lengths = at->keys[0]->d_lengths;
        a.out = attn_out;
        a.part = at->part;
        a.counters = at->counters;
        a.status = status;
        a.rope = static_cast<const float *>(dec->rope.p);
        a.seq_count = B;
        a.heads = d.kv_heads;
        a.rows = gqa;
        a.splits = 1;
        max_splits = std::min(max_splits, at->max_splits);
    }
    if (enc_stage == ~0u) enc_stage = 0;
    // shared memory: the attention plan and the GEMV activations share region U; the staged
    // encode tables and the query scratch follow
    int optin = 0, sms = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t QM = gqa <= 3 ? 3u : 8u, QP = QM <= 4 ? 4u : 8u, TT = attention_tile_tokens(hd_dim);
    const attn::Plan pl = attn::make_plan(KKind::Packed, 0, step::D, QP, TT, row_stride, scale_stride, max_cent,
                                          (uint32_t)optin - 64u, 2, QM);
    const uint32_t BT = B == 1 ? 1u : 4u;
    const uint32_t max_in = std::max(std::max(d.hidden, att_w), d.intermediate);
    // GEMV activations, and in the o_proj phase the split-merge weights after them
    // attention tasks of whole CTA tiles, few enough per pair that their partials and the new
    // row's fit the partial buffers
    if (max_splits < 2) return bail(BGTQ_EINVAL, "decoder: the attention objects need room for two partials");
    const uint32_t chunk = attn::kWarps * TT, tiles = (cap + chunk - 1) / chunk;
    const uint32_t task_tokens = chunk * ((tiles + max_splits - 2) / (max_splits - 1));
    const uint32_t max_nt = (cap + task_tokens - 1) / task_tokens + 1;  // partial slots per pair
    // region U: the attention plan, or the GEMV activations with (o_proj phase) the merge
    // weights and a copy of the partials after them
    const uint32_t off_part = attn::align128(4u * (BT * max_in + BT * d.q_heads * (2 * max_nt + 2)));
    const uint32_t part_bytes = attn::align16(4u * max_nt * B * d.q_heads * (hd_dim + 2));
    const bool part_copy = off_part + part_bytes <= 128u * 1024u;
    const uint32_t region_u = attn::align128(std::max(pl.total, part_copy ? off_part + part_bytes : off_part));
    const uint32_t off_e = region_u, off_r = attn::align128(off_e + enc_stage), off_q = off_r + 4u * hd_dim * hd_dim + 4u * hd_dim;
    const uint32_t off_lk = (off_q + 4u * (step::kQrawFloats + step::kQtFloats) + 1023u) & ~1023u;
    const uint32_t smem = off_lk + 4u * pl.cent_alloc;
    const void *kern = pick_kernel(gqa, B);
    cudaFuncAttributes fa{};
    if (!ck(cudaFuncGetAttributes(&fa, kern))) return bail(BGTQ_ECUDA, "decoder: kernel attributes");
    if (smem + fa.sharedSizeBytes > (size_t)optin)
        return bail(BGTQ_EINVAL, "decoder: shared memory plan exceeds the device (" + std::to_string(smem) + " bytes)");
    if (!ck(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)))
        return bail(BGTQ_ECUDA, "decoder: kernel attributes");
    int occ = 0;
    if (!ck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, step::kThreads, smem)) || occ < 1)
        return bail(BGTQ_ECUDA, "decoder: the step kernel does not fit an SM");
    // one CTA per SM by default: fewer arrivals per grid barrier outweigh the second CTA's
    // extra loads in flight
    const int per_sm = std::min(occ, d.ctas_per_sm ? (int)d.ctas_per_sm : 1);
    dec->ctas = (uint32_t)(sms * per_sm);
    if (dec->ctas < d.kv_heads * ((B + step::kWarps - 1) / step::kWarps) + d.kv_heads * B)
        return bail(BGTQ_EINVAL, "decoder: too few CTAs for the append and query phases");
    dec->smem = smem;
    dec->kernel = kern;
    if (!ck(cudaMemcpy(dec->layers.p, hl.data(), sizeof(Layer) * L, cudaMemcpyHostToDevice)))
        return bail(BGTQ_ECUDA, "decoder: layer upload");
    step::Args &A = dec->args;
    std::memset(&A, 0, sizeof(A));
    A.layers = static_cast<const Layer *>(dec->layers.p);
    A.n_layers = L;
    A.batch = B;
    A.hidden = d.hidden;
    A.q_heads = d.q_heads;
    A.kv_heads = d.kv_heads;
    A.gqa = gqa;
    A.d = hd_dim;
    A.inter = d.intermediate;
    A.vocab = d.vocab;
    A.qkv_row = qkv_row;
    A.eps = d.rms_eps;
    A.emb = d.embedding;
    A.qkv = qkv;
    A.att = attn_out;
    A.act = act;
    A.final_norm = d.final_norm;
    A.lm_head = reinterpret_cast<const __half *>(d.lm_head);
    A.pl = pl;
    A.task_tokens = task_tokens;
    A.enc_stage = enc_stage;
    A.off_e = off_e;
    A.off_r = off_r;
    A.off_part = part_copy ? off_part : 0u;
    A.off_lk = off_lk;
    A.off_q = off_q;
    A.bar = static_cast<uint32_t *>(dec->bar.p);
    A.status = status;
    *out = dec;
    return BGTQ_OK;
}

bgtq_status bgtq_decoder_step(bgtq_decoder *dec, const int64_t *tokens, float *h, float *logits, void *stream) {
    if (!dec || !h || !logits) return dfail(BGTQ_EINVAL, "null argument");
    if (tokens && !dec->args.emb) return dfail(BGTQ_EINVAL, "decoder: token ids need the embedding");
    const uint32_t B = dec->desc.batch, H = dec->desc.kv_heads;
    step::Args A = dec->args;
    // every layer's stores hold one length per sequence; the step appends one row
    for (uint32_t s = 0; s < B; ++s) {
        const uint32_t len = dec->att[0]->keys[0]->lengths[s];
        for (bgtq_attention *at : dec->att)
            for (uint32_t hh = 0; hh < H; ++hh) {
                if (at->keys[hh]->lengths[s] != len || at->values[hh]->lengths[s] != len)
                    return dfail(BGTQ_EBUSY, "decoder: K/V lengths must match across heads and layers");
                if ((uint64_t)len + 1 > std::min(at->keys[hh]->capacity, at->values[hh]->capacity))
                    return dfail(BGTQ_ECAPACITY, "K capacity exceeded");
            }
        A.len_new[s] = len + 1;
    }
    A.tokens = tokens;
    A.h = h;
    A.logits = logits;
    A.trace = dec->tracing ? static_cast<unsigned long long *>(dec->trace.p) : nullptr;
    A.bar_base = dec->bar_epoch;
    Guard g(dec->device);
    if (!g.ok) return dfail(BGTQ_ECUDA, "cannot select device");
    void *params[] = {&A};
    const cudaError_t e = cudaLaunchCooperativeKernel(dec->kernel, dim3(dec->ctas), dim3(step::kThreads), params,
                                                      dec->smem, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return dfail(BGTQ_ECUDA, std::string("decoder step launch: ") + cudaGetErrorString(e));
    dec->bar_epoch += (unsigned long long)step::kBarriersPerLayer * dec->desc.layers * dec->ctas;
    for (bgtq_attention *at : dec->att)
        for (uint32_t hh = 0; hh < H; ++hh)
            for (uint32_t s = 0; s < B; ++s) {
                ++at->keys[hh]->lengths[s];
                ++at->values[hh]->lengths[s];
            }
    return BGTQ_OK;
}

bgtq_status bgtq_decoder_info(const bgtq_decoder *dec, uint32_t *ctas, uint32_t *smem_bytes, uint32_t *table_bytes) {
    if (!dec) return dfail(BGTQ_EINVAL, "null argument");
    if (ctas) *ctas = dec->ctas;
    if (smem_bytes) *smem_bytes = dec->smem;
    if (table_bytes) *table_bytes = dec->args.enc_stage;
    return BGTQ_OK;
}

bgtq_status bgtq_decoder_trace(bgtq_decoder *dec, int on, uint64_t *out, uint32_t cap, uint32_t *n_out) {
    if (!dec) return dfail(BGTQ_EINVAL, "null argument");
    const uint32_t n = 2 + 5 * dec->desc.layers;
    Guard g(dec->device);
    if (!g.ok) return dfail(BGTQ_ECUDA, "cannot select device");
    if (on && dec->trace.ensure(8u * n) != cudaSuccess) return dfail(BGTQ_ECUDA, "trace allocation");
    if (out && dec->tracing) {
        if (cudaMemcpy(out, dec->trace.p, 8u * std::min(cap, n), cudaMemcpyDeviceToHost) != cudaSuccess)
            return dfail(BGTQ_ECUDA, "trace download");
    }
    if (n_out) *n_out = n;
    dec->tracing = on != 0;
    return BGTQ_OK;
}

void bgtq_decoder_destroy(bgtq_decoder *dec) {
    if (!dec) return;
    {
        Guard g(dec->device);
        dec->layers.release();
        dec->scratch.release();
        dec->bar.release();
        dec->rope.release();
        dec->trace.release();
    }
    delete dec;
}

}  // extern "C"
