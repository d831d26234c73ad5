// Device pieces of the warp-per-key K encode shared by the append kernels (encode.cu) and
// the persistent decode step (step.cu): one warp encodes one key in the canonical order of
// the CPU oracle, bit for bit, from tables in global or shared memory.  Every translation
// unit including this file is compiled with -fmad=false: no separate multiply / add pair
// may be contracted; every fused multiply-add here is an explicit fmaf.
#pragma once
#include <cuda_fp16.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace {

// Shared-memory scratch of one warp's key in the warp-per-key kernels.
struct WarpKey {
    float xs[kMaxDim];         // permuted FP16 key as FP32, then normalised
    float cv[kMaxDim];         // codebook value of each dimension's code
    float nrm[kMaxGroups];
    uint8_t codes[kMaxDim];
    uint32_t orow[kMaxDim / 4 + 1];
    uint16_t srow[8];
};

// The encode of one key held in wk.xs (already permuted, FP16-exact values) by one warp,
// written to row dst_row of sequence dseq: same arithmetic and order as encode_kernel,
// bit for bit - group sums and scales sequential per group (one lane per group), every
// y_j one lane's sequential FMA chain over its group, ascending.
// kSmem: the table pointers of h point into shared memory (plain loads; __ldg is for global
// memory only).
template <bool kSmem>
__device__ __forceinline__ float table_load(const float *p) {
    if constexpr (kSmem) return *p;
    else return __ldg(p);
}

template <bool kSmem>
__device__ __forceinline__ void warp_encode(const EncodeHead &h, uint32_t d, WarpKey &wk, uint32_t dseq,
                                            uint32_t dst_row, int lane) {
    const uint32_t ns = h.ns, ng = h.ng;
    const uint32_t row_words = h.row_stride / 4, sc_words = h.scale_stride / 2;
    uint8_t *ob = reinterpret_cast<uint8_t *>(wk.orow);
    __syncwarp();
    if ((uint32_t)lane < ng) {
        float acc = 0.0f;
#pragma unroll 8
        for (uint32_t i = h.group_off[lane]; i < h.group_off[lane + 1]; ++i) acc = fmaf(wk.xs[i], wk.xs[i], acc);
        wk.nrm[lane] = sqrtf(acc + 1e-30f);
    }
    __syncwarp();
    for (uint32_t i = lane; i < d; i += 32) {
        const float n = wk.nrm[h.t.group_of[i]];
        wk.xs[i] = wk.xs[i] / (n > 1e-10f ? n : 1.0f);
    }
    __syncwarp();
    for (uint32_t j = lane; j < d; j += 32) {
        const uint32_t g = h.t.group_of[j];
        const float *rj = h.t.rot + (uint64_t)j * d;
        float y = 0.0f;
#pragma unroll 8
        for (uint32_t i = h.group_off[g]; i < h.group_off[g + 1]; ++i) y = fmaf(wk.xs[i], table_load<kSmem>(rj + i), y);
        float t = (y - h.t.off[j]) * h.t.inv[j];
        t = fminf(fmaxf(t, 0.0f), 255.0f);
        wk.codes[j] = h.t.lut[(uint32_t)h.t.cbidx[j] * 256u + (uint32_t)t];
    }
    __syncwarp();
    // every lane fetches its dimensions' codebook values first, so the sequential per-group
    // sums below read shared memory instead of waiting on two dependent loads per dimension
    for (uint32_t j = lane; j < d; j += 32) wk.cv[j] = h.t.cent[h.t.cb_base[j] + wk.codes[j]];
    __syncwarp();
    if ((uint32_t)lane < ng) {
        float cl = 0.0f;
#pragma unroll 8
        for (uint32_t j = h.group_off[lane]; j < h.group_off[lane + 1]; ++j) cl = fmaf(wk.cv[j], wk.cv[j], cl);
        wk.srow[lane] = __half_as_ushort(__float2half_rn(wk.nrm[lane] / fmaxf(sqrtf(cl), 1e-10f)));
    } else if ((uint32_t)lane < 8) {
        wk.srow[lane] = 0;
    }
    for (uint32_t b = lane; b < row_words * 4; b += 32) {
        uint32_t v = 0;
        if (b < ns / 2) v = (uint32_t)wk.codes[2 * b] | ((uint32_t)wk.codes[2 * b + 1] << 4);
        else if (b < ns / 2 + (d - ns)) v = wk.codes[ns + (b - ns / 2)];
        ob[b] = (uint8_t)v;
    }
    __syncwarp();
    uint32_t *dst = reinterpret_cast<uint32_t *>(h.packed + (uint64_t)dseq * h.k_seq_stride +
                                                 (uint64_t)dst_row * h.row_stride);
    for (uint32_t c = lane; c < row_words; c += 32) dst[c] = wk.orow[c];
    if ((uint32_t)lane < sc_words) {
        uint32_t *sdst = reinterpret_cast<uint32_t *>(h.scales + (uint64_t)dseq * h.s_seq_stride +
                                                      (uint64_t)dst_row * h.scale_stride);
        sdst[lane] = (uint32_t)wk.srow[2 * lane] | ((uint32_t)wk.srow[2 * lane + 1] << 16);
    }
    __syncwarp();
}

// Bound on the polls of the table-staging mbarrier (a copy of at most 40 KB lands in
// microseconds; the bound only keeps a broken copy from hanging the kernel).
constexpr uint32_t kStageWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool stage_try_wait(uint32_t bar) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool stage_wait(uint32_t bar) {
    for (uint32_t i = 0; i < kStageWaitLimit; ++i)
        if (stage_try_wait(bar)) return true;
    return false;
}

// Starts the copy of the encode tables of g (the leading part of its table blob, up to the
// attention lookup; 16-byte aligned, a multiple of 16 bytes) into tab_s with one bulk
// asynchronous copy (cp.async.bulk, no multicast) that completes on the mbarrier at bar, and
// writes g with its table pointers moved there into hs.  Called by every thread of the CTA;
// ends with a barrier, after which the threads wait on bar (stage_wait) before reading tab_s.
__device__ __forceinline__ void stage_head_tables(const EncodeHead &g, unsigned char *tab_s, EncodeHead &hs,
                                                  uint64_t *bar) {
    const unsigned char *b = static_cast<const unsigned char *>(g.t.blob);
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)(reinterpret_cast<const unsigned char *>(g.t.lookup) - b);
        const uint32_t ba = smem_addr(bar);
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(ba) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ba), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_addr(tab_s)),
                     "l"(b), "r"(bytes), "r"(ba)
                     : "memory");
        hs = g;
        hs.t.rot = reinterpret_cast<const float *>(tab_s + (reinterpret_cast<const unsigned char *>(g.t.rot) - b));
        hs.t.cent = reinterpret_cast<const float *>(tab_s + (reinterpret_cast<const unsigned char *>(g.t.cent) - b));
        hs.t.off = reinterpret_cast<const float *>(tab_s + (reinterpret_cast<const unsigned char *>(g.t.off) - b));
        hs.t.inv = reinterpret_cast<const float *>(tab_s + (reinterpret_cast<const unsigned char *>(g.t.inv) - b));
        hs.t.lut = tab_s + (g.t.lut - b);
        hs.t.perm = tab_s + (g.t.perm - b);
        hs.t.group_of = tab_s + (g.t.group_of - b);
        hs.t.cbidx = tab_s + (g.t.cbidx - b);
        hs.t.cb_base =
            reinterpret_cast<const uint16_t *>(tab_s + (reinterpret_cast<const unsigned char *>(g.t.cb_base) - b));
    }
    __syncthreads();
}

// After stage_head_tables: true when the whole warp saw the staged tables land (then it
// reads them from shared memory).  A warp whose bounded wait ran out reports it in status and
// reads the global tables instead (same values, so the result is unchanged).
__device__ __forceinline__ bool staged_tables_ready(uint64_t *bar, uint32_t *status) {
    const bool ok = __all_sync(0xffffffffu, stage_wait(smem_addr(bar)));
    if (!ok && (threadIdx.x & 31) == 0 && status) atomicOr(status, kStatusWaitTimeout);
    return ok;
}
// Before a CTA that staged tables exits: a warp whose wait ran out waits (bounded) once more,
// so no copy into its shared memory is left in flight when it can.
__device__ __forceinline__ void staged_tables_drain(uint64_t *bar, bool ready) {
    if (!ready) stage_wait(smem_addr(bar));
}

// Element i of an FP16 or FP32 source.
__device__ __forceinline__ float src_elem(const void *p, uint64_t i, uint32_t f16) {
    return f16 ? __half2float(static_cast<const __half *>(p)[i]) : static_cast<const float *>(p)[i];
}

// Dynamic shared memory for staging every head's encode tables (the leading part of its
// table blob: the blob puts the encode tables first, the attention lookup after them), or 0
// when some head's part does not fit the default shared-memory window beside the warp-per-key
// kernels' static arrays, or its pointers are not laid out that way.
inline uint32_t encode_stage_bytes(const EncodeHead *heads, uint32_t n) {
    constexpr uintptr_t kStageMax = 40u * 1024u;
    uint32_t stage = 0;
    for (uint32_t h = 0; h < n; ++h) {
        const DeviceTables &t = heads[h].t;
        const uintptr_t b = reinterpret_cast<uintptr_t>(t.blob), end = reinterpret_cast<uintptr_t>(t.lookup);
        const uintptr_t ptrs[] = {reinterpret_cast<uintptr_t>(t.rot),   reinterpret_cast<uintptr_t>(t.cent),
                                  reinterpret_cast<uintptr_t>(t.off),   reinterpret_cast<uintptr_t>(t.inv),
                                  reinterpret_cast<uintptr_t>(t.lut),   reinterpret_cast<uintptr_t>(t.perm),
                                  reinterpret_cast<uintptr_t>(t.group_of), reinterpret_cast<uintptr_t>(t.cbidx),
                                  reinterpret_cast<uintptr_t>(t.cb_base)};
        bool ok = b != 0 && end > b && end - b <= kStageMax && (b & 15u) == 0 && ((end - b) & 15u) == 0;
        for (uintptr_t q : ptrs) ok = ok && q >= b && q < end;
        if (!ok) return 0;
        stage = stage > (uint32_t)(end - b) ? stage : (uint32_t)(end - b);
    }
    return stage;
}

}  // namespace
}  // namespace bgtq
