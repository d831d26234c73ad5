// Instantiation table and host launch logic for the attention kernels.
#include <algorithm>
#include <mutex>

#include "attention_impl.cuh"

namespace bgtq {
namespace {

using attn::Plan;

struct Entry {
    cudaError_t (*run)(const AttnArgs &, const Plan &, uint32_t, dim3, cudaStream_t);
    int (*occ)(const Plan &);
    cudaError_t (*load)();
    uint32_t qp, qm;
};

// Makes the driver load the kernel's code now (with lazy module loading it would load,
// and take device memory, on its first launch).
template <int D, int QM, KKind KK, bool VF32>
cudaError_t load_kernel() {
    cudaFuncAttributes fa;
    return cudaFuncGetAttributes(&fa, attn::attn_kernel<D, QM, KK, VF32>);
}

template <int D, int QM, KKind KK, bool VF32>
Entry entry() {
    return Entry{&attn::run<D, QM, KK, VF32>, &attn::occupancy<D, QM, KK, VF32>, &load_kernel<D, QM, KK, VF32>,
                 (uint32_t)attn::QPad<QM>::QP, (uint32_t)QM};
}

template <int D, KKind KK, bool VF32>
Entry pick_qm(uint32_t rows) {
    if constexpr (KK == KKind::Packed) {
        if (rows <= 1) return entry<D, 1, KK, VF32>();
        if (rows <= 2) return entry<D, 2, KK, VF32>();
        if (rows <= 3) return entry<D, 3, KK, VF32>();
        if (rows <= 4) return entry<D, 4, KK, VF32>();
        return entry<D, 8, KK, VF32>();
    } else {
        if (rows <= 1) return entry<D, 1, KK, VF32>();
        if (rows <= 4) return entry<D, 4, KK, VF32>();
        return entry<D, 8, KK, VF32>();
    }
}

template <int D>
Entry pick(KKind kk, int v_f32, uint32_t rows) {
    switch (kk) {
        case KKind::Packed: return v_f32 ? pick_qm<D, KKind::Packed, true>(rows) : pick_qm<D, KKind::Packed, false>(rows);
        case KKind::F16: return v_f32 ? pick_qm<D, KKind::F16, true>(rows) : pick_qm<D, KKind::F16, false>(rows);
        default: return v_f32 ? pick_qm<D, KKind::F32, true>(rows) : pick_qm<D, KKind::F32, false>(rows);
    }
}

Entry pick_entry(KKind kk, int v_f32, uint32_t D, uint32_t rows) {
    switch (D) {
        case 16: return pick<16>(kk, v_f32, rows);
        case 32: return pick<32>(kk, v_f32, rows);
        case 64: return pick<64>(kk, v_f32, rows);
        default: return pick<128>(kk, v_f32, rows);
    }
}

uint32_t dim_template(uint32_t d) { return d <= 16 ? 16u : d <= 32 ? 32u : d <= 64 ? 64u : 128u; }

// Resident CTAs per SM of a specialised kernel (the dynamic shared-memory limit set first),
// remembered per (kernel, device, shared-memory size).
int jit_occupancy(const void *k, int dev, uint32_t smem) {
    struct Slot { const void *k; int dev; uint32_t smem; int n; };
    static Slot slots[16] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    for (const Slot &sl : slots)
        if (sl.k == k && sl.dev == dev && sl.smem == smem) return sl.n;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, attn::kThreads, smem);
    static int next = 0;
    slots[next] = Slot{k, dev, smem, n};
    next = (next + 1) % 16;
    return n;
}

__global__ void probs_kernel(const float *logits, const float *lse, float *probs, uint64_t rows, uint32_t tokens,
                             uint32_t stride) {
    const uint64_t total = rows * tokens;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / tokens, t = i % tokens;
        const float lg = logits[r * stride + t];
        probs[r * stride + t] = lg == -INFINITY ? 0.0f : expf(lg - lse[r]);
    }
}

}  // namespace

// The kernel's own tile size (Geo<D>::TT): split boundaries and shared-memory plans use it,
// and whole-tile copies stay inside the capacity because it divides the row padding.
uint32_t attention_tile_tokens(uint32_t d) {
    static_assert(kTileRows % attn::Geo<16>::TT == 0 && kTileRows % attn::Geo<32>::TT == 0 &&
                      kTileRows % attn::Geo<64>::TT == 0 && kTileRows % attn::Geo<128>::TT == 0,
                  "tiles must divide the capacity padding");
    switch (dim_template(d)) {
        case 16: return attn::Geo<16>::TT;
        case 32: return attn::Geo<32>::TT;
        case 64: return attn::Geo<64>::TT;
        default: return attn::Geo<128>::TT;
    }
}

uint32_t attention_qm(KKind kk, uint32_t rows) { return pick_entry(kk, 0, 64, rows).qm; }

cudaError_t preload_attention_kernels(KKind kk) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, attn::qrot_kernel);
    for (uint32_t D : {16u, 32u, 64u, 128u})
        for (uint32_t rows : {1u, 2u, 3u, 4u, 8u})
            for (int vf = 0; vf < 2 && e == cudaSuccess; ++vf) e = pick_entry(kk, vf, D, rows).load();
    return e;
}

size_t attention_smem_bytes(KKind kk, int v_f32, uint32_t d, uint32_t rows, uint32_t row_stride,
                            uint32_t scale_stride, uint32_t max_cent) {
    const uint32_t D = dim_template(d);
    const Entry e = pick_entry(kk, v_f32, D, rows);
    return attn::make_plan(kk, v_f32, D, e.qp, attention_tile_tokens(d), row_stride, scale_stride, max_cent,
                           227u * 1024u, 2, e.qm).total;
}

cudaError_t launch_probs(const float *logits, const float *lse, float *probs, uint64_t rows, uint32_t tokens,
                         uint32_t stride, cudaStream_t s) {
    const uint64_t total = rows * tokens;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 148u * 8u) blocks = 148u * 8u;
    if (blocks == 0) return cudaSuccess;
    probs_kernel<<<(unsigned)blocks, 256, 0, s>>>(logits, lse, probs, rows, tokens, stride);
    return cudaGetLastError();
}

// Split-KV factor: minimise (waves of CTAs) x (tokens per split), i.e. the quantised
// critical path of a grid of pairs*splits equal CTAs over `slots` resident CTAs.
static void choose_splits(uint32_t pairs, uint32_t max_len, uint32_t chunk, uint32_t slots, uint32_t forced,
                          uint32_t cap, uint32_t *splits, uint32_t *tps) {
    const uint32_t max_s = std::max(1u, std::min(cap, (max_len + chunk - 1) / chunk));
    uint32_t best_s = 1;
    uint64_t best_cost = ~0ull;
    if (forced) {
        best_s = std::min(forced, max_s);
    } else {
        for (uint32_t sp = 1; sp <= max_s; ++sp) {
            const uint32_t t = ((max_len + sp - 1) / sp + chunk - 1) / chunk * chunk;
            const uint64_t waves = ((uint64_t)pairs * sp + slots - 1) / slots;
            // each CTA also pays a fixed start-up (tables, first tile latency, merge)
            // worth about one tile round of its warps
            const uint64_t cost = waves * (t + chunk);
            if (cost < best_cost) { best_cost = cost; best_s = sp; }
        }
    }
    uint32_t t = ((max_len + best_s - 1) / best_s + chunk - 1) / chunk * chunk;
    if (t == 0) t = chunk;
    *tps = t;
    *splits = std::max(1u, (max_len + t - 1) / t);
}

// Stream-K plan: `total` = pairs x nt CTA tiles (nt = tiles of one pair) over at most one
// wave of CTAs, `per` tiles each.  A CTA pays the same fixed start-up as a split (tables,
// first tile latency, merge) for each pair segment it runs.  Chosen when its critical path
// undercuts the split-KV plan's by a margin, and when every pair's segments fit the partial
// buffers (at most `cap` per pair), or whenever it is possible (`always`).
static bool choose_stream_k(uint32_t pairs, uint32_t max_len, uint32_t chunk, uint32_t slots, uint32_t splits,
                            uint32_t tps, uint32_t cap, bool always, uint32_t *units, uint32_t *per) {
    const uint64_t nt = (max_len + chunk - 1) / chunk, total = (uint64_t)pairs * nt;
    if (total < 2 || slots == 0) return false;
    uint64_t k = (total + slots - 1) / slots;
    while ((nt + k - 1) / k + 1 > cap) ++k;
    if (always) {
        *units = (uint32_t)((total + k - 1) / k);
        *per = (uint32_t)k;
        return true;
    }
    const uint64_t w = (total + k - 1) / k;
    // segments per CTA: a range of k tiles meets at most ceil(k / nt) + 1 pairs
    const uint64_t segs = std::min<uint64_t>((k + nt - 1) / nt + 1, k);
    const uint64_t sk_cost = k * chunk + segs * chunk;
    const uint64_t waves = ((uint64_t)pairs * splits + slots - 1) / slots;
    const uint64_t kv_cost = waves * (tps + chunk);
    if (sk_cost * 8 > kv_cost * 7) return false;  // within 12.5 %: keep split-KV
    *units = (uint32_t)w;
    *per = (uint32_t)k;
    return true;
}

cudaError_t launch_attention(const AttnArgs &a_in, KKind kk, int v_f32, uint32_t d, uint32_t max_cent,
                             uint32_t max_len, uint32_t forced_splits, uint32_t max_splits, int schedule,
                             uint32_t *splits_out, uint32_t *sk_out, cudaStream_t s, uint32_t *launches_out) {
    AttnArgs a = a_in;
    const uint32_t D = dim_template(d);
    const Entry e = pick_entry(kk, v_f32, D, a.rows);
    uint32_t row_stride = 0, scale_stride = 4;
    for (uint32_t h = 0; h < a.heads; ++h) {
        row_stride = std::max(row_stride, a.head[h].row_stride);
        scale_stride = std::max(scale_stride, a.head[h].scale_stride);
    }
    const uint32_t TT = attention_tile_tokens(d);
    int dev = 0, sms = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const Plan pl =
        attn::make_plan(kk, v_f32, D, e.qp, TT, row_stride, scale_stride, max_cent, (uint32_t)optin - 64u, 2, e.qm);
    if (pl.total > (uint32_t)optin) return cudaErrorInvalidConfiguration;
    // packed keys: the kernel specialised for the heads' group structures, once available.
    // Automatic mode keeps launches of one partial wave of the generic kernel on the generic
    // kernel: they are latency-bound, the specialised kernel's fewer instructions do not
    // shorten them, and its larger unrolled bodies (one per layer and head structure) start
    // every launch with cold instruction caches (the SmolLM2 decode step took 1.67 ms with
    // the specialised kernels against 1.28 ms with the generic one)
    const uint32_t chunk = attn::kWarps * TT, pairs = a.seq_count * a.heads;
    bool try_jit = kk == KKind::Packed && jit_mode() != 0;
    if (try_jit && jit_mode() == 2 && !forced_splits) {
        const int g_per_sm = std::max(1, e.occ(pl));
        const uint32_t g_slots = (uint32_t)(sms * g_per_sm);
        uint32_t sp = 1, tp = 0;
        choose_splits(pairs, max_len, chunk, g_slots, 0, std::max(1u, max_splits), &sp, &tp);
        if ((uint64_t)pairs * sp <= g_slots) try_jit = false;
    }
    const void *jk = nullptr;
    bool head_major = false;
    if (try_jit) {
        JitKey key{};
        key.D = D;
        key.QM = e.qm;
        key.vf32 = v_f32 ? 1u : 0u;
        key.heads = a.heads;
        bool ok = true;
        for (uint32_t h = 0; h < a.heads; ++h) {
            const AttnHead &hh = a.head[h];
            ok &= hh.ng >= 1 && hh.ng <= (uint32_t)kMaxGroups;
            key.head[h].ns = hh.ns;
            key.head[h].ng = hh.ng;
            for (uint32_t g = 0; g <= hh.ng && g <= (uint32_t)kMaxGroups; ++g) key.head[h].group_off[g] = hh.group_off[g];
        }
        if (ok) jk = jit_attention_kernel(key, s, &head_major);
    }
    int per_sm = jk ? jit_occupancy(jk, dev, pl.total) : e.occ(pl);
    if (per_sm < 1) per_sm = 1;
    uint32_t splits = 1, tps = 0;
    const uint32_t slots = (uint32_t)(sms * per_sm);
    choose_splits(pairs, max_len, chunk, slots, forced_splits, std::max(1u, max_splits), &splits, &tps);
    a.splits = splits;
    a.tokens_per_split = tps;
    a.sk_units = a.sk_tiles = a.sk_pair_tiles = 0;
    dim3 grid(splits, a.heads, a.seq_count);
    // Stream-K for launches that split-KV fits poorly in whole waves: one wave of equal
    // ranges of CTA tiles.  Only kernels that serve every head with one body (a head-major
    // grid has one body per group structure).
    if (!forced_splits && !head_major && max_len && schedule != 1) {
        uint32_t units = 0, per = 0;
        if (choose_stream_k(pairs, max_len, chunk, slots, splits, tps, std::max(1u, max_splits), schedule == 2, &units,
                            &per)) {
            a.sk_units = units;
            a.sk_tiles = per;
            a.sk_pair_tiles = (max_len + chunk - 1) / chunk;
            grid = dim3(units, 1, 1);
            splits = (a.sk_pair_tiles + per - 1) / per + 1;  // most segments of one pair
        }
    }
    if (splits_out) *splits_out = splits;
    if (sk_out) *sk_out = a.sk_units;
    // one partial wave of split-KV CTAs over packed keys: each CTA rotates its pair's queries
    // itself (the rotation, transposed in rows of D + 1 floats, the raw query rows and the
    // permutation and group tables staged in its tile buffers; the records and lookup offsets
    // in its P buffers), which takes a launch off the critical path of small batches; larger
    // launches rotate once per pair in a launch of their own
    const uint32_t stage_bytes = attn::kWarps * pl.warp_bytes, pbuf_bytes = pl.bars - pl.pbuf;
    a.fuse_q = kk == KKind::Packed && d <= 64u && !a.sk_units && (uint64_t)pairs * splits <= slots &&
                       stage_bytes >= 4u * (D * (D + 1) + kMaxRows * D) + 2u * D &&
                       pbuf_bytes >= 4u * D * e.qp + 2u * D
                   ? 1u
                   : 0u;
    if (launches_out) *launches_out = a.fuse_q ? 1u : 2u;
    cudaError_t err = cudaSuccess;
    if (!a.fuse_q) {
        err = launch_pdl(attn::qrot_kernel, dim3(a.heads, a.seq_count), dim3(128), 0, s, a, d, D, e.qp,
                         kk == KKind::Packed ? 1 : 0);
        if (err != cudaSuccess) return err;
    }
    if (jk) {
        uint32_t dd = d;
        Plan plc = pl;
        void *args[] = {&a, &plc, &dd};
        if (head_major) grid = dim3(splits, a.seq_count, a.heads);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(attn::kThreads);
        cfg.dynamicSmemBytes = pl.total;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelExC(&cfg, jk, args);
    }
    return e.run(a, pl, d, grid, s);
}

}  // namespace bgtq
