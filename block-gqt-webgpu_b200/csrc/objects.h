// Definitions of the opaque C ABI objects, shared by the ABI translation units.
#pragma once

#include <vector>

#include "bgtq_internal.h"

namespace bgtq {

// Device buffer that grows on demand (staging and workspace of the ABI objects).
struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    cudaError_t ensure(size_t n) {
        if (n <= bytes) return cudaSuccess;
        release();
        cudaError_t e = cudaMalloc(&p, n);
        if (e == cudaSuccess) bytes = n;
        return e;
    }
};

}  // namespace bgtq

struct bgtq_tables {
    int device = 0;
    bgtq::Layout L;
    bgtq::DeviceTables dt;
};

struct bgtq_keys {
    bgtq_keys_kind kind;
    int device = 0;
    bgtq::Layout L;          // packed/compressed only
    bgtq::DeviceTables dt;
    uint32_t dim = 0, D = 0, capacity = 0, cap_alloc = 0, sequences = 0;
    uint32_t row_stride = 0;    // bytes between device rows
    uint32_t scale_stride = 0;  // halves between device scale rows
    uint8_t *rows = nullptr;
    uint16_t *scales = nullptr;
    uint32_t *d_lengths = nullptr;
    std::vector<uint32_t> lengths;
    bgtq::DevBuf row0, staging, materialized;
    std::vector<bgtq_allocation> ledger;
};

struct bgtq_values {
    bgtq_dtype dtype;
    int device = 0;
    uint32_t dim = 0, D = 0, capacity = 0, cap_alloc = 0, sequences = 0;
    void *data = nullptr;
    uint32_t *d_lengths = nullptr;
    std::vector<uint32_t> lengths;
    bgtq::DevBuf row0, staging;
};

struct bgtq_attention {
    uint32_t heads = 0, rows = 0, dim = 0, sequences = 0;
    int device = 0;
    std::vector<bgtq_keys *> keys;
    std::vector<bgtq_values *> values;
    float *part = nullptr;
    uint32_t *counters = nullptr;
    float *lse = nullptr;
    float *qt = nullptr;
    bgtq::DevBuf q_dev, pos_dev, out_dev, logits_dev, probs_dev, prefill_qt;
    uint32_t forced_splits = 0, last_splits = 0, last_launches = 0, max_splits = 64, last_sk_units = 0;
    int schedule = 0;  // 0 automatic, 1 split-KV only, 2 stream-K whenever the kernel allows
    uint32_t prefill_kernel = 0;  // 0: tcgen05 / TMEM kernel, 1: mma.sync kernel
    bgtq::DevBuf rope;            // RoPE table when queries arrive before RoPE (else empty)
    bool use_rope = false;
    bool plan_capacity = false;   // split plan for the keys' capacity (graph replays)
};

namespace bgtq {
// Kernel arguments of one packed-key head with its value store (every attention entry
// point over packed keys fills its heads through this one function).
void fill_packed_head(AttnHead &ah, const bgtq_keys *k, const bgtq_values *v);
// Encode arguments of one packed-key store (every K append fills its heads through this).
void fill_encode_head(const bgtq_keys *k, EncodeHead &h);
}  // namespace bgtq
