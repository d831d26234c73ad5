// Internal declarations shared by the C ABI (abi.cpp) and the kernels (*.cu).
#pragma once

// The kernel structs and constants below also compile under NVRTC (__CUDACC_RTC__), which
// builds layout-specialised attention kernels at run time (jit.cpp); host-only parts are
// guarded.
#ifndef __CUDACC_RTC__
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/bgtq.h"
#else
typedef unsigned char uint8_t;
typedef unsigned short uint16_t;
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;
typedef int int32_t;
typedef long long int64_t;
typedef unsigned long size_t;
#ifndef INFINITY
#define INFINITY (1.0f / 0.0f)
#endif
#endif

namespace bgtq {

constexpr int kMaxDim = 128;
constexpr int kMaxGroups = 8;
constexpr int kMaxHeads = 8;      // KV heads bound to one attention object / one launch
constexpr int kMaxRows = 8;       // query rows per KV head
constexpr uint32_t kTileRows = 64; // capacity is padded to a multiple of this

// Programmatic dependent launch.  Kernels of the decode chain (model GEMVs, K/V append,
// query rotation, attention) are launched with programmatic stream serialisation, so the
// next kernel's launch overlaps the end of the one before it; each of them waits for its
// predecessor's completion (griddepcontrol.wait) before it reads anything another kernel
// writes and before it writes any memory - only constant data (weights, the stores' own
// tables) is fetched ahead of the wait - and each allows its own successor to launch as
// soon as all of its CTAs have started (griddepcontrol.launch_dependents), so a successor
// only ever takes the slots the last wave frees.  Launched without the attribute, both are
// no-ops.
#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

// Device status word bits (bgtq_device_status).
constexpr uint32_t kStatusWaitTimeout = 1u;   // an mbarrier wait hit its iteration bound
constexpr uint32_t kStatusBadLength = 2u;     // a kernel saw a length beyond capacity

#ifndef __CUDACC_RTC__
// Host copy of one validated layout (src/webgpu/layout.ts:2-31) plus what the kernels
// derive from it once: compact per-dimension codebooks and group boundaries.
struct Layout {
    uint32_t d = 0, ng = 0, row_bytes = 0, norm_stride = 0, ns = 0, maxc = 0, ncb = 0;
    uint32_t logical_rb = 0, dev_row_stride = 0, dev_scale_stride = 0;
    std::vector<uint8_t> perm, group_of, pos_to_cb, lut;   // lut: ncb*256 codes
    std::vector<float> rot, cent, off, inv;                // rot d*d, cent d*maxc
    uint32_t group_off[kMaxGroups + 1] = {};               // group g = dims [off[g], off[g+1])
    uint32_t bound_mask[4] = {};                           // bit j: a group starts at dim j (j > 0)
    std::vector<uint16_t> cb_base;                         // compact centroid base per dim
    std::vector<float> cent_compact;                       // per-dim codebooks, 2^w entries each
    // Decode-attention lookup layout (build_lookup_layout): nibble dimensions in 512-byte
    // run slots, byte dimensions in power-of-two slots aligned to their size.
    std::vector<float> lookup;                             // the table, slot by slot
    std::vector<uint16_t> lookup_off;                      // per dim: float offset of its slot
    std::vector<uint32_t> ranges;                          // [2d] PackedKeys group ranges
};

// Parse + validate the flattened tables.  Returns BGTQ_OK or an error with message.
bgtq_status parse_layout(const uint32_t *config, size_t n_config, const float *table, size_t n_table, Layout &out,
                         std::string &err);
#endif  // __CUDACC_RTC__

// Device copy of one head's tables (one allocation, 16-byte aligned sections).
struct DeviceTables {
    void *blob = nullptr;
    size_t bytes = 0;
    const float *rot = nullptr;        // [d][d] row j = output j
    const float *cent = nullptr;       // compact codebooks
    const float *off = nullptr, *inv = nullptr;
    const uint8_t *lut = nullptr;      // [ncb][256]
    const uint8_t *perm = nullptr, *group_of = nullptr, *cbidx = nullptr;
    const uint16_t *cb_base = nullptr;
    const float *lookup = nullptr;     // Layout::lookup
    const uint16_t *lookup_off = nullptr;
};

// Per-head constants of the encode kernel.
struct EncodeHead {
    DeviceTables t;
    uint8_t *packed;           // base of sequence 0 row 0
    uint16_t *scales;
    uint64_t k_seq_stride;     // bytes between sequences
    uint64_t s_seq_stride;     // halves between sequences
    uint32_t row_stride;       // bytes between packed rows (an odd number of 32-bit words)
    uint32_t scale_stride;     // halves between scale rows (4 or 8)
    uint32_t ns, ng, n_cent, ncb;
    uint32_t bound_mask[4];
    uint32_t group_off[kMaxGroups + 1];
    uint64_t src_head_offset;  // elements added to the source address for this head
    uint32_t *lengths;         // device per-sequence lengths (updated by the launch)
};

struct EncodeArgs {
    EncodeHead head[kMaxHeads];
    const void *src;
    uint64_t row_stride, seq_stride;  // source elements
    const uint32_t *row0;             // device start row per sequence (nullable -> row0_scalar)
    uint32_t row0_scalar;
    uint32_t count, seq_first, seq_count, heads;
    int src_f32;
    uint32_t *status;                 // device status word (bounded-wait timeouts), nullable
};

// Model-path append: RoPE'd K and V of `count` tokens per sequence for `heads` KV heads,
// read from FP32 projections (src + s*seq_stride + t*row_stride; K of head h at k_offset +
// h*d, V at v_offset + h*d, in floats).
struct KvRopeArgs {
    EncodeHead head[kMaxHeads];
    void *v[kMaxHeads];             // FP16 value rows, sequence 0 row 0
    uint32_t *v_lengths[kMaxHeads];
    const void *k_src, *v_src;      // head h of token t of sequence s at + s*seq_stride + t*row_stride + h*dim
    const uint32_t *start;          // device lengths of the first key store (start rows)
    uint64_t v_seq_stride[kMaxHeads];  // halves between sequences of each value store
    uint64_t row_stride, seq_stride;   // source elements
    uint32_t k_f16, v_f16, rope;       // FP16 (else FP32) sources; RoPE on K with inv_freq
    uint32_t count, seq_first, seq_count, heads, vD, v_swizzle;
    uint32_t capacity;              // rows every store can hold: rows at or past it are refused
    uint32_t *status;               // device status word (kStatusBadLength on a refusal)
    uint32_t *ticket;               // zero between launches: counts finished CTAs
    float inv_freq[kMaxDim / 2];
};

// Per-head constants of the attention kernels.
struct AttnHead {
    const uint8_t *k;          // packed rows | FP16 K rows | FP32 K rows, sequence 0 row 0
    const uint16_t *scales;
    const void *v;
    const float *rot;          // dense rotation (packed path)
    const float *cent;         // compact codebooks (packed path)
    const float *lookup;       // decode-attention lookup layout of the codebooks
    const uint16_t *lookup_off;
    const uint8_t *perm, *group_of;
    uint64_t k_seq_stride;     // bytes
    uint64_t s_seq_stride;     // halves
    uint64_t v_seq_stride;     // bytes
    uint32_t row_stride;       // bytes between K rows
    uint32_t scale_stride;     // halves
    uint32_t ns, ng, n_cent, n_lookup;
    uint32_t bound_mask[4];
    uint32_t group_off[kMaxGroups + 1];
    uint16_t cb_base[kMaxDim];
};

struct AttnArgs {
    AttnHead head[kMaxHeads];
    const float *q;            // [S][H][R][d]
    float *qt;                 // [S][H][D][QP] query records (written by qrot_kernel)
    const uint32_t *positions; // [S][R] or null
    const uint32_t *lengths;   // [sequences] key lengths (device), indexed seq_first + s
    float *out;                // [S][H][R][D]
    float *logits;             // optional [S][H][R][logit_stride]
    float *lse;                // optional [S][H][R]
    float *part;               // [splits][S][H][R][D + 2]
    uint32_t *counters;        // [S][H], zero between launches
    uint32_t *status;
    const float *rope;         // optional [d/2] RoPE table: queries arrive before RoPE
    uint32_t seq_first, seq_count, heads, rows, splits, tokens_per_split, causal, logit_stride;
    // stream-K (sk_units != 0 CTAs): each pair spans sk_pair_tiles tiles of kWarps warp tiles,
    // dealt to the CTAs sk_tiles at a time in head-major pair order; splits is then unused
    uint32_t sk_units, sk_tiles, sk_pair_tiles;
    uint32_t fuse_q;  // split-KV CTAs rotate their pair's queries themselves (no rotation launch)
};

// Prefill: n query positions per sequence, all gqa query heads of each KV head.
struct PrefillArgs {
    AttnHead head[kMaxHeads];
    const float *q;            // [S][n][heads*gqa][d]
    float *qt;                 // [S][n][heads*gqa][64] code-domain queries (rotation kernel)
    float *out;                // [S][n][heads*gqa][d]
    const uint32_t *lengths;   // [sequences] key lengths (device), indexed seq_first + s
    uint32_t *status;
    const float *rope;         // optional [d/2] RoPE table: queries arrive before RoPE
    uint32_t seq_first, seq_count, heads, gqa, n, pos_first, d;
};

struct ReconArgs {
    DeviceTables t;
    const uint8_t *packed;
    const uint16_t *scales;
    uint32_t row_stride, scale_stride, ns, d, rows;
    float *out;
};

enum class KKind { Packed, F16, F32 };

#ifndef __CUDACC_RTC__
// Kernel launchers (return cudaError_t of the launch).
cudaError_t launch_encode(const EncodeArgs &a, uint32_t d, uint32_t smem_cent_floats, uint32_t max_ncb,
                          cudaStream_t s);
cudaError_t launch_kv_rope_append(const KvRopeArgs &a, uint32_t d, cudaStream_t s);
cudaError_t launch_copy_rows(void *dst, uint64_t dst_seq_stride, uint32_t dst_row_elems, int dst_f32,
                             const void *src, uint64_t src_row_stride, uint64_t src_seq_stride, int src_f32,
                             const uint32_t *row0, uint32_t row0_scalar, uint32_t count, uint32_t seq_first,
                             uint32_t seq_count, uint32_t *lengths, uint32_t d, int swizzle, cudaStream_t s);
// FP16 value rows of 64 or 128 halves are stored chunk-swizzled (see copy_rows_kernel).
inline bool values_swizzled(int f32, uint32_t D) { return !f32 && (D == 64 || D == 128); }
cudaError_t launch_reconstruct(const ReconArgs &a, uint32_t n_cent, cudaStream_t s);


// Attention over a.seq_count sequences x a.heads KV heads; picks the split-KV factor
// (forced_splits = 0: automatic) and writes it to *splits_out, or a stream-K schedule
// (schedule 0: when it is estimated faster; 1: never; 2: whenever the kernel allows) and
// writes its CTA count to *sk_out (0 for split-KV); *launches_out: kernels launched (the
// query rotation runs inside the attention CTAs of a launch of one partial wave).
cudaError_t launch_attention(const AttnArgs &a, KKind kk, int v_f32, uint32_t d, uint32_t max_cent,
                             uint32_t max_len, uint32_t forced_splits, uint32_t max_splits, int schedule,
                             uint32_t *splits_out, uint32_t *sk_out, cudaStream_t s, uint32_t *launches_out = nullptr);
// Causal prefill attention (packed keys, FP16 values, head dim <= 64): the query rotation,
// then the tcgen05/TMEM kernel (umma != 0) or the mma.sync kernel.
cudaError_t launch_prefill(const PrefillArgs &a, uint32_t max_cent, int umma, cudaStream_t s);
cudaError_t launch_prefill_tc(const PrefillArgs &a, uint32_t max_cent, cudaStream_t s);
cudaError_t launch_probs(const float *logits, const float *lse, float *probs, uint64_t rows, uint32_t tokens,
                         uint32_t stride, cudaStream_t s);
// Query rows per CTA tile (the QM template) the decode-attention kernels use for `rows` rows.
uint32_t attention_qm(KKind kk, uint32_t rows);
// Loads the code of every generic decode-attention kernel for keys of kind kk (and the
// query rotation) on the current device, so that later launches load nothing.
cudaError_t preload_attention_kernels(KKind kk);
// Shared-memory bytes the attention kernel needs for a launch; 0 if unsupported.
size_t attention_smem_bytes(KKind kk, int v_f32, uint32_t d, uint32_t rows_bound, uint32_t row_stride,
                            uint32_t scale_stride, uint32_t max_cent);
uint32_t attention_tile_tokens(uint32_t d);
// Layout-specialised decode attention (jit.cpp): the kernel for the heads' group structures
// of packed keys, compiled at run time; null while it is not (yet) available, in which case
// the generic kernel runs.  *head_major: the kernel takes the grid (splits, sequences, heads)
// instead of (splits, heads, sequences).
struct JitLayout {
    uint32_t ns, ng;
    uint32_t group_off[kMaxGroups + 1];
};
struct JitKey {
    uint32_t D, QM, vf32, heads;
    JitLayout head[kMaxHeads];
};
const void *jit_attention_kernel(const JitKey &key, cudaStream_t stream, bool *head_major);
void jit_set_enabled(int on);  // 0 off, 1 every launch, 2 automatic
int jit_mode();
// The calling thread's launches keep the generic kernel while on != 0 (an entry point that
// promises no allocation at attention time: loading a specialised kernel allocates).
void jit_suppress_on_thread(int on);

// Launch `kern` with programmatic stream serialisation (see pdl_wait).
#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}
#endif
uint32_t *device_status_word(int device);  // lazily allocated per device
uint32_t *device_status_word_if_present(int device);  // never allocates; null if absent
void set_last_error(const std::string &message);     // message of bgtq_last_error()

#endif  // __CUDACC_RTC__

}  // namespace bgtq
