/*
 * bgtq.h - C ABI of the B200 Block-GTQ key-cache library (libbgtq.so).
 *
 * Two hot paths, each a hand-written sm_100a CUDA kernel:
 *   1. K encode: permute -> per-group norm -> block-diagonal rotation -> LUT
 *      quantisation -> nibble/byte packing + FP16 corrected scales.
 *   2. Compressed-K GQA attention: flash-decoding over packed K rows and an FP16 or
 *      FP32 V cache; each key is dequantised in registers against a query rotated
 *      into the code domain, never materialised.
 *
 * The objects mirror the reference's TypeScript surface (reference paths are inside
 * the amw720386/block-gqt-webgpu repository):
 *   bgtq_tables      <- BlockGTQParameters + tables()/validateLayout()  src/webgpu/layout.ts:2-31
 *   bgtq_keys        <- PackedKeys      src/runtime/packed-keys.ts:7-52
 *                       FP16Keys        src/runtime/keys.ts:16-27
 *                       CompressedKeys  src/runtime/compressed-keys.ts:5-59
 *   bgtq_values      <- Values          src/runtime/values.ts:3-16 (FP32) and the
 *                       model's FP16 V cache  src/model/decoder.ts:20-21, append.wgsl:6-10
 *   bgtq_attention   <- OptimizedAttention  src/attention/optimized.ts:5-45 and
 *                       AttentionSession    src/attention/attention.ts:19-70
 * A WebGPU buffer per object becomes device memory owned by the object; the
 * reference's single sequence per store generalises to `sequences` independent
 * sequences so that one object covers one (layer, KV head) of a whole batch.
 *
 * Conventions
 *   - Every function returns a bgtq_status.  Status codes map onto the reference's
 *     synchronous errors: RangeError -> BGTQ_EINVAL / BGTQ_ECAPACITY / BGTQ_ENONFINITE /
 *     BGTQ_ELAYOUT, Error -> BGTQ_EBUSY / BGTQ_ELAYOUT.  Validation happens before any
 *     state changes, so a rejected call leaves the object untouched
 *     (tests/webgpu/runtime-contracts.ts:24-25).  bgtq_last_error() gives the message.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).  Work
 *     is stream-ordered; objects are not thread-safe.
 *   - Pointers flagged `host` are ordinary (ideally pinned) host memory; otherwise they
 *     are device pointers on the object's device.
 *   - No C++ exception crosses this boundary; no call allocates on the hot path.
 */
#ifndef BGTQ_H
#define BGTQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t bgtq_status;
enum {
    BGTQ_OK = 0,
    BGTQ_EINVAL = 1,      /* RangeError: shapes, counts, positions  (keys.ts:12, optimized.ts:30) */
    BGTQ_ECAPACITY = 2,   /* RangeError: capacity exceeded          (keys.ts:14, values.ts:12) */
    BGTQ_ENONFINITE = 3,  /* RangeError: non-finite input           (keys.ts:13, buffers.ts:19-21) */
    BGTQ_EBUSY = 4,       /* Error: storage not ready / K,V mismatch (packed-keys.ts:50, optimized.ts:34) */
    BGTQ_ELAYOUT = 5,     /* RangeError/Error: layout or tables     (layout.ts:8-23, packed-keys.ts:15-23) */
    BGTQ_ETIMEOUT = 6,    /* a bounded device wait expired; the device status word says where */
    BGTQ_ECUDA = 7,       /* CUDA runtime error */
    BGTQ_ENOMEM = 8       /* device or host allocation failed */
};

typedef enum { BGTQ_F16 = 1, BGTQ_F32 = 2 } bgtq_dtype;
typedef enum { BGTQ_KEYS_PACKED = 1, BGTQ_KEYS_FP16 = 2, BGTQ_KEYS_COMPRESSED = 3 } bgtq_keys_kind;

typedef struct bgtq_tables bgtq_tables;
typedef struct bgtq_keys bgtq_keys;
typedef struct bgtq_values bgtq_values;
typedef struct bgtq_attention bgtq_attention;

/* Shape of a validated layout.  row_bytes / norm_stride are the reference's strides
 * (config[2], config[3]); the device strides pad them to 16 B / 8 B for aligned loads. */
typedef struct bgtq_layout_info {
    uint32_t dim, groups, row_bytes, norm_stride, nibble_dims, max_centroids;
    uint32_t logical_row_bytes;   /* nibble_dims/2 + dim - nibble_dims */
    uint32_t device_row_stride;   /* bytes between packed rows in device memory */
    uint32_t device_scale_stride; /* FP16 scales between rows in device memory */
    uint32_t codebooks;           /* code LUT rows (config payload / 256) */
} bgtq_layout_info;

/* One device allocation owned by an object, with the reference's ledger roles
 * ("persistent-k", "persistent-v", "shared", "scratch"; src/webgpu/buffers.ts:1). */
typedef struct bgtq_allocation {
    const char *name;
    const char *role;
    uint64_t bytes;
} bgtq_allocation;

/* ---- errors ------------------------------------------------------------------ */
const char *bgtq_status_string(bgtq_status s);
/* Message of the last failing call on this thread ("" if none). */
const char *bgtq_last_error(void);
/* Library version string. */
const char *bgtq_version(void);

/* ---- host-only helpers (no GPU needed) ----------------------------------------- */

/* Greedy bit allocation: widths minimising sum s_i*4^-b_i with sum b_i = budget,
 * min_bits <= b_i <= max_bits; first index wins ties; priorities in FP64 of FP32 scores.
 * Replaces src/reference/allocator.py:4-17 (upstream vendor/blockgtq/allocator.py:20-55). */
bgtq_status bgtq_allocate_bits(const float *scores, uint32_t n, int64_t budget, int32_t min_bits,
                               int32_t max_bits, int64_t *widths_out);

/* Table builder: per-pair widths[dim/2] (1..8) -> the flattened config (u32) and table (f32)
 * of src/webgpu/layout.ts:24-31, as the reference's calibration builds them:
 * BlockGTQPipeline._post_allocation_setup (vendor/blockgtq/block_gtq_pipeline.py:151-246:
 * pairs ordered by width, one group per width, identity blocks below rotation_threshold and
 * NumPy-seeded Haar rotations (seed 42 + width) at or above it, Lloyd-Max centroids),
 * build_code_lut (vendor/blockgtq/quant_kernels.py:276-364) and build_pack_meta
 * (vendor/blockgtq/quantizer.py:34-106).  Pairs are ordered by width as torch.argsort
 * orders them (equal widths by libstdc++ std::sort over (width, index)), or by pair_order
 * when it is given (a width-ascending permutation of the pairs, e.g. an existing
 * calibration's).  row_pad bytes are added to the packed row;
 * norm_stride 0 means the group count.  With config or table NULL only the lengths are
 * returned (size query). */
bgtq_status bgtq_tables_build(uint32_t dim, const int64_t *widths, const int64_t *pair_order,
                              uint32_t rotation_threshold, uint32_t row_pad, uint32_t norm_stride, uint32_t *config,
                              size_t config_capacity, size_t *config_len, float *table, size_t table_capacity,
                              size_t *table_len);

/* The Haar rotation of size n that NumPy gives for default_rng(seed) (standard normals, QR,
 * columns signed by diag(R), det +1), row-major FP32 (block_gtq_pipeline.py:81-92). */
bgtq_status bgtq_haar_rotation(uint32_t n, uint64_t seed, float *out);

/* MSE-optimal scalar centroids (2^bits values, ascending, FP32) for N(0, 1/n)
 * (block_gtq_pipeline.py:24-78). */
bgtq_status bgtq_optimal_centroids(uint32_t bits, uint32_t n, float *out);

/* Layout-specialised decode attention: launches over packed keys use a kernel compiled at run
 * time for their heads' group structures (the toolkit's nvcc, else NVRTC; once per key and
 * process; identical results, fewer instructions).  Heads sharing one structure compile on the
 * first launch; heads with several compile on a background thread while the generic kernel
 * runs, and a later launch outside a graph capture loads the result.  on = 0 keeps the
 * generic kernel (also BGTQ_LAYOUT_JIT=0 in the environment), 1 specialises every launch
 * (BGTQ_LAYOUT_JIT=1), 2 (the default) every launch of more than one wave of CTAs: launches of
 * one partial wave are latency-bound and stay on the generic kernel.  No counterpart in the
 * reference. */
bgtq_status bgtq_set_layout_jit(int on);
/* Specialised kernels loaded / keys that failed to build (and use the generic kernel). */
bgtq_status bgtq_layout_jit_stats(uint32_t *built, uint32_t *failed);
/* The same counters with the compile step apart: kernels compiled (cubins ready, whether or
 * not a launch has loaded them yet), loaded, and failed.  Any pointer may be NULL. */
bgtq_status bgtq_layout_jit_counts(uint32_t *compiled, uint32_t *loaded, uint32_t *failed);
/* Wait up to timeout_ms for the background compiles queued so far, then load every compiled
 * kernel, so the next launches (and a graph recorded after this call) use them.  Call it
 * outside a graph capture.  BGTQ_ETIMEOUT if compiles were still running at the limit (what
 * had finished is loaded). */
bgtq_status bgtq_layout_jit_wait(uint32_t timeout_ms);

/* Ahead-of-time layout-specialised kernel: compiles the decode-attention kernel for `heads`
 * packed-key heads with these flattened tables (config/table as for bgtq_tables_create),
 * `rows` query rows per head and FP16 (v_f32 = 0) or FP32 values with the toolkit's nvcc
 * (host only, no GPU needed) and stores the cubin in `dir` under a name made from the heads'
 * group structures and the kernel sources (written to name_out if given; an existing file of
 * that name is kept).  Launches look in bgtq/aot/ beside the library first, so a process on
 * a host without the toolkit still gets the specialised kernel for prebuilt structures.  No
 * counterpart in the reference. */
bgtq_status bgtq_layout_jit_prebuild(const char *dir, uint32_t heads, const uint32_t *const *configs,
                                     const size_t *n_configs, const float *const *tables, const size_t *n_tables,
                                     uint32_t rows, int v_f32, char *name_out, size_t name_capacity);
/* Keys whose kernel this process took from a prebuilt cubin. */
bgtq_status bgtq_layout_jit_prebuilt(uint32_t *n);

/* Fixture files of the reference's tests (tests/oracles/fixture.py:13-49): a JSON manifest
 * (metadata + array descriptors dtype f32/u32/u8/f16/u16, shape, offset, nbytes) beside a
 * little-endian payload checked by length and SHA-256.  Read errors are BGTQ_ELAYOUT with
 * read_fixture's messages ("Unsupported fixture format", "Fixture payload length/hash
 * mismatch", "Invalid array descriptor: <name>"). */
typedef struct bgtq_fixture bgtq_fixture;
bgtq_status bgtq_fixture_read(const char *json_path, bgtq_fixture **out);
bgtq_status bgtq_fixture_array_count(const bgtq_fixture *f, uint32_t *n);
/* Array `index` in manifest order; data points into the fixture (valid until destroy). */
bgtq_status bgtq_fixture_array(const bgtq_fixture *f, uint32_t index, const char **name, const char **dtype,
                               uint32_t *ndim, const uint64_t **shape, const void **data, uint64_t *nbytes);
/* The manifest text as read (metadata included). */
bgtq_status bgtq_fixture_manifest(const bgtq_fixture *f, const char **json);
void bgtq_fixture_destroy(bgtq_fixture *f);
/* write_fixture: arrays (C order) into <json_path stem>.bin, each on a 4-byte boundary, and
 * the manifest = metadata_json (a JSON object, may be NULL) + version (kept if given, else
 * 1), endianness, binary, byte_length, sha256, arrays. */
bgtq_status bgtq_fixture_write(const char *json_path, const char *metadata_json, uint32_t n_arrays,
                               const char *const *names, const char *const *dtypes, const uint32_t *ndims,
                               const uint64_t *const *shapes, const void *const *data);

/* validateLayout() plus the PackedKeys inverse-group check, on host memory only.
 * config/table are the flattened tables() output (src/webgpu/layout.ts:24-31).
 * ranges_out (nullable, 2*dim entries) receives the [start,end) group bounds of each
 * dimension exactly as PackedKeys builds them (src/runtime/packed-keys.ts:15-23). */
bgtq_status bgtq_layout_validate(const uint32_t *config, size_t n_config, const float *table, size_t n_table,
                                 uint32_t *ranges_out, bgtq_layout_info *info_out);

/* ---- tables ------------------------------------------------------------------------ */

/* Validate and upload one head's tables to `device`.  Replaces tables() + the upload of
 * the K integer/float tables and `ranges` (packed-keys.ts:24-27). */
bgtq_status bgtq_tables_create(const uint32_t *config, size_t n_config, const float *table, size_t n_table,
                               int device, bgtq_tables **out);
bgtq_status bgtq_tables_info(const bgtq_tables *t, bgtq_layout_info *info_out);
void bgtq_tables_destroy(bgtq_tables *t);

/* ---- key stores ------------------------------------------------------------------- */

/* kind PACKED/COMPRESSED need tables (dim is taken from them); FP16 needs dim only.
 * capacity <= 2^31 rows per sequence (the reference caps at the WebGPU dispatch limit,
 * packed-keys.ts:13).  Device memory is zero-filled, as WebGPU buffers are. */
bgtq_status bgtq_keys_create(bgtq_keys_kind kind, const bgtq_tables *tables, uint32_t dim, uint32_t capacity,
                             uint32_t sequences, int device, bgtq_keys **out);
void bgtq_keys_destroy(bgtq_keys *k);

/* Append `count` rows to each of `seq_count` sequences starting at `seq_first`.
 * src element (s, r, i) is at src[s*seq_stride + r*row_stride + i] (elements of dtype).
 * F16 sources are FP16 bits (PackedKeys.append(Uint16Array), keys.ts:11-15); F32 sources
 * are rounded to FP16 first (model path, src/model/codec.wgsl:14).  Host sources are
 * checked for whole non-empty rows and finite values before anything is written; device
 * sources are trusted like the reference's GPU-resident model path.  Packed/compressed
 * stores run the encode kernel; FP16 stores copy (converting F32). */
bgtq_status bgtq_keys_append(bgtq_keys *k, const void *src, bgtq_dtype dtype, int host, uint32_t count,
                             uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                             void *stream);
bgtq_status bgtq_keys_length(const bgtq_keys *k, uint32_t seq, uint32_t *length_out);
/* Model-path append of one layer (src/model/decoder.ts:44-50: RoPE on K, encode_k per KV
 * head, V append) in one launch: for `count` new tokens of sequences [seq_first,
 * seq_first+seq_count), reads the FP32 projections at src + s*seq_stride + t*row_stride
 * (floats; K of KV head h at k_offset + h*dim, V at v_offset + h*dim), applies split-half
 * RoPE (src/model/kernels.wgsl:49-54) to K at each token's cache row with the host table
 * inv_freq[dim/2], encodes it into keys[h] and writes V as FP16 into values[h].  Needs
 * packed keys and FP16 values of one head dim with equal lengths; src is device memory;
 * stream-ordered (start rows are read from the device). */
bgtq_status bgtq_append_kv_rope(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, const float *src,
                                uint64_t row_stride, uint64_t seq_stride, uint32_t k_offset, uint32_t v_offset,
                                uint32_t count, uint32_t seq_first, uint32_t seq_count, const float *inv_freq,
                                void *stream);
/* K/V append of one layer for `heads` KV heads in one launch (the per-head
 * PackedKeys.append + Values.append of src/runtime/packed-keys.ts:39-48 and
 * src/runtime/values.ts:9-14, batched): K and V of head h, token t, sequence s at
 * src + s*seq_stride + t*row_stride + h*dim elements (FP16 or FP32, no RoPE); K is
 * FP16-rounded and encoded into keys[h], V written as FP16 into values[h].  Needs packed
 * keys and FP16 values of one head dim with equal lengths.  host != 0: the sources are host
 * memory holding dense [seq_count][count][heads][dim] blocks, checked for finite values
 * (BGTQ_ENONFINITE) and uploaded in stream order without a host wait - page-locked sources
 * must stay unchanged until the stream has passed the call, and host appends to the same
 * first store share its staging buffer, so issue them on one stream.  Stream-ordered. */
bgtq_status bgtq_append_kv(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, const void *k_src,
                           bgtq_dtype k_dtype, const void *v_src, bgtq_dtype v_dtype, int host, uint32_t count,
                           uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                           void *stream);
/* Start every sequence of the store over (lengths 0), keeping its capacity: a new request
 * reusing the cache.  Rows past a length are never attended, so their old contents stay
 * until appends overwrite them.  No counterpart in the reference (its stores only grow);
 * stream-ordered like appends. */
bgtq_status bgtq_keys_reset(bgtq_keys *k, void *stream);
bgtq_status bgtq_keys_info(const bgtq_keys *k, bgtq_keys_kind *kind, uint32_t *dim, uint32_t *capacity,
                           uint32_t *sequences);

/* The Block-GTQ layout of a packed / compressed key store (its tables' shape and strides). */
bgtq_status bgtq_keys_layout(const bgtq_keys *k, bgtq_layout_info *info_out);

/* Copy rows [row0, row0+count) of sequence `seq` to host memory in the reference's
 * strides: packed rows of config rowBytes bytes, scales of config normStride FP16 bits
 * (zero padded), as the reference's packed/norms GPU buffers hold them.  FP16 stores
 * return FP16 K rows in `packed_out` (2*dim bytes each) and ignore scales_out.
 * Synchronous (inspection / tests only). */
bgtq_status bgtq_keys_read(const bgtq_keys *k, uint32_t seq, uint32_t row0, uint32_t count, uint8_t *packed_out,
                           uint16_t *scales_out);

/* CompressedKeys.prepare(): materialise FP32 K of sequence `seq` (all `length` rows) into
 * device memory `out` [length][dim] (mixed.wgsl:decode).  Test/debug path. */
bgtq_status bgtq_keys_reconstruct(const bgtq_keys *k, uint32_t seq, float *out, void *stream);

bgtq_status bgtq_keys_allocations(const bgtq_keys *k, bgtq_allocation *out, uint32_t capacity_n, uint32_t *n_out);

/* ---- value stores ----------------------------------------------------------------- */

/* dtype F32 mirrors the synthetic Values (values.ts:7); F16 mirrors the model V cache. */
bgtq_status bgtq_values_create(bgtq_dtype dtype, uint32_t dim, uint32_t capacity, uint32_t sequences, int device,
                               bgtq_values **out);
void bgtq_values_destroy(bgtq_values *v);
/* Same addressing and validation as bgtq_keys_append (values.ts:9-14). */
bgtq_status bgtq_values_append(bgtq_values *v, const void *src, bgtq_dtype dtype, int host, uint32_t count,
                               uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                               void *stream);
bgtq_status bgtq_values_length(const bgtq_values *v, uint32_t seq, uint32_t *length_out);
bgtq_status bgtq_values_info(const bgtq_values *v, bgtq_dtype *dtype, uint32_t *dim, uint32_t *capacity,
                             uint32_t *sequences);
/* Copy rows [row0, row0+count) of sequence `seq` to host memory as the store holds them:
 * FP16 bits or FP32, `dim` elements per row, in dimension order (the device layout's chunk
 * swizzle undone).  Synchronous (inspection / tests only).  No counterpart in the reference. */
bgtq_status bgtq_values_read(const bgtq_values *v, uint32_t seq, uint32_t row0, uint32_t count, void *out);
/* As bgtq_keys_reset, for a value store. */
bgtq_status bgtq_values_reset(bgtq_values *v, void *stream);

/* ---- attention ------------------------------------------------------------------- */

/* Bind `heads` KV heads (keys[h], values[h]) that share dim, capacity and sequence
 * count; each head serves up to `rows` query rows (GQA group size x query positions;
 * the reference's maxQueries, optimized.ts:20).  rows <= 8.  Mirrors
 * OptimizedAttention.create (optimized.ts:20-28) / AttentionEngine.session. */
bgtq_status bgtq_attention_create(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, uint32_t rows,
                                  bgtq_attention **out);
void bgtq_attention_destroy(bgtq_attention *a);

/* One attention pass for sequences [seq_first, seq_first+seq_count) with `rows` query
 * rows per head (<= the bound rows).
 *   q        [seq_count][heads][rows][dim] FP32 (GQA: query head h*rows+r uses KV head h)
 *   positions [seq_count][rows] u32 context positions, or NULL for "last token"
 *   causal   mask tokens t > position (attention.wgsl:15); non-causal attends all keys
 *   out      [seq_count][heads][rows][dim] FP32
 *   logits   optional [seq_count][heads][rows][length] FP32 (inspect(): raw q.k/sqrt(d),
 *            -inf where masked); needs equal lengths across the sequences
 *   probs    optional, same shape as logits (requires logits)
 * host=1: q/positions/out/logits/probs are host memory, copied inside the call, which
 * returns with the outputs in place.  host=2: the same, but the call does not wait: the
 * downloads are queued on the stream and the outputs are valid once the caller has
 * synchronised it (page-locked outputs; q may be reused on return).  Calls on one attention
 * object share its staging buffers, so issue them on one stream.
 * Errors (optimized.ts:29-35): empty or mismatched K/V lengths, rows out of range,
 * positions >= length, non-finite host Q.  Mirrors setQueries()+attend(). */
bgtq_status bgtq_attend(bgtq_attention *a, const float *q, const uint32_t *positions, int causal, uint32_t rows,
                        uint32_t seq_first, uint32_t seq_count, float *out, float *logits, float *probs, int host,
                        void *stream);

/* Causal prefill over packed keys: the model path's chunked prefill (src/model/decoder.ts:
 * 30-81; compressed_dot / softmax / weighted, src/model/compressed-dot.wgsl:14-31 and
 * src/model/attention.wgsl:13-39) for n query positions pos_first .. pos_first+n-1 of
 * sequences [seq_first, seq_first+seq_count), all gqa query heads of each of the object's
 * KV heads (query head h*gqa + r uses KV head h).  q and out: [seq_count][n][heads*gqa][dim]
 * FP32, token-major like a model's activations; a row at position p sees keys 0..p.
 * Requires packed keys, FP16 values, dim <= 64, gqa 1..8, and keys/values appended up to
 * pos_first+n on every sequence (equal K/V lengths).  host != 0: q/out are host memory
 * (staged, call synchronises).  Errors: BGTQ_EINVAL (shape, kind, positions), BGTQ_EBUSY
 * (K/V lengths), BGTQ_ENONFINITE (host Q). */
bgtq_status bgtq_attend_prefill(bgtq_attention *a, const float *q, uint32_t pos_first, uint32_t n, uint32_t gqa,
                                uint32_t seq_first, uint32_t seq_count, float *out, int host, void *stream);

/* Split-KV factor the last bgtq_attend used (diagnostics / benches). */
bgtq_status bgtq_attention_last_splits(const bgtq_attention *a, uint32_t *splits_out);
/* Force a split-KV factor (0 = automatic). */
bgtq_status bgtq_attention_set_splits(bgtq_attention *a, uint32_t splits);
/* Decode schedule: 0 automatic (stream-K when estimated faster than split-KV: launches whose
 * split-KV grid fills its last wave poorly), 1 split-KV only, 2 stream-K whenever the kernel
 * allows (tests).  Stream-K deals the pairs' key tiles to one wave of CTAs in equal ranges;
 * a forced split count (set_splits) implies split-KV.  No counterpart in the reference,
 * whose decode is one workgroup per (query head, position). */
bgtq_status bgtq_attention_set_schedule(bgtq_attention *a, int mode);
/* CTAs of the last bgtq_attend's stream-K launch, 0 when it used split-KV. */
bgtq_status bgtq_attention_last_stream_k(const bgtq_attention *a, uint32_t *units_out);
/* For launches recorded once (CUDA graph capture) and replayed while sequences grow: on != 0
 * makes bgtq_attend plan its split-KV factor for the keys' capacity instead of the current
 * lengths, so a replay covers every row appended since.  No counterpart in the reference. */
bgtq_status bgtq_attention_plan_for_capacity(bgtq_attention *a, int on);
/* Replayed appends (bgtq_append_kv_rope inside a graph) advance the device lengths only;
 * these copy them back to the host-side bookkeeping that later calls validate against. */
bgtq_status bgtq_keys_sync_lengths(bgtq_keys *k);
bgtq_status bgtq_values_sync_lengths(bgtq_values *v);
/* Queries arrive before RoPE (the model path's raw Q projection): bgtq_attend and
 * bgtq_attend_prefill apply split-half RoPE (src/model/kernels.wgsl:49-54) with the table
 * inv_freq[n], n = dim/2, at each query's position (positions[], else the last appended
 * row; prefill: pos_first + t) before attending.  n = 0 turns it off. */
bgtq_status bgtq_attention_set_rope(bgtq_attention *a, const float *inv_freq, uint32_t n);
/* Which tensor-core kernel bgtq_attend_prefill runs: 0 = tcgen05 UMMA with TMEM
 * accumulators (default), 1 = mma.sync (diagnostics, A/B comparisons).  Both compute the
 * same causal attention to the same tolerance. */
bgtq_status bgtq_attention_set_prefill_kernel(bgtq_attention *a, uint32_t kernel);
/* Number of kernel launches issued by the last bgtq_attend (benches count launches). */
bgtq_status bgtq_attention_last_launches(const bgtq_attention *a, uint32_t *launches_out);

/* Attention without any device allocation (no counterpart in the reference, which has
 * no such constraint).  For callers that must not allocate device memory when they run
 * attention: a server whose memory pool has taken all free device memory once the
 * caches exist, or a plugin inside a framework that owns every device allocation and
 * forbids the plugin's own cudaMalloc.  It needs no bgtq_attention object: `heads` packed
 * key stores and their value stores (same rules as bgtq_attention_create) are attended
 * directly, with device pointers only (q/positions/out as in bgtq_attend; no logit
 * capture; always the generic, ahead-of-time compiled kernel).  Scratch comes from one
 * fixed array of 4 MiB + 64 KiB inside the library on every GPU that loads it, kept until
 * the process exits: at most 262,144 floats of query records (sequences x heads x padded
 * dim x padded rows; padded dim is 16/32/64/128, padded rows 1/2/4/8) and 16,384
 * (sequence, head) pairs - larger requests fail with BGTQ_EINVAL - and the split-KV
 * factor is limited to what 3 MiB of partials hold.  All calls share that array and it
 * keeps the last call's contents: calls whose kernels may overlap on the GPU race, so
 * serialise them (one stream per device).  The first call on a device does the set-up
 * (looks up the array's address with cudaGetSymbolAddress and loads the code of every
 * kernel this call can launch); make it before any stream capture starts.  Do not use it
 * on a device across a cudaDeviceReset. */
bgtq_status bgtq_attend_static(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, const float *q,
                               const uint32_t *positions, int causal, uint32_t rows, uint32_t seq_first,
                               uint32_t seq_count, float *out, void *stream);

/* ---- model decode kernels -------------------------------------------------------- */

/* Fused decode-step GEMVs of the model path (the matmul / RMSNorm / SiLU-gate shaders of
 * src/model/kernels.wgsl:11-54 as src/model/decoder.ts:31-81 chains them), for `batch` <= 8
 * activation rows x[b] (FP32, row stride x_stride floats, in % 8 == 0) and FP16 weights w
 * [rows][in] (16-byte aligned), FP32 arithmetic:
 *   mode 0: y[b][r]  = w[r] . rmsnorm(x[b]) + bias[r]      (bias nullable; Q/K/V, lm_head)
 *   mode 1: y[b][r] += w[r] . x[b]                          (residual add; o_proj, down_proj)
 *   mode 2: y[b][r]  = silu(w[r] . n) * (w[out + r] . n)    (n = rmsnorm(x[b]); gate rows then up rows)
 * rmsnorm(v) = v * rsqrt(mean(v^2) + eps) * norm_w.  r < out; y has row stride y_stride
 * floats and must not overlap x.  Stream-ordered. */
bgtq_status bgtq_model_gemv(int mode, const float *x, uint32_t batch, uint64_t x_stride, uint32_t in,
                            const float *norm_w, float eps, const uint16_t *w, const float *bias, uint32_t out,
                            float *y, uint64_t y_stride, void *stream);

/* Persistent decode step of a decoder model (src/model/decoder.ts:31-81 decode: per layer
 * RMSNorm + Q/K/V (+ bias), RoPE + K encode + V append, compressed-K GQA attention, o_proj +
 * residual, RMSNorm + gate/up + SiLU, down_proj + residual; final RMSNorm + lm_head) as ONE
 * cooperative launch with grid-wide barriers between the phases, replacing the seven
 * launches per layer of bgtq_model_gemv / bgtq_append_kv_rope / bgtq_attend.  Same
 * arithmetic as those entry points (the K encode bit for bit).  No counterpart in the
 * reference, whose decoder dispatches one compute pass per shader. */
typedef struct bgtq_decoder bgtq_decoder;
typedef struct {
    uint32_t layers, batch, hidden, q_heads, kv_heads, head_dim, intermediate, vocab;
    float rms_eps;
    const float *inv_freq;               /* host [head_dim / 2]: split-half RoPE table of Q and K */
    const float *const *ln1;             /* [layers] device RMSNorm weights [hidden] */
    const float *const *qkv_bias;        /* [layers] device [(q_heads + 2 kv_heads) head_dim], or null */
    const float *const *ln2;             /* [layers] device [hidden] */
    const uint16_t *const *w_qkv;        /* [layers] FP16 [(q_heads + 2 kv_heads) head_dim][hidden] */
    const uint16_t *const *w_o;          /* [layers] FP16 [hidden][q_heads head_dim] */
    const uint16_t *const *w_gate_up;    /* [layers] FP16 [2 intermediate][hidden]: gate rows, up rows */
    const uint16_t *const *w_down;       /* [layers] FP16 [hidden][intermediate] */
    const float *final_norm;             /* device [hidden] */
    const uint16_t *lm_head;             /* FP16 [vocab][hidden] */
    const float *embedding;              /* FP32 [vocab][hidden] for token-id steps, or null */
    bgtq_attention *const *attention;    /* [layers]: kv_heads packed-key stores + FP16 value stores */
    uint32_t ctas_per_sm;                /* resident CTAs per SM (0: one; at most as many as fit) */
} bgtq_decoder_desc;
/* Requires head_dim 64, gqa = q_heads / kv_heads in 1..8, kv_heads <= 8, batch 1..4,
 * hidden, intermediate and q_heads head_dim multiples of 8, 16-byte aligned weights, and
 * attention objects of kv_heads heads, >= gqa query rows and >= batch sequences.  The step
 * covers sequences 0 .. batch-1.  Errors: BGTQ_EINVAL (shape), BGTQ_ECUDA. */
bgtq_status bgtq_decoder_create(const bgtq_decoder_desc *desc, bgtq_decoder **out);
/* One token per sequence.  tokens: device int64 [batch] token ids (needs the embedding), or
 * null when h already holds the embedded rows.  h: device FP32 [batch][hidden], the residual
 * stream (overwritten); logits: device FP32 [batch][vocab].  Every layer's stores must hold
 * the same length per sequence, below their capacity.  Stream-ordered; moves the stores'
 * lengths on by one.  A barrier wait that runs out sets the device status word
 * (bgtq_device_status) and every later step of the object ends at its first barrier.
 * Steps of one decoder share its barrier words and scratch: issue them in order on one
 * stream, and destroy the decoder only after its last step has finished on the GPU.
 * Errors: BGTQ_EINVAL, BGTQ_EBUSY (lengths), BGTQ_ECAPACITY, BGTQ_ECUDA. */
bgtq_status bgtq_decoder_step(bgtq_decoder *dec, const int64_t *tokens, float *h, float *logits, void *stream);
/* Phase timing: on != 0 makes later steps record CTA 0's global-timer stamps (ns) at the
 * start, after each of the 5 phases of every layer (Q/K/V; append and attention; o_proj;
 * gate/up; down) and at the end (2 + 5 layers stamps).
 * out (nullable, cap entries): the last traced step's stamps, copied synchronously before
 * the switch takes effect; *n_out = the stamp count. */
bgtq_status bgtq_decoder_trace(bgtq_decoder *dec, int on, uint64_t *out, uint32_t cap, uint32_t *n_out);
/* CTAs of the cooperative launch, its dynamic shared memory per CTA, and the bytes of encode
 * tables the append CTAs stage in shared memory (0: read from global memory).  Nullable. */
bgtq_status bgtq_decoder_info(const bgtq_decoder *dec, uint32_t *ctas, uint32_t *smem_bytes, uint32_t *table_bytes);
void bgtq_decoder_destroy(bgtq_decoder *dec);

/* Device status word written by kernels (0 = fine); reading it synchronises. */
bgtq_status bgtq_device_status(int device, uint32_t *status_out);

#ifdef __cplusplus
}
#endif
#endif /* BGTQ_H */
