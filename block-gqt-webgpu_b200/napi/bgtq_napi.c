/*
 * bgtq_napi.c - Node-API addon over libbgtq.so: the drop-in for the reference's WebGPU
 * calls.  The reference's TypeScript classes keep their public surface and call these
 * functions where they used to record WebGPU passes (see napi/index.ts):
 *
 *   validateLayout(config: Uint32Array, table: Float32Array)
 *       -> {dim, groups, rowBytes, normStride, nibbleDims, maxCentroids, ranges: Uint32Array}
 *       layout.ts validateLayout (src/webgpu/layout.ts:8-23) + the PackedKeys group ranges
 *       (src/runtime/packed-keys.ts:15-23)
 *   allocateBits(scores: Float32Array, budget, minBits, maxBits) -> Int32Array
 *       src/reference/allocator.py:4-17
 *   buildTables(widths: Int32Array, rotationThreshold, rowPad, normStride)
 *       -> {config: Uint32Array, table: Float32Array}   (the calibration's table build)
 *   packedKeysCreate(config, table, capacity, sequences, device) -> handle
 *       PackedKeys.create (packed-keys.ts:32-38)
 *   fp16KeysCreate(dim, capacity, sequences, device) -> handle      FP16Keys (keys.ts:16-27)
 *   valuesCreate(f32: boolean, dim, capacity, sequences, device) -> handle   Values (values.ts:3-8)
 *   keysAppend(keys, rows: Uint16Array | Float32Array, seqFirst)   PackedKeys/FP16Keys.append
 *   valuesAppend(values, rows: Uint16Array | Float32Array, seqFirst)   Values.append (values.ts:9-14)
 *   keysLength(keys, seq) / valuesLength(values, seq) -> number
 *   keysRead(keys, seq) -> {packed: Uint8Array, scales: Uint16Array}   (the packed/norms buffers)
 *   attentionCreate(keys: handle[], values: handle[], rows) -> handle
 *       OptimizedAttention.create / AttentionEngine.session (optimized.ts:20-28, attention.ts:16)
 *   attend(att, q: Float32Array, positions: Uint32Array | null, causal, rows, out: Float32Array,
 *          logits?: Float32Array, probs?: Float32Array)
 *       setQueries + attend / record + inspect (optimized.ts:29-43)
 *   attendPrefill(att, q: Float32Array, posFirst, n, gqa, out: Float32Array)
 *       the model's chunked prefill (src/model/decoder.ts:52-56)
 *   destroy(handle)   the objects' destroy() (packed-keys.ts:51); handles are also freed
 *       when garbage-collected
 *   deviceStatus(device) -> number
 *
 * Every call is synchronous and takes host typed arrays (the reference's Uint16Array /
 * Float32Array arguments); the library copies them in and, for attention, out again.  A
 * failing call throws what the reference throws: RangeError for shapes, capacity,
 * non-finite input and layouts (keys.ts:12-14, layout.ts:13-22, optimized.ts:30), Error
 * otherwise (packed-keys.ts:50), with the library's message.
 *
 * Build with node-gyp (napi/binding.gyp) against include/bgtq.h and libbgtq.so.
 */
#include <stdbool.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <node_api.h>

#include "bgtq.h"

enum { H_KEYS = 1, H_VALUES = 2, H_ATTENTION = 3 };
#define MAX_ARGS 8

/* A JS handle: the library object and its kind; freed by destroy() or the finalizer. */
typedef struct handle {
    int kind;
    void *obj;
} handle;

static void free_obj(handle *h) {
    if (!h || !h->obj) return;
    if (h->kind == H_KEYS) bgtq_keys_destroy((bgtq_keys *)h->obj);
    else if (h->kind == H_VALUES) bgtq_values_destroy((bgtq_values *)h->obj);
    else if (h->kind == H_ATTENTION) bgtq_attention_destroy((bgtq_attention *)h->obj);
    h->obj = NULL;
}

static void finalize_handle(napi_env env, void *data, void *hint) {
    (void)env;
    (void)hint;
    handle *h = (handle *)data;
    free_obj(h);
    free(h);
}

static napi_value throw_status(napi_env env, bgtq_status s) {
    const char *msg = bgtq_last_error();
    if (!msg || !*msg) msg = bgtq_status_string(s);
    if (s == BGTQ_EINVAL || s == BGTQ_ECAPACITY || s == BGTQ_ENONFINITE || s == BGTQ_ELAYOUT)
        napi_throw_range_error(env, NULL, msg);
    else
        napi_throw_error(env, NULL, msg);
    return NULL;
}

static napi_value throw_range(napi_env env, const char *msg) {
    napi_throw_range_error(env, NULL, msg);
    return NULL;
}

typedef struct args {
    size_t n;
    napi_value v[MAX_ARGS];
} args;

static bool get_args(napi_env env, napi_callback_info info, args *a) {
    a->n = MAX_ARGS;
    return napi_get_cb_info(env, info, &a->n, a->v, NULL, NULL) == napi_ok;
}

/* Optional trailing arguments: absent, undefined and null all mean "not given". */
static bool given(napi_env env, const args *a, size_t i) {
    napi_valuetype t;
    if (i >= a->n || napi_typeof(env, a->v[i], &t) != napi_ok) return false;
    return t != napi_undefined && t != napi_null;
}

static bool u32_arg(napi_env env, const args *a, size_t i, uint32_t dflt, uint32_t *out) {
    if (!given(env, a, i)) {
        *out = dflt;
        return true;
    }
    return napi_get_value_uint32(env, a->v[i], out) == napi_ok;
}

/* A typed array of the wanted element type (data, element count). */
static bool typed(napi_env env, napi_value v, napi_typedarray_type want, void **data, size_t *len) {
    bool is = false;
    napi_typedarray_type t;
    if (napi_is_typedarray(env, v, &is) != napi_ok || !is) return false;
    if (napi_get_typedarray_info(env, v, &t, len, data, NULL, NULL) != napi_ok) return false;
    return t == want;
}

static handle *handle_arg(napi_env env, napi_value v, int kind) {
    void *p = NULL;
    if (napi_get_value_external(env, v, &p) != napi_ok || !p) return NULL;
    handle *h = (handle *)p;
    return h->kind == kind && h->obj ? h : NULL;
}

static napi_value wrap(napi_env env, int kind, void *obj) {
    handle *h = (handle *)malloc(sizeof(handle));
    napi_value out = NULL;
    if (!h) {
        napi_throw_error(env, NULL, "out of host memory");
        return NULL;
    }
    h->kind = kind;
    h->obj = obj;
    if (napi_create_external(env, h, finalize_handle, NULL, &out) != napi_ok) {
        free_obj(h);
        free(h);
        napi_throw_error(env, NULL, "cannot create handle");
        return NULL;
    }
    return out;
}

static napi_value new_typed(napi_env env, napi_typedarray_type t, size_t elem, size_t n, void **data) {
    napi_value ab, out;
    if (napi_create_arraybuffer(env, elem * n, data, &ab) != napi_ok) return NULL;
    if (napi_create_typedarray(env, t, n, ab, 0, &out) != napi_ok) return NULL;
    return out;
}

static void set_u32(napi_env env, napi_value obj, const char *name, uint32_t v) {
    napi_value x;
    napi_create_uint32(env, v, &x);
    napi_set_named_property(env, obj, name, x);
}

/* ---- host-only: layout, allocator, tables ---- */

static napi_value validate_layout(napi_env env, napi_callback_info info) {
    args a;
    void *cfg, *tab;
    size_t nc, nt;
    if (!get_args(env, info, &a) || a.n < 2 || !typed(env, a.v[0], napi_uint32_array, &cfg, &nc) ||
        !typed(env, a.v[1], napi_float32_array, &tab, &nt))
        return throw_range(env, "validateLayout(config: Uint32Array, table: Float32Array)");
    bgtq_layout_info li;
    uint32_t *ranges = (uint32_t *)calloc(2 * 128, sizeof(uint32_t));
    if (!ranges) return throw_range(env, "out of host memory");
    bgtq_status s = bgtq_layout_validate((const uint32_t *)cfg, nc, (const float *)tab, nt, ranges, &li);
    if (s) {
        free(ranges);
        return throw_status(env, s);
    }
    napi_value out, r;
    void *rd;
    napi_create_object(env, &out);
    set_u32(env, out, "dim", li.dim);
    set_u32(env, out, "groups", li.groups);
    set_u32(env, out, "rowBytes", li.row_bytes);
    set_u32(env, out, "normStride", li.norm_stride);
    set_u32(env, out, "nibbleDims", li.nibble_dims);
    set_u32(env, out, "maxCentroids", li.max_centroids);
    r = new_typed(env, napi_uint32_array, 4, 2 * (size_t)li.dim, &rd);
    if (r) {
        memcpy(rd, ranges, 8 * (size_t)li.dim);
        napi_set_named_property(env, out, "ranges", r);
    }
    free(ranges);
    return out;
}

static napi_value allocate_bits(napi_env env, napi_callback_info info) {
    args a;
    void *sc;
    size_t n;
    uint32_t budget, lo, hi;
    if (!get_args(env, info, &a) || a.n < 4 || !typed(env, a.v[0], napi_float32_array, &sc, &n) ||
        !u32_arg(env, &a, 1, 0, &budget) || !u32_arg(env, &a, 2, 1, &lo) || !u32_arg(env, &a, 3, 8, &hi))
        return throw_range(env, "allocateBits(scores: Float32Array, budget, minBits, maxBits)");
    int64_t *w = (int64_t *)calloc(n ? n : 1, sizeof(int64_t));
    if (!w) return throw_range(env, "out of host memory");
    bgtq_status s = bgtq_allocate_bits((const float *)sc, (uint32_t)n, budget, (int32_t)lo, (int32_t)hi, w);
    if (s) {
        free(w);
        return throw_status(env, s);
    }
    void *od;
    napi_value out = new_typed(env, napi_int32_array, 4, n, &od);
    for (size_t i = 0; out && i < n; ++i) ((int32_t *)od)[i] = (int32_t)w[i];
    free(w);
    return out;
}

static napi_value build_tables(napi_env env, napi_callback_info info) {
    args a;
    void *wd;
    size_t n;
    uint32_t thr, pad, ns;
    if (!get_args(env, info, &a) || a.n < 1 || !typed(env, a.v[0], napi_int32_array, &wd, &n) ||
        !u32_arg(env, &a, 1, 3, &thr) || !u32_arg(env, &a, 2, 0, &pad) || !u32_arg(env, &a, 3, 0, &ns))
        return throw_range(env, "buildTables(widths: Int32Array, rotationThreshold, rowPad, normStride)");
    int64_t *w = (int64_t *)calloc(n ? n : 1, sizeof(int64_t));
    if (!w) return throw_range(env, "out of host memory");
    for (size_t i = 0; i < n; ++i) w[i] = ((const int32_t *)wd)[i];
    size_t nc = 0, nt = 0;
    bgtq_status s = bgtq_tables_build((uint32_t)(2 * n), w, NULL, thr, pad, ns, NULL, 0, &nc, NULL, 0, &nt);
    void *cd = NULL, *td = NULL;
    napi_value cfg = NULL, tab = NULL, out = NULL;
    if (!s) {
        cfg = new_typed(env, napi_uint32_array, 4, nc, &cd);
        tab = new_typed(env, napi_float32_array, 4, nt, &td);
        if (!cfg || !tab) s = BGTQ_ENOMEM;
    }
    if (!s) s = bgtq_tables_build((uint32_t)(2 * n), w, NULL, thr, pad, ns, (uint32_t *)cd, nc, &nc, (float *)td, nt, &nt);
    free(w);
    if (s) return throw_status(env, s);
    napi_create_object(env, &out);
    napi_set_named_property(env, out, "config", cfg);
    napi_set_named_property(env, out, "table", tab);
    return out;
}

/* ---- stores ---- */

static napi_value packed_keys_create(napi_env env, napi_callback_info info) {
    args a;
    void *cfg, *tab;
    size_t nc, nt;
    uint32_t cap, seqs, dev;
    if (!get_args(env, info, &a) || a.n < 3 || !typed(env, a.v[0], napi_uint32_array, &cfg, &nc) ||
        !typed(env, a.v[1], napi_float32_array, &tab, &nt) || !u32_arg(env, &a, 2, 0, &cap) ||
        !u32_arg(env, &a, 3, 1, &seqs) || !u32_arg(env, &a, 4, 0, &dev))
        return throw_range(env, "packedKeysCreate(config, table, capacity, sequences, device)");
    bgtq_tables *t = NULL;
    bgtq_keys *k = NULL;
    bgtq_status s = bgtq_tables_create((const uint32_t *)cfg, nc, (const float *)tab, nt, (int)dev, &t);
    if (s) return throw_status(env, s);
    s = bgtq_keys_create(BGTQ_KEYS_PACKED, t, 0, cap, seqs, (int)dev, &k);
    bgtq_tables_destroy(t);
    if (s) return throw_status(env, s);
    return wrap(env, H_KEYS, k);
}

static napi_value fp16_keys_create(napi_env env, napi_callback_info info) {
    args a;
    uint32_t dim, cap, seqs, dev;
    if (!get_args(env, info, &a) || a.n < 2 || !u32_arg(env, &a, 0, 0, &dim) || !u32_arg(env, &a, 1, 0, &cap) ||
        !u32_arg(env, &a, 2, 1, &seqs) || !u32_arg(env, &a, 3, 0, &dev))
        return throw_range(env, "fp16KeysCreate(dim, capacity, sequences, device)");
    bgtq_keys *k = NULL;
    bgtq_status s = bgtq_keys_create(BGTQ_KEYS_FP16, NULL, dim, cap, seqs, (int)dev, &k);
    return s ? throw_status(env, s) : wrap(env, H_KEYS, k);
}

static napi_value values_create(napi_env env, napi_callback_info info) {
    args a;
    bool f32 = true;
    uint32_t dim, cap, seqs, dev;
    if (!get_args(env, info, &a) || a.n < 3 || napi_get_value_bool(env, a.v[0], &f32) != napi_ok ||
        !u32_arg(env, &a, 1, 0, &dim) || !u32_arg(env, &a, 2, 0, &cap) || !u32_arg(env, &a, 3, 1, &seqs) ||
        !u32_arg(env, &a, 4, 0, &dev))
        return throw_range(env, "valuesCreate(f32, dim, capacity, sequences, device)");
    bgtq_values *v = NULL;
    bgtq_status s = bgtq_values_create(f32 ? BGTQ_F32 : BGTQ_F16, dim, cap, seqs, (int)dev, &v);
    return s ? throw_status(env, s) : wrap(env, H_VALUES, v);
}

/* rows: Uint16Array (FP16 bits) or Float32Array, whole rows of `dim` for one sequence */
static bool rows_arg(napi_env env, napi_value v, void **data, size_t *n, bgtq_dtype *dt) {
    if (typed(env, v, napi_uint16_array, data, n)) {
        *dt = BGTQ_F16;
        return true;
    }
    if (typed(env, v, napi_float32_array, data, n)) {
        *dt = BGTQ_F32;
        return true;
    }
    return false;
}

static napi_value keys_append(napi_env env, napi_callback_info info) {
    args a;
    void *rows;
    size_t n;
    bgtq_dtype dt;
    uint32_t seq;
    handle *h;
    if (!get_args(env, info, &a) || a.n < 2 || !(h = handle_arg(env, a.v[0], H_KEYS)) ||
        !rows_arg(env, a.v[1], &rows, &n, &dt) || !u32_arg(env, &a, 2, 0, &seq))
        return throw_range(env, "keysAppend(keys, rows: Uint16Array | Float32Array, seqFirst)");
    uint32_t dim = 0;
    bgtq_keys_info((bgtq_keys *)h->obj, NULL, &dim, NULL, NULL);
    if (!n || !dim || n % dim) return throw_range(env, "K append must contain whole nonempty rows");
    bgtq_status s = bgtq_keys_append((bgtq_keys *)h->obj, rows, dt, 1, (uint32_t)(n / dim), dim, seq, 1, n, NULL);
    return s ? throw_status(env, s) : NULL;
}

static napi_value values_append(napi_env env, napi_callback_info info) {
    args a;
    void *rows;
    size_t n;
    bgtq_dtype dt;
    uint32_t seq, dim = 0;
    handle *h;
    if (!get_args(env, info, &a) || a.n < 2 || !(h = handle_arg(env, a.v[0], H_VALUES)) ||
        !rows_arg(env, a.v[1], &rows, &n, &dt) || !u32_arg(env, &a, 2, 0, &seq))
        return throw_range(env, "valuesAppend(values, rows: Uint16Array | Float32Array, seqFirst)");
    bgtq_values_info((bgtq_values *)h->obj, NULL, &dim, NULL, NULL);
    if (!n || !dim || n % dim) return throw_range(env, "V append must contain whole nonempty rows");
    bgtq_status s = bgtq_values_append((bgtq_values *)h->obj, rows, dt, 1, (uint32_t)(n / dim), dim, seq, 1, n, NULL);
    return s ? throw_status(env, s) : NULL;
}

static napi_value store_length(napi_env env, napi_callback_info info, int kind) {
    args a;
    uint32_t seq, len = 0;
    handle *h;
    if (!get_args(env, info, &a) || a.n < 1 || !(h = handle_arg(env, a.v[0], kind)) || !u32_arg(env, &a, 1, 0, &seq))
        return throw_range(env, "length(store, seq)");
    bgtq_status s = kind == H_KEYS ? bgtq_keys_length((bgtq_keys *)h->obj, seq, &len)
                                   : bgtq_values_length((bgtq_values *)h->obj, seq, &len);
    if (s) return throw_status(env, s);
    napi_value out;
    napi_create_uint32(env, len, &out);
    return out;
}
static napi_value keys_length(napi_env env, napi_callback_info info) { return store_length(env, info, H_KEYS); }
static napi_value values_length(napi_env env, napi_callback_info info) { return store_length(env, info, H_VALUES); }

/* the packed rows (config rowBytes each) and FP16 scale bits (normStride each) of a sequence,
   as the reference's packed / norms buffers hold them */
static napi_value keys_read(napi_env env, napi_callback_info info) {
    args a;
    uint32_t seq, len = 0;
    handle *h;
    if (!get_args(env, info, &a) || a.n < 1 || !(h = handle_arg(env, a.v[0], H_KEYS)) || !u32_arg(env, &a, 1, 0, &seq))
        return throw_range(env, "keysRead(keys, seq)");
    bgtq_keys *k = (bgtq_keys *)h->obj;
    bgtq_keys_kind kind;
    uint32_t dim;
    bgtq_status s = bgtq_keys_length(k, seq, &len);
    if (!s) s = bgtq_keys_info(k, &kind, &dim, NULL, NULL);
    if (s) return throw_status(env, s);
    if (kind == BGTQ_KEYS_FP16) {
        void *d;
        napi_value rows = new_typed(env, napi_uint16_array, 2, (size_t)len * dim, &d);
        s = rows ? bgtq_keys_read(k, seq, 0, len, (uint8_t *)d, NULL) : BGTQ_ENOMEM;
        return s ? throw_status(env, s) : rows;
    }
    bgtq_layout_info li;
    memset(&li, 0, sizeof li);
    s = bgtq_keys_layout(k, &li);
    if (s) return throw_status(env, s);
    void *pd, *sd;
    napi_value packed = new_typed(env, napi_uint8_array, 1, (size_t)len * li.row_bytes, &pd);
    napi_value scales = new_typed(env, napi_uint16_array, 2, (size_t)len * li.norm_stride, &sd);
    s = packed && scales ? bgtq_keys_read(k, seq, 0, len, (uint8_t *)pd, (uint16_t *)sd) : BGTQ_ENOMEM;
    if (s) return throw_status(env, s);
    napi_value out;
    napi_create_object(env, &out);
    napi_set_named_property(env, out, "packed", packed);
    napi_set_named_property(env, out, "scales", scales);
    return out;
}

/* ---- attention ---- */

static napi_value attention_create(napi_env env, napi_callback_info info) {
    args a;
    uint32_t nk = 0, nv = 0, rows;
    if (!get_args(env, info, &a) || a.n < 3 || napi_get_array_length(env, a.v[0], &nk) != napi_ok ||
        napi_get_array_length(env, a.v[1], &nv) != napi_ok || nk != nv || nk < 1 || nk > 8 ||
        !u32_arg(env, &a, 2, 0, &rows))
        return throw_range(env, "attentionCreate(keys: handle[], values: handle[], rows)");
    bgtq_keys *ks[8];
    bgtq_values *vs[8];
    for (uint32_t i = 0; i < nk; ++i) {
        napi_value ek, ev;
        handle *hk, *hv;
        if (napi_get_element(env, a.v[0], i, &ek) != napi_ok || napi_get_element(env, a.v[1], i, &ev) != napi_ok ||
            !(hk = handle_arg(env, ek, H_KEYS)) || !(hv = handle_arg(env, ev, H_VALUES)))
            return throw_range(env, "Incompatible attention storage");
        ks[i] = (bgtq_keys *)hk->obj;
        vs[i] = (bgtq_values *)hv->obj;
    }
    bgtq_attention *att = NULL;
    bgtq_status s = bgtq_attention_create(nk, ks, vs, rows, &att);
    return s ? throw_status(env, s) : wrap(env, H_ATTENTION, att);
}

/* q [heads][rows][dim] of sequence 0 (the reference's one-sequence session), positions
   [rows] or null (last token), out [heads][rows][dim]; logits / probs [heads][rows][length]
   when inspecting */
static napi_value attend(napi_env env, napi_callback_info info) {
    args a;
    handle *h;
    void *q, *pos = NULL, *out, *lg = NULL, *pr = NULL;
    size_t nq, npos = 0, nout, nl = 0, np = 0;
    bool causal = false;
    uint32_t rows;
    if (!get_args(env, info, &a) || a.n < 6 || !(h = handle_arg(env, a.v[0], H_ATTENTION)) ||
        !typed(env, a.v[1], napi_float32_array, &q, &nq) ||
        (given(env, &a, 2) && !typed(env, a.v[2], napi_uint32_array, &pos, &npos)) ||
        napi_get_value_bool(env, a.v[3], &causal) != napi_ok || !u32_arg(env, &a, 4, 0, &rows) ||
        !typed(env, a.v[5], napi_float32_array, &out, &nout) ||
        (given(env, &a, 6) && !typed(env, a.v[6], napi_float32_array, &lg, &nl)) ||
        (given(env, &a, 7) && !typed(env, a.v[7], napi_float32_array, &pr, &np)))
        return throw_range(env, "attend(att, q, positions, causal, rows, out, logits?, probs?)");
    if (nq != nout || (pos && npos != rows) || (pr && !lg))
        return throw_range(env, "Invalid Q/K/V shape or positions");
    bgtq_status s = bgtq_attend((bgtq_attention *)h->obj, (const float *)q, (const uint32_t *)pos, causal ? 1 : 0, rows,
                                0, 1, (float *)out, (float *)lg, (float *)pr, 1, NULL);
    return s ? throw_status(env, s) : NULL;
}

/* q / out [n][heads * gqa][dim] of sequence 0, positions posFirst .. posFirst + n - 1 */
static napi_value attend_prefill(napi_env env, napi_callback_info info) {
    args a;
    handle *h;
    void *q, *out;
    size_t nq, nout;
    uint32_t pos0, n, gqa;
    if (!get_args(env, info, &a) || a.n < 6 || !(h = handle_arg(env, a.v[0], H_ATTENTION)) ||
        !typed(env, a.v[1], napi_float32_array, &q, &nq) || !u32_arg(env, &a, 2, 0, &pos0) ||
        !u32_arg(env, &a, 3, 0, &n) || !u32_arg(env, &a, 4, 0, &gqa) ||
        !typed(env, a.v[5], napi_float32_array, &out, &nout) || nq != nout)
        return throw_range(env, "attendPrefill(att, q, posFirst, n, gqa, out)");
    bgtq_status s = bgtq_attend_prefill((bgtq_attention *)h->obj, (const float *)q, pos0, n, gqa, 0, 1, (float *)out, 1,
                                        NULL);
    return s ? throw_status(env, s) : NULL;
}

static napi_value destroy(napi_env env, napi_callback_info info) {
    args a;
    void *p = NULL;
    if (get_args(env, info, &a) && a.n >= 1 && napi_get_value_external(env, a.v[0], &p) == napi_ok && p)
        free_obj((handle *)p);  /* the handle itself goes with the JS object */
    return NULL;
}

static napi_value device_status(napi_env env, napi_callback_info info) {
    args a;
    uint32_t dev, st = 0;
    if (!get_args(env, info, &a) || !u32_arg(env, &a, 0, 0, &dev)) return throw_range(env, "deviceStatus(device)");
    bgtq_status s = bgtq_device_status((int)dev, &st);
    if (s) return throw_status(env, s);
    napi_value out;
    napi_create_uint32(env, st, &out);
    return out;
}

/* ---- module ---- */

napi_value bgtq_napi_init(napi_env env, napi_value exports) {
    static const struct {
        const char *name;
        napi_callback fn;
    } fns[] = {{"validateLayout", validate_layout}, {"allocateBits", allocate_bits},
               {"buildTables", build_tables},       {"packedKeysCreate", packed_keys_create},
               {"fp16KeysCreate", fp16_keys_create}, {"valuesCreate", values_create},
               {"keysAppend", keys_append},         {"valuesAppend", values_append},
               {"keysLength", keys_length},         {"valuesLength", values_length},
               {"keysRead", keys_read},             {"attentionCreate", attention_create},
               {"attend", attend},                  {"attendPrefill", attend_prefill},
               {"destroy", destroy},                {"deviceStatus", device_status}};
    for (size_t i = 0; i < sizeof fns / sizeof fns[0]; ++i) {
        napi_value f;
        if (napi_create_function(env, fns[i].name, NAPI_AUTO_LENGTH, fns[i].fn, NULL, &f) != napi_ok ||
            napi_set_named_property(env, exports, fns[i].name, f) != napi_ok)
            return NULL;
    }
    return exports;
}

#ifdef NAPI_MODULE_INIT
NAPI_MODULE_INIT() { return bgtq_napi_init(env, exports); }
#endif
