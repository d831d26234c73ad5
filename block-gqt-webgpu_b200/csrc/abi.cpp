// C ABI of libbgtq.so: object lifetimes, validation (before any state change, as the
// reference's RangeError/Error checks are), host<->device staging and kernel launches.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "objects.h"

using namespace bgtq;

namespace {

thread_local std::string g_err;

bgtq_status fail(bgtq_status s, const std::string &msg) {
    g_err = msg;
    return s;
}
bgtq_status cuda_fail(cudaError_t e, const char *where) {
    g_err = std::string(where) + ": " + cudaGetErrorString(e);
    return BGTQ_ECUDA;
}
#define CK(expr, where)                                   \
    do {                                                  \
        cudaError_t e_ = (expr);                          \
        if (e_ != cudaSuccess) return cuda_fail(e_, where); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

uint32_t dim_template(uint32_t d) { return d <= 16 ? 16u : d <= 32 ? 32u : d <= 64 ? 64u : 128u; }
uint32_t round_up(uint32_t x, uint32_t m) { return (x + m - 1) / m * m; }

std::mutex g_status_mu;
uint32_t *g_status[64] = {};

}  // namespace

namespace bgtq {
void set_last_error(const std::string &message) { g_err = message; }

uint32_t *device_status_word_if_present(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_status_mu);
    return g_status[device];
}

uint32_t *device_status_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (!g_status[device]) {
        void *p = nullptr;
        if (cudaMalloc(&p, sizeof(uint32_t)) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, sizeof(uint32_t));
        g_status[device] = static_cast<uint32_t *>(p);
    }
    return g_status[device];
}
}  // namespace bgtq

namespace {

cudaError_t upload_tables(const Layout &L, DeviceTables &dt) {
    const size_t n_rot = (size_t)L.d * L.d, n_cent = L.cent_compact.size();
    auto a16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
    size_t off = 0;
    const size_t o_rot = off; off = a16(off + 4 * n_rot);
    const size_t o_cent = off; off = a16(off + 4 * (n_cent ? n_cent : 1));
    const size_t o_off = off; off = a16(off + 4 * L.d);
    const size_t o_inv = off; off = a16(off + 4 * L.d);
    const size_t o_lut = off; off = a16(off + L.lut.size());
    const size_t o_perm = off; off = a16(off + L.d);
    const size_t o_grp = off; off = a16(off + L.d);
    const size_t o_cbi = off; off = a16(off + L.d);
    const size_t o_cbb = off; off = a16(off + 2 * L.d);
    const size_t o_lk = off; off = a16(off + 4 * L.lookup.size());
    const size_t o_lko = off; off = a16(off + 2 * L.d);
    std::vector<unsigned char> host(off, 0);
    std::memcpy(host.data() + o_rot, L.rot.data(), 4 * n_rot);
    if (n_cent) std::memcpy(host.data() + o_cent, L.cent_compact.data(), 4 * n_cent);
    std::memcpy(host.data() + o_off, L.off.data(), 4 * L.d);
    std::memcpy(host.data() + o_inv, L.inv.data(), 4 * L.d);
    std::memcpy(host.data() + o_lut, L.lut.data(), L.lut.size());
    std::memcpy(host.data() + o_perm, L.perm.data(), L.d);
    std::memcpy(host.data() + o_grp, L.group_of.data(), L.d);
    std::memcpy(host.data() + o_cbi, L.pos_to_cb.data(), L.d);
    std::memcpy(host.data() + o_cbb, L.cb_base.data(), 2 * L.d);
    std::memcpy(host.data() + o_lk, L.lookup.data(), 4 * L.lookup.size());
    std::memcpy(host.data() + o_lko, L.lookup_off.data(), 2 * L.d);
    void *blob = nullptr;
    cudaError_t e = cudaMalloc(&blob, off);
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(blob, host.data(), off, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(blob);
        return e;
    }
    unsigned char *b = static_cast<unsigned char *>(blob);
    dt.blob = blob;
    dt.bytes = off;
    dt.rot = reinterpret_cast<const float *>(b + o_rot);
    dt.cent = reinterpret_cast<const float *>(b + o_cent);
    dt.off = reinterpret_cast<const float *>(b + o_off);
    dt.inv = reinterpret_cast<const float *>(b + o_inv);
    dt.lut = b + o_lut;
    dt.perm = b + o_perm;
    dt.group_of = b + o_grp;
    dt.cbidx = b + o_cbi;
    dt.cb_base = reinterpret_cast<const uint16_t *>(b + o_cbb);
    dt.lookup = reinterpret_cast<const float *>(b + o_lk);
    dt.lookup_off = reinterpret_cast<const uint16_t *>(b + o_lko);
    return cudaSuccess;
}

// Branch-free per row (the exponent field all ones marks Inf / NaN), so the compiler
// vectorises it: host appends are checked on every call.
bool host_finite(const void *src, bgtq_dtype dt, uint32_t dim, uint32_t count, uint64_t row_stride, uint32_t seq_count,
                 uint64_t seq_stride) {
    for (uint32_t s = 0; s < seq_count; ++s)
        for (uint32_t r = 0; r < count; ++r) {
            const uint64_t base = s * seq_stride + r * row_stride;
            uint32_t bad = 0;
            if (dt == BGTQ_F16) {
                const uint16_t *p = static_cast<const uint16_t *>(src) + base;
                for (uint32_t i = 0; i < dim; ++i) bad |= (uint32_t)((p[i] & 0x7c00u) == 0x7c00u);
            } else {
                const uint32_t *p = static_cast<const uint32_t *>(src) + base;
                for (uint32_t i = 0; i < dim; ++i) bad |= (uint32_t)((p[i] & 0x7f800000u) == 0x7f800000u);
            }
            if (bad) return false;
        }
    return true;
}

// Common validation + host staging of an append source.  On success `dsrc`,
// `drow`, `dseq` describe a device-resident source.
bgtq_status stage_source(const void *src, bgtq_dtype dtype, int host, uint32_t dim, uint32_t count, uint64_t row_stride,
                         uint32_t seq_count, uint64_t seq_stride, DevBuf &staging, cudaStream_t stream,
                         const void **dsrc, uint64_t *drow, uint64_t *dseq) {
    const size_t es = dtype == BGTQ_F16 ? 2 : 4;
    if (host) {
        if (!host_finite(src, dtype, dim, count, row_stride, seq_count, seq_stride))
            return fail(BGTQ_ENONFINITE, dtype == BGTQ_F16 ? "Finite FP16 K required" : "finite inputs required");
        const size_t bytes = (size_t)seq_count * count * dim * es;
        CK(staging.ensure(bytes), "staging allocation");
        if (row_stride == dim && (seq_count == 1 || seq_stride == (uint64_t)count * dim)) {
            CK(cudaMemcpyAsync(staging.p, src, bytes, cudaMemcpyHostToDevice, stream), "append upload");
        } else {
            for (uint32_t s = 0; s < seq_count; ++s)
                CK(cudaMemcpy2DAsync(static_cast<unsigned char *>(staging.p) + (size_t)s * count * dim * es, dim * es,
                                     static_cast<const unsigned char *>(src) + s * seq_stride * es, row_stride * es,
                                     dim * es, count, cudaMemcpyHostToDevice, stream),
                   "append upload");
        }
        *dsrc = staging.p;
        *drow = dim;
        *dseq = (uint64_t)count * dim;
    } else {
        *dsrc = src;
        *drow = row_stride;
        *dseq = seq_stride;
    }
    return BGTQ_OK;
}

// Start row of every target sequence: scalar when all equal, else a device vector.
bgtq_status start_rows(const std::vector<uint32_t> &lengths, uint32_t seq_first, uint32_t seq_count, DevBuf &buf,
                       cudaStream_t stream, const uint32_t **dev, uint32_t *scalar, std::vector<uint32_t> &tmp) {
    bool uniform = true;
    for (uint32_t s = 1; s < seq_count; ++s) uniform &= lengths[seq_first + s] == lengths[seq_first];
    *scalar = lengths[seq_first];
    *dev = nullptr;
    if (!uniform) {
        tmp.assign(lengths.begin() + seq_first, lengths.begin() + seq_first + seq_count);
        CK(buf.ensure(sizeof(uint32_t) * seq_count), "row0 allocation");
        CK(cudaMemcpyAsync(buf.p, tmp.data(), sizeof(uint32_t) * seq_count, cudaMemcpyHostToDevice, stream),
           "row0 upload");
        *dev = static_cast<const uint32_t *>(buf.p);
    }
    return BGTQ_OK;
}

bgtq_status check_append(uint32_t dim, uint32_t capacity, uint32_t sequences, const std::vector<uint32_t> &lengths,
                         const void *src, bgtq_dtype dtype, uint32_t count, uint64_t row_stride, uint32_t seq_first,
                         uint32_t seq_count, const char *what) {
    if (!src || dtype < BGTQ_F16 || dtype > BGTQ_F32) return fail(BGTQ_EINVAL, std::string(what) + ": invalid source");
    if (!count || !seq_count || row_stride < dim)
        return fail(BGTQ_EINVAL, std::string(what) + " append must contain whole nonempty rows");
    if ((uint64_t)seq_first + seq_count > sequences) return fail(BGTQ_EINVAL, std::string(what) + ": sequence range");
    for (uint32_t s = 0; s < seq_count; ++s)
        if ((uint64_t)lengths[seq_first + s] + count > capacity)
            return fail(BGTQ_ECAPACITY, std::string(what) + " capacity exceeded");
    return BGTQ_OK;
}

}  // namespace

extern "C" {

const char *bgtq_status_string(bgtq_status s) {
    switch (s) {
        case BGTQ_OK: return "ok";
        case BGTQ_EINVAL: return "invalid argument";
        case BGTQ_ECAPACITY: return "capacity exceeded";
        case BGTQ_ENONFINITE: return "non-finite input";
        case BGTQ_EBUSY: return "storage not ready";
        case BGTQ_ELAYOUT: return "invalid layout";
        case BGTQ_ETIMEOUT: return "device wait timed out";
        case BGTQ_ECUDA: return "CUDA error";
        case BGTQ_ENOMEM: return "out of memory";
        default: return "unknown status";
    }
}
const char *bgtq_last_error(void) { return g_err.c_str(); }
const char *bgtq_version(void) { return "bgtq-b200 0.1 (sm_100a)"; }

bgtq_status bgtq_layout_validate(const uint32_t *config, size_t n_config, const float *table, size_t n_table,
                                 uint32_t *ranges_out, bgtq_layout_info *info) {
    Layout L;
    std::string err;
    bgtq_status s = parse_layout(config, n_config, table, n_table, L, err);
    if (s != BGTQ_OK) return fail(s, err);
    if (ranges_out) std::copy(L.ranges.begin(), L.ranges.end(), ranges_out);
    if (info) {
        info->dim = L.d; info->groups = L.ng; info->row_bytes = L.row_bytes; info->norm_stride = L.norm_stride;
        info->nibble_dims = L.ns; info->max_centroids = L.maxc; info->logical_row_bytes = L.logical_rb;
        info->device_row_stride = L.dev_row_stride; info->device_scale_stride = L.dev_scale_stride;
        info->codebooks = L.ncb;
    }
    return BGTQ_OK;
}

bgtq_status bgtq_tables_create(const uint32_t *config, size_t n_config, const float *table, size_t n_table, int device,
                               bgtq_tables **out) {
    if (!out) return fail(BGTQ_EINVAL, "null output");
    auto *t = new bgtq_tables();
    std::string err;
    bgtq_status s = parse_layout(config, n_config, table, n_table, t->L, err);
    if (s != BGTQ_OK) {
        delete t;
        return fail(s, err);
    }
    DeviceGuard g(device);
    if (!g.ok) {
        delete t;
        return fail(BGTQ_ECUDA, "cannot select device");
    }
    t->device = device;
    cudaError_t e = upload_tables(t->L, t->dt);
    if (e != cudaSuccess) {
        delete t;
        return cuda_fail(e, "tables upload");
    }
    *out = t;
    return BGTQ_OK;
}

bgtq_status bgtq_tables_info(const bgtq_tables *t, bgtq_layout_info *info) {
    if (!t || !info) return fail(BGTQ_EINVAL, "null argument");
    const Layout &L = t->L;
    info->dim = L.d; info->groups = L.ng; info->row_bytes = L.row_bytes; info->norm_stride = L.norm_stride;
    info->nibble_dims = L.ns; info->max_centroids = L.maxc; info->logical_row_bytes = L.logical_rb;
    info->device_row_stride = L.dev_row_stride; info->device_scale_stride = L.dev_scale_stride;
    info->codebooks = L.ncb;
    return BGTQ_OK;
}

void bgtq_tables_destroy(bgtq_tables *t) {
    if (!t) return;
    DeviceGuard g(t->device);
    if (t->dt.blob) cudaFree(t->dt.blob);
    delete t;
}

bgtq_status bgtq_keys_create(bgtq_keys_kind kind, const bgtq_tables *tables, uint32_t dim, uint32_t capacity,
                             uint32_t sequences, int device, bgtq_keys **out) {
    if (!out) return fail(BGTQ_EINVAL, "null output");
    if (kind != BGTQ_KEYS_PACKED && kind != BGTQ_KEYS_FP16 && kind != BGTQ_KEYS_COMPRESSED)
        return fail(BGTQ_EINVAL, "Invalid K kind");
    if (kind != BGTQ_KEYS_FP16 && !tables) return fail(BGTQ_ELAYOUT, "Block-GTQ keys need tables");
    if (kind == BGTQ_KEYS_FP16 && (dim < 2 || dim % 2 || dim > 128)) return fail(BGTQ_EINVAL, "Invalid K dimensions");
    if (capacity < 1 || capacity > (1u << 31) || sequences < 1) return fail(BGTQ_EINVAL, "Unsupported K capacity");
    auto *k = new bgtq_keys();
    k->kind = kind;
    k->device = device;
    k->capacity = capacity;
    k->sequences = sequences;
    k->cap_alloc = round_up(capacity, kTileRows);
    DeviceGuard g(device);
    if (!g.ok) {
        delete k;
        return fail(BGTQ_ECUDA, "cannot select device");
    }
    // the device status word every kernel reports into exists once any store does, so
    // entry points that must not allocate (bgtq_attend_static) always find it
    if (!device_status_word(device)) {
        delete k;
        return fail(BGTQ_ENOMEM, "status word allocation failed");
    }
    auto cleanup = [&](bgtq_status s, const std::string &m) {
        if (k->rows) cudaFree(k->rows);
        if (k->scales) cudaFree(k->scales);
        if (k->d_lengths) cudaFree(k->d_lengths);
        if (k->dt.blob) cudaFree(k->dt.blob);
        delete k;
        return fail(s, m);
    };
    if (kind == BGTQ_KEYS_FP16) {
        k->dim = dim;
        k->D = dim_template(dim);
        k->row_stride = k->D * 2;
    } else {
        k->L = tables->L;
        k->dim = k->L.d;
        k->D = dim_template(k->dim);
        k->row_stride = k->L.dev_row_stride;
        k->scale_stride = k->L.dev_scale_stride;
        cudaError_t e = upload_tables(k->L, k->dt);
        if (e != cudaSuccess) return cleanup(BGTQ_ECUDA, std::string("tables upload: ") + cudaGetErrorString(e));
        k->ledger.push_back({"K tables", "shared", (uint64_t)k->dt.bytes});
    }
    const size_t rows_bytes = (size_t)sequences * k->cap_alloc * k->row_stride;
    if (cudaMalloc(&k->rows, rows_bytes) != cudaSuccess) return cleanup(BGTQ_ENOMEM, "K allocation failed");
    cudaMemset(k->rows, 0, rows_bytes);
    k->ledger.push_back({kind == BGTQ_KEYS_FP16 ? "FP16 K" : "K nibble/byte capacity", "persistent-k", rows_bytes});
    if (kind != BGTQ_KEYS_FP16) {
        const size_t sb = (size_t)sequences * k->cap_alloc * k->scale_stride * 2;
        if (cudaMalloc(&k->scales, sb) != cudaSuccess) return cleanup(BGTQ_ENOMEM, "K scale allocation failed");
        cudaMemset(k->scales, 0, sb);
        k->ledger.push_back({"K FP16 scale capacity", "persistent-k", sb});
    }
    // per-sequence lengths, then one word the K/V append kernel counts its finished CTAs in
    if (cudaMalloc(&k->d_lengths, sizeof(uint32_t) * (sequences + 1)) != cudaSuccess)
        return cleanup(BGTQ_ENOMEM, "length allocation failed");
    cudaMemset(k->d_lengths, 0, sizeof(uint32_t) * (sequences + 1));
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cleanup(BGTQ_ECUDA, std::string("K init: ") + cudaGetErrorString(e));
    k->lengths.assign(sequences, 0);
    *out = k;
    return BGTQ_OK;
}

void bgtq_keys_destroy(bgtq_keys *k) {
    if (!k) return;
    DeviceGuard g(k->device);
    cudaFree(k->rows);
    if (k->scales) cudaFree(k->scales);
    cudaFree(k->d_lengths);
    if (k->dt.blob) cudaFree(k->dt.blob);
    k->row0.release();
    k->staging.release();
    k->materialized.release();
    delete k;
}

bgtq_status bgtq_keys_append(bgtq_keys *k, const void *src, bgtq_dtype dtype, int host, uint32_t count,
                             uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                             void *stream_) {
    if (!k) return fail(BGTQ_EINVAL, "null keys");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    bgtq_status s = check_append(k->dim, k->capacity, k->sequences, k->lengths, src, dtype, count, row_stride,
                                 seq_first, seq_count, "K");
    if (s != BGTQ_OK) return s;
    const bool packed = k->kind != BGTQ_KEYS_FP16;
    if (!host && packed) {
        const size_t align = dtype == BGTQ_F16 ? 4 : 8;
        if (reinterpret_cast<uintptr_t>(src) % align || row_stride % 2 || (seq_count > 1 && seq_stride % 2))
            return fail(BGTQ_EINVAL, "device K source must be aligned with even strides");
    }
    DeviceGuard g(k->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    const void *dsrc;
    uint64_t drow, dseq;
    s = stage_source(src, dtype, host, k->dim, count, row_stride, seq_count, seq_stride, k->staging, stream, &dsrc, &drow,
                     &dseq);
    if (s != BGTQ_OK) return s;
    const uint32_t *row0 = nullptr;
    uint32_t row0_scalar = 0;
    std::vector<uint32_t> tmp;
    s = start_rows(k->lengths, seq_first, seq_count, k->row0, stream, &row0, &row0_scalar, tmp);
    if (s != BGTQ_OK) return s;
    cudaError_t e;
    if (packed) {
        EncodeArgs a;
        std::memset(&a, 0, sizeof(a));
        fill_encode_head(k, a.head[0]);
        a.src = dsrc;
        a.row_stride = drow;
        a.seq_stride = dseq;
        a.row0 = row0;
        a.row0_scalar = row0_scalar;
        a.count = count;
        a.seq_first = seq_first;
        a.seq_count = seq_count;
        a.heads = 1;
        a.src_f32 = dtype == BGTQ_F32;
        a.status = device_status_word(k->device);
        e = launch_encode(a, k->dim, (uint32_t)k->L.cent_compact.size() + 256u, k->L.ncb, stream);
    } else {
        e = launch_copy_rows(k->rows, (uint64_t)k->cap_alloc * k->D, k->D, 0, dsrc, drow, dseq, dtype == BGTQ_F32, row0,
                             row0_scalar, count, seq_first, seq_count, k->d_lengths, k->dim, 0, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "K append launch");
    if (host) {
        e = cudaStreamSynchronize(stream);  // the staging buffer is reused by the next call
        if (e != cudaSuccess) return cuda_fail(e, "K append");
    }
    for (uint32_t i = 0; i < seq_count; ++i) k->lengths[seq_first + i] += count;
    return BGTQ_OK;
}

namespace {
// Shared checks and launch of the one-launch K/V appends (bgtq_append_kv_rope, bgtq_append_kv).
bgtq_status append_kv_common(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, KvRopeArgs &a,
                             uint32_t count, uint32_t seq_first, uint32_t seq_count, void *stream_) {
    if (!keys || !values || heads < 1 || heads > (uint32_t)kMaxHeads) return fail(BGTQ_EINVAL, "Invalid K/V append");
    const bgtq_keys *k0 = keys[0];
    if (!k0) return fail(BGTQ_EINVAL, "Invalid K/V append");
    const uint32_t d = k0->dim;
    if (d % 2 || !count || !seq_count || (uint64_t)seq_first + seq_count > k0->sequences)
        return fail(BGTQ_EINVAL, "Invalid K/V append");
    for (uint32_t h = 0; h < heads; ++h) {
        const bgtq_keys *k = keys[h];
        const bgtq_values *v = values[h];
        if (!k || !v || k->kind != BGTQ_KEYS_PACKED || k->dim != d || v->dim != d || v->dtype != BGTQ_F16 ||
            k->device != k0->device || v->device != k0->device || k->sequences != k0->sequences ||
            v->sequences != k0->sequences)
            return fail(BGTQ_EINVAL, "K/V append needs packed keys and FP16 values of one head dim");
        for (uint32_t s = 0; s < seq_count; ++s) {
            const uint32_t seq = seq_first + s, L = k0->lengths[seq];
            if (k->lengths[seq] != L || v->lengths[seq] != L) return fail(BGTQ_EBUSY, "K/V lengths must match");
            if ((uint64_t)L + count > std::min(k->capacity, v->capacity))
                return fail(BGTQ_ECAPACITY, "K capacity exceeded");
        }
    }
    DeviceGuard g(k0->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    for (uint32_t h = 0; h < heads; ++h) {
        fill_encode_head(keys[h], a.head[h]);
        a.v[h] = values[h]->data;
        a.v_lengths[h] = values[h]->d_lengths;
        a.v_seq_stride[h] = (uint64_t)values[h]->cap_alloc * values[h]->D;
    }
    a.start = k0->d_lengths;
    a.ticket = k0->d_lengths + k0->sequences;
    a.count = count;
    a.seq_first = seq_first;
    a.seq_count = seq_count;
    a.heads = heads;
    a.vD = values[0]->D;
    a.v_swizzle = values_swizzled(0, values[0]->D) ? 1u : 0u;
    a.capacity = ~0u;
    for (uint32_t h = 0; h < heads; ++h) a.capacity = std::min(a.capacity, std::min(keys[h]->capacity, values[h]->capacity));
    a.status = device_status_word(k0->device);
    if (!a.status) return fail(BGTQ_ECUDA, "no status word");
    cudaError_t e = launch_kv_rope_append(a, d, static_cast<cudaStream_t>(stream_));
    if (e != cudaSuccess) return cuda_fail(e, "K/V append launch");
    for (uint32_t h = 0; h < heads; ++h)
        for (uint32_t s = 0; s < seq_count; ++s) {
            keys[h]->lengths[seq_first + s] += count;
            values[h]->lengths[seq_first + s] += count;
        }
    return BGTQ_OK;
}
}  // namespace

bgtq_status bgtq_append_kv_rope(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, const float *src,
                                uint64_t row_stride, uint64_t seq_stride, uint32_t k_offset, uint32_t v_offset,
                                uint32_t count, uint32_t seq_first, uint32_t seq_count, const float *inv_freq,
                                void *stream_) {
    if (!keys || !keys[0] || !src || !inv_freq || reinterpret_cast<uintptr_t>(src) % 4 ||
        row_stride < (uint64_t)std::max(k_offset, v_offset) + heads * keys[0]->dim)
        return fail(BGTQ_EINVAL, "Invalid K/V append");
    KvRopeArgs a;
    std::memset(&a, 0, sizeof(a));
    a.k_src = src + k_offset;
    a.v_src = src + v_offset;
    a.row_stride = row_stride;
    a.seq_stride = seq_stride;
    a.rope = 1;
    for (uint32_t p = 0; p < keys[0]->dim / 2 && p < kMaxDim / 2; ++p) a.inv_freq[p] = inv_freq[p];
    return append_kv_common(heads, keys, values, a, count, seq_first, seq_count, stream_);
}

bgtq_status bgtq_append_kv(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, const void *k_src,
                           bgtq_dtype k_dtype, const void *v_src, bgtq_dtype v_dtype, int host, uint32_t count,
                           uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                           void *stream_) {
    if (!keys || !keys[0] || !values || !values[0] || !k_src || !v_src || (k_dtype != BGTQ_F16 && k_dtype != BGTQ_F32) ||
        (v_dtype != BGTQ_F16 && v_dtype != BGTQ_F32) || row_stride < (uint64_t)heads * keys[0]->dim ||
        reinterpret_cast<uintptr_t>(k_src) % (k_dtype == BGTQ_F16 ? 2 : 4) ||
        reinterpret_cast<uintptr_t>(v_src) % (v_dtype == BGTQ_F16 ? 2 : 4))
        return fail(BGTQ_EINVAL, "Invalid K/V append");
    if (host) {
        // host sources: one dense [seq_count][count][heads][dim] block each, checked, then
        // uploaded to the first stores' staging buffers in stream order (no host wait: a later
        // upload into the same buffer is queued behind this launch on the same stream)
        const uint32_t d = keys[0]->dim;
        const uint64_t n = (uint64_t)seq_count * count * heads * d;
        if (row_stride != (uint64_t)heads * d || (seq_count > 1 && seq_stride != (uint64_t)count * row_stride) ||
            !count || !seq_count)
            return fail(BGTQ_EINVAL, "host K/V append needs dense [sequences][count][heads][dim] sources");
        if (!host_finite(k_src, k_dtype, (uint32_t)(n / seq_count), 1, 0, seq_count, (uint64_t)count * row_stride))
            return fail(BGTQ_ENONFINITE, "Finite FP16 K required");
        if (!host_finite(v_src, v_dtype, (uint32_t)(n / seq_count), 1, 0, seq_count, (uint64_t)count * row_stride))
            return fail(BGTQ_ENONFINITE, "finite inputs required");
        DeviceGuard g(keys[0]->device);
        if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
        cudaStream_t stream = static_cast<cudaStream_t>(stream_);
        const size_t kb = n * (k_dtype == BGTQ_F16 ? 2 : 4), vb = n * (v_dtype == BGTQ_F16 ? 2 : 4);
        CK(keys[0]->staging.ensure(kb), "staging allocation");
        CK(values[0]->staging.ensure(vb), "staging allocation");
        CK(cudaMemcpyAsync(keys[0]->staging.p, k_src, kb, cudaMemcpyHostToDevice, stream), "K upload");
        CK(cudaMemcpyAsync(values[0]->staging.p, v_src, vb, cudaMemcpyHostToDevice, stream), "V upload");
        k_src = keys[0]->staging.p;
        v_src = values[0]->staging.p;
        seq_stride = (uint64_t)count * row_stride;
    }
    KvRopeArgs a;
    std::memset(&a, 0, sizeof(a));
    a.k_src = k_src;
    a.v_src = v_src;
    a.k_f16 = k_dtype == BGTQ_F16 ? 1u : 0u;
    a.v_f16 = v_dtype == BGTQ_F16 ? 1u : 0u;
    a.row_stride = row_stride;
    a.seq_stride = seq_stride;
    return append_kv_common(heads, keys, values, a, count, seq_first, seq_count, stream_);
}

bgtq_status bgtq_keys_length(const bgtq_keys *k, uint32_t seq, uint32_t *out) {
    if (!k || !out || seq >= k->sequences) return fail(BGTQ_EINVAL, "invalid argument");
    *out = k->lengths[seq];
    return BGTQ_OK;
}

bgtq_status bgtq_keys_reset(bgtq_keys *k, void *stream) {
    if (!k) return fail(BGTQ_EINVAL, "null keys");
    DeviceGuard g(k->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    CK(cudaMemsetAsync(k->d_lengths, 0, (size_t)k->sequences * 4, static_cast<cudaStream_t>(stream)), "reset");
    std::fill(k->lengths.begin(), k->lengths.end(), 0u);
    return BGTQ_OK;
}

bgtq_status bgtq_keys_info(const bgtq_keys *k, bgtq_keys_kind *kind, uint32_t *dim, uint32_t *capacity,
                           uint32_t *sequences) {
    if (!k) return fail(BGTQ_EINVAL, "null keys");
    if (kind) *kind = k->kind;
    if (dim) *dim = k->dim;
    if (capacity) *capacity = k->capacity;
    if (sequences) *sequences = k->sequences;
    return BGTQ_OK;
}

bgtq_status bgtq_keys_layout(const bgtq_keys *k, bgtq_layout_info *info) {
    if (!k || !info) return fail(BGTQ_EINVAL, "null argument");
    if (k->kind == BGTQ_KEYS_FP16) return fail(BGTQ_EINVAL, "FP16 keys have no Block-GTQ layout");
    const Layout &L = k->L;
    info->dim = L.d;
    info->groups = L.ng;
    info->row_bytes = L.row_bytes;
    info->norm_stride = L.norm_stride;
    info->nibble_dims = L.ns;
    info->max_centroids = L.maxc;
    info->logical_row_bytes = L.logical_rb;
    info->device_row_stride = L.dev_row_stride;
    info->device_scale_stride = L.dev_scale_stride;
    info->codebooks = L.ncb;
    return BGTQ_OK;
}

bgtq_status bgtq_keys_read(const bgtq_keys *k, uint32_t seq, uint32_t row0, uint32_t count, uint8_t *packed_out,
                           uint16_t *scales_out) {
    if (!k || seq >= k->sequences || (uint64_t)row0 + count > k->cap_alloc) return fail(BGTQ_EINVAL, "invalid range");
    DeviceGuard g(k->device);
    CK(cudaDeviceSynchronize(), "K read");
    if (k->kind == BGTQ_KEYS_FP16) {
        if (packed_out && count)
            CK(cudaMemcpy2D(packed_out, (size_t)k->dim * 2,
                            k->rows + ((uint64_t)seq * k->cap_alloc + row0) * k->row_stride, k->row_stride,
                            (size_t)k->dim * 2, count, cudaMemcpyDeviceToHost),
               "K read");
        return BGTQ_OK;
    }
    const uint32_t rb = k->L.row_bytes, w = std::min(rb, k->row_stride);
    if (packed_out && count) {
        std::memset(packed_out, 0, (size_t)rb * count);
        CK(cudaMemcpy2D(packed_out, rb, k->rows + ((uint64_t)seq * k->cap_alloc + row0) * k->row_stride, k->row_stride, w,
                        count, cudaMemcpyDeviceToHost),
           "K read");
    }
    if (scales_out && count) {
        const uint32_t ns = k->L.norm_stride, ws = std::min(ns, k->scale_stride);
        std::memset(scales_out, 0, (size_t)ns * 2 * count);
        CK(cudaMemcpy2D(scales_out, (size_t)ns * 2,
                        k->scales + ((uint64_t)seq * k->cap_alloc + row0) * k->scale_stride, (size_t)k->scale_stride * 2,
                        (size_t)ws * 2, count, cudaMemcpyDeviceToHost),
           "K read");
    }
    return BGTQ_OK;
}

static bgtq_status reconstruct_into(const bgtq_keys *k, uint32_t seq, float *out, cudaStream_t stream) {
    ReconArgs a;
    std::memset(&a, 0, sizeof(a));
    a.t = k->dt;
    a.packed = k->rows + (uint64_t)seq * k->cap_alloc * k->row_stride;
    a.scales = k->scales + (uint64_t)seq * k->cap_alloc * k->scale_stride;
    a.row_stride = k->row_stride;
    a.scale_stride = k->scale_stride;
    a.ns = k->L.ns;
    a.d = k->dim;
    a.rows = k->lengths[seq];
    a.out = out;
    cudaError_t e = launch_reconstruct(a, (uint32_t)k->L.cent_compact.size(), stream);
    if (e != cudaSuccess) return cuda_fail(e, "reconstruct launch");
    return BGTQ_OK;
}

bgtq_status bgtq_keys_reconstruct(const bgtq_keys *k, uint32_t seq, float *out, void *stream) {
    if (!k || !out || seq >= k->sequences) return fail(BGTQ_EINVAL, "invalid argument");
    if (k->kind == BGTQ_KEYS_FP16) return fail(BGTQ_EINVAL, "FP16 keys need no reconstruction");
    DeviceGuard g(k->device);
    return reconstruct_into(k, seq, out, static_cast<cudaStream_t>(stream));
}

bgtq_status bgtq_keys_allocations(const bgtq_keys *k, bgtq_allocation *out, uint32_t cap, uint32_t *n_out) {
    if (!k) return fail(BGTQ_EINVAL, "null keys");
    std::vector<bgtq_allocation> all = k->ledger;
    if (k->materialized.bytes) all.push_back({"materialized FP32 K", "scratch", (uint64_t)k->materialized.bytes});
    if (n_out) *n_out = (uint32_t)all.size();
    for (uint32_t i = 0; out && i < cap && i < all.size(); ++i) out[i] = all[i];
    return BGTQ_OK;
}

bgtq_status bgtq_values_create(bgtq_dtype dtype, uint32_t dim, uint32_t capacity, uint32_t sequences, int device,
                               bgtq_values **out) {
    if (!out) return fail(BGTQ_EINVAL, "null output");
    if ((dtype != BGTQ_F16 && dtype != BGTQ_F32) || dim < 1 || dim > 128 || capacity < 1 || capacity > (1u << 31) ||
        sequences < 1)
        return fail(BGTQ_EINVAL, "Invalid V dimensions");
    auto *v = new bgtq_values();
    v->dtype = dtype;
    v->device = device;
    v->dim = dim;
    v->D = dim_template(dim);
    v->capacity = capacity;
    v->cap_alloc = round_up(capacity, kTileRows);
    v->sequences = sequences;
    DeviceGuard g(device);
    if (!device_status_word(device)) {
        delete v;
        return fail(BGTQ_ENOMEM, "status word allocation failed");
    }
    const size_t es = dtype == BGTQ_F16 ? 2 : 4;
    const size_t bytes = (size_t)sequences * v->cap_alloc * v->D * es;
    if (cudaMalloc(&v->data, bytes) != cudaSuccess) {
        delete v;
        return fail(BGTQ_ENOMEM, "V allocation failed");
    }
    if (cudaMalloc(&v->d_lengths, sizeof(uint32_t) * sequences) != cudaSuccess) {
        cudaFree(v->data);
        delete v;
        return fail(BGTQ_ENOMEM, "V allocation failed");
    }
    cudaMemset(v->data, 0, bytes);
    cudaMemset(v->d_lengths, 0, sizeof(uint32_t) * sequences);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(v->data);
        cudaFree(v->d_lengths);
        delete v;
        return cuda_fail(e, "V init");
    }
    v->lengths.assign(sequences, 0);
    *out = v;
    return BGTQ_OK;
}

void bgtq_values_destroy(bgtq_values *v) {
    if (!v) return;
    DeviceGuard g(v->device);
    cudaFree(v->data);
    cudaFree(v->d_lengths);
    v->row0.release();
    v->staging.release();
    delete v;
}

bgtq_status bgtq_values_append(bgtq_values *v, const void *src, bgtq_dtype dtype, int host, uint32_t count,
                               uint64_t row_stride, uint32_t seq_first, uint32_t seq_count, uint64_t seq_stride,
                               void *stream_) {
    if (!v) return fail(BGTQ_EINVAL, "null values");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    bgtq_status s = check_append(v->dim, v->capacity, v->sequences, v->lengths, src, dtype, count, row_stride, seq_first,
                                 seq_count, "V");
    if (s != BGTQ_OK) return s;
    DeviceGuard g(v->device);
    const void *dsrc;
    uint64_t drow, dseq;
    s = stage_source(src, dtype, host, v->dim, count, row_stride, seq_count, seq_stride, v->staging, stream, &dsrc, &drow,
                     &dseq);
    if (s != BGTQ_OK) return s;
    const uint32_t *row0 = nullptr;
    uint32_t row0_scalar = 0;
    std::vector<uint32_t> tmp;
    s = start_rows(v->lengths, seq_first, seq_count, v->row0, stream, &row0, &row0_scalar, tmp);
    if (s != BGTQ_OK) return s;
    cudaError_t e = launch_copy_rows(v->data, (uint64_t)v->cap_alloc * v->D, v->D, v->dtype == BGTQ_F32, dsrc, drow, dseq,
                                     dtype == BGTQ_F32, row0, row0_scalar, count, seq_first, seq_count, v->d_lengths,
                                     v->dim, values_swizzled(v->dtype == BGTQ_F32, v->D) ? 1 : 0, stream);
    if (e != cudaSuccess) return cuda_fail(e, "V append launch");
    if (host) {
        e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "V append");
    }
    for (uint32_t i = 0; i < seq_count; ++i) v->lengths[seq_first + i] += count;
    return BGTQ_OK;
}

bgtq_status bgtq_values_info(const bgtq_values *v, bgtq_dtype *dtype, uint32_t *dim, uint32_t *capacity,
                             uint32_t *sequences) {
    if (!v) return fail(BGTQ_EINVAL, "null argument");
    if (dtype) *dtype = v->dtype;
    if (dim) *dim = v->dim;
    if (capacity) *capacity = v->capacity;
    if (sequences) *sequences = v->sequences;
    return BGTQ_OK;
}

bgtq_status bgtq_values_read(const bgtq_values *v, uint32_t seq, uint32_t row0, uint32_t count, void *out) {
    if (!v || !out || seq >= v->sequences || (uint64_t)row0 + count > v->cap_alloc)
        return fail(BGTQ_EINVAL, "invalid range");
    if (!count) return BGTQ_OK;
    DeviceGuard g(v->device);
    CK(cudaDeviceSynchronize(), "V read");
    const size_t es = v->dtype == BGTQ_F32 ? 4 : 2, row = (size_t)v->D * es;
    std::vector<unsigned char> raw((size_t)count * row);
    CK(cudaMemcpy(raw.data(), static_cast<const unsigned char *>(v->data) + ((uint64_t)seq * v->cap_alloc + row0) * row,
                  raw.size(), cudaMemcpyDeviceToHost),
       "V read");
    const bool swz = values_swizzled(v->dtype == BGTQ_F32, v->D);
    unsigned char *o = static_cast<unsigned char *>(out);
    for (uint32_t r = 0; r < count; ++r) {
        const uint32_t t = row0 + r;
        for (uint32_t e = 0; e < v->dim; ++e) {
            uint32_t de = e;
            if (swz) {
                const uint32_t c = e >> 3;
                de = (((c & ~7u) | ((c ^ t) & 7u)) << 3) | (e & 7u);
            }
            std::memcpy(o + ((size_t)r * v->dim + e) * es, raw.data() + (size_t)r * row + (size_t)de * es, es);
        }
    }
    return BGTQ_OK;
}

bgtq_status bgtq_values_length(const bgtq_values *v, uint32_t seq, uint32_t *out) {
    if (!v || !out || seq >= v->sequences) return fail(BGTQ_EINVAL, "invalid argument");
    *out = v->lengths[seq];
    return BGTQ_OK;
}

bgtq_status bgtq_values_reset(bgtq_values *v, void *stream) {
    if (!v) return fail(BGTQ_EINVAL, "null values");
    DeviceGuard g(v->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    CK(cudaMemsetAsync(v->d_lengths, 0, (size_t)v->sequences * 4, static_cast<cudaStream_t>(stream)), "reset");
    std::fill(v->lengths.begin(), v->lengths.end(), 0u);
    return BGTQ_OK;
}

bgtq_status bgtq_attention_create(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values, uint32_t rows,
                                  bgtq_attention **out) {
    if (!out || !keys || !values || heads < 1 || heads > (uint32_t)kMaxHeads)
        return fail(BGTQ_EINVAL, "Incompatible attention storage");
    if (rows < 1 || rows > (uint32_t)kMaxRows) return fail(BGTQ_EINVAL, "Incompatible attention storage");
    for (uint32_t h = 0; h < heads; ++h) {
        const bgtq_keys *k = keys[h];
        const bgtq_values *v = values[h];
        if (!k || !v || k->device != v->device || k->dim != v->dim || k->capacity != v->capacity ||
            k->sequences != v->sequences || k->device != keys[0]->device || k->dim != keys[0]->dim ||
            k->capacity != keys[0]->capacity || k->sequences != keys[0]->sequences || k->kind != keys[0]->kind ||
            v->dtype != values[0]->dtype)
            return fail(BGTQ_EINVAL, "Incompatible attention storage");
    }
    auto *a = new bgtq_attention();
    a->heads = heads;
    a->rows = rows;
    a->dim = keys[0]->dim;
    a->sequences = keys[0]->sequences;
    a->device = keys[0]->device;
    a->keys.assign(keys, keys + heads);
    a->values.assign(values, values + heads);
    DeviceGuard g(a->device);
    const size_t pairs = (size_t)a->sequences * heads;
    // split-KV partials: up to 64 splits, capped at 16 MiB of workspace
    const size_t per_split = pairs * rows * (a->dim + 2) * sizeof(float);
    a->max_splits = (uint32_t)std::max<size_t>(1, std::min<size_t>(64, (16u << 20) / per_split));
    const size_t part_bytes = a->max_splits * per_split;
    if (cudaMalloc(&a->part, part_bytes) != cudaSuccess || cudaMalloc(&a->counters, pairs * sizeof(uint32_t)) != cudaSuccess ||
        cudaMalloc(&a->lse, pairs * rows * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&a->qt, pairs * kMaxDim * kMaxRows * sizeof(float)) != cudaSuccess) {
        if (a->part) cudaFree(a->part);
        if (a->counters) cudaFree(a->counters);
        if (a->lse) cudaFree(a->lse);
        delete a;
        return fail(BGTQ_ENOMEM, "attention workspace allocation failed");
    }
    cudaMemset(a->counters, 0, pairs * sizeof(uint32_t));
    if (!device_status_word(a->device)) {
        bgtq_attention_destroy(a);
        return fail(BGTQ_ENOMEM, "status word allocation failed");
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        bgtq_attention_destroy(a);
        return cuda_fail(e, "attention init");
    }
    *out = a;
    return BGTQ_OK;
}

void bgtq_attention_destroy(bgtq_attention *a) {
    if (!a) return;
    DeviceGuard g(a->device);
    if (a->part) cudaFree(a->part);
    if (a->counters) cudaFree(a->counters);
    if (a->lse) cudaFree(a->lse);
    if (a->qt) cudaFree(a->qt);
    a->q_dev.release();
    a->pos_dev.release();
    a->out_dev.release();
    a->logits_dev.release();
    a->probs_dev.release();
    a->prefill_qt.release();
    a->rope.release();
    delete a;
}

}  // extern "C"

namespace bgtq {
// Kernel arguments of one packed-key head with its value store.
void fill_encode_head(const bgtq_keys *k, EncodeHead &h) {
    std::memset(&h, 0, sizeof(h));
    h.t = k->dt;
    h.packed = k->rows;
    h.scales = k->scales;
    h.k_seq_stride = (uint64_t)k->cap_alloc * k->row_stride;
    h.s_seq_stride = (uint64_t)k->cap_alloc * k->scale_stride;
    h.row_stride = k->row_stride;
    h.scale_stride = k->scale_stride;
    h.ns = k->L.ns;
    h.ng = k->L.ng;
    h.n_cent = (uint32_t)k->L.cent_compact.size();
    h.ncb = k->L.ncb;
    for (int i = 0; i < 4; ++i) h.bound_mask[i] = k->L.bound_mask[i];
    for (int g = 0; g <= kMaxGroups; ++g) h.group_off[g] = k->L.group_off[g];
    h.lengths = k->d_lengths;
}

void fill_packed_head(AttnHead &ah, const bgtq_keys *k, const bgtq_values *v) {
    const size_t vsz = v->dtype == BGTQ_F32 ? 4 : 2;
    ah.v = v->data;
    ah.v_seq_stride = (uint64_t)v->cap_alloc * v->D * vsz;
    ah.k = k->rows;
    ah.k_seq_stride = (uint64_t)k->cap_alloc * k->row_stride;
    ah.row_stride = k->row_stride;
    ah.scales = k->scales;
    ah.s_seq_stride = (uint64_t)k->cap_alloc * k->scale_stride;
    ah.scale_stride = k->scale_stride;
    ah.rot = k->dt.rot;
    ah.cent = k->dt.cent;
    ah.perm = k->dt.perm;
    ah.group_of = k->dt.group_of;
    ah.ns = k->L.ns;
    ah.ng = k->L.ng;
    ah.n_cent = (uint32_t)k->L.cent_compact.size();
    ah.lookup = k->dt.lookup;
    ah.lookup_off = k->dt.lookup_off;
    ah.n_lookup = (uint32_t)k->L.lookup.size();
    for (int i = 0; i < 4; ++i) ah.bound_mask[i] = k->L.bound_mask[i];
    for (int gi = 0; gi <= kMaxGroups; ++gi) ah.group_off[gi] = k->L.group_off[gi];
    for (uint32_t j = 0; j < (uint32_t)kMaxDim; ++j) ah.cb_base[j] = j < k->dim ? k->L.cb_base[j] : (uint16_t)ah.n_cent;
}
}  // namespace bgtq

extern "C" {

bgtq_status bgtq_attend(bgtq_attention *at, const float *q, const uint32_t *positions, int causal, uint32_t rows,
                        uint32_t seq_first, uint32_t seq_count, float *out, float *logits, float *probs, int host,
                        void *stream_) {
    if (!at || !q || !out) return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    if (rows < 1 || rows > at->rows || !seq_count || (uint64_t)seq_first + seq_count > at->sequences)
        return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    if (probs && !logits) return fail(BGTQ_EINVAL, "probabilities need logits");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const uint32_t d = at->dim, H = at->heads;
    // optimized.ts:29-31: ready storage, equal K/V lengths, positions inside the context
    uint32_t max_len = 0, min_len = ~0u;
    for (uint32_t s = 0; s < seq_count; ++s) {
        const uint32_t seq = seq_first + s, L = at->keys[0]->lengths[seq];
        for (uint32_t h = 0; h < H; ++h)
            if (at->keys[h]->lengths[seq] != L || at->values[h]->lengths[seq] != L)
                return fail(BGTQ_EBUSY, "K/V lengths must match and be nonzero");
        if (!L) return fail(BGTQ_EBUSY, "K/V lengths must match and be nonzero");
        max_len = std::max(max_len, L);
        min_len = std::min(min_len, L);
    }
    if (logits && min_len != max_len) return fail(BGTQ_EINVAL, "logit capture needs equal lengths");
    // a launch recorded once and replayed while the sequences grow plans its splits for the
    // longest length it may meet
    const uint32_t plan_len = at->plan_capacity && !logits ? at->keys[0]->capacity : max_len;
    if (host) {
        if (!host_finite(q, BGTQ_F32, d, seq_count * H * rows, d, 1, 0))
            return fail(BGTQ_ENONFINITE, "Q: finite inputs required");
        if (positions)
            for (uint32_t s = 0; s < seq_count; ++s)
                for (uint32_t r = 0; r < rows; ++r)
                    if (positions[(size_t)s * rows + r] >= at->keys[0]->lengths[seq_first + s])
                        return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    }
    DeviceGuard g(at->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    uint32_t launches = 0;
    const float *dq = q;
    const uint32_t *dpos = positions;
    float *dout = out, *dlogits = logits, *dprobs = probs;
    const size_t nq = (size_t)seq_count * H * rows * d;
    const size_t nl = (size_t)seq_count * H * rows * max_len;
    if (host) {
        CK(at->q_dev.ensure(nq * 4), "Q staging");
        CK(at->out_dev.ensure(nq * 4), "output staging");
        CK(cudaMemcpyAsync(at->q_dev.p, q, nq * 4, cudaMemcpyHostToDevice, stream), "Q upload");
        dq = static_cast<const float *>(at->q_dev.p);
        dout = static_cast<float *>(at->out_dev.p);
        if (positions) {
            CK(at->pos_dev.ensure((size_t)seq_count * rows * 4), "position staging");
            CK(cudaMemcpyAsync(at->pos_dev.p, positions, (size_t)seq_count * rows * 4, cudaMemcpyHostToDevice, stream),
               "position upload");
            dpos = static_cast<const uint32_t *>(at->pos_dev.p);
        }
        if (logits) {
            CK(at->logits_dev.ensure(nl * 4), "logit staging");
            dlogits = static_cast<float *>(at->logits_dev.p);
        }
        if (probs) {
            CK(at->probs_dev.ensure(nl * 4), "probability staging");
            dprobs = static_cast<float *>(at->probs_dev.p);
        }
    }
    // FP32 keys for the materialising (CompressedKeys) path: reconstruct, then dense attention
    const bgtq_keys *k0 = at->keys[0];
    KKind kk = k0->kind == BGTQ_KEYS_PACKED ? KKind::Packed : k0->kind == BGTQ_KEYS_FP16 ? KKind::F16 : KKind::F32;
    AttnArgs a;
    std::memset(&a, 0, sizeof(a));
    uint32_t max_cent = 0;
    for (uint32_t h = 0; h < H; ++h) {
        bgtq_keys *k = at->keys[h];
        const bgtq_values *v = at->values[h];
        AttnHead &ah = a.head[h];
        const size_t vsz = v->dtype == BGTQ_F32 ? 4 : 2;
        ah.v = v->data;
        ah.v_seq_stride = (uint64_t)v->cap_alloc * v->D * vsz;
        if (kk == KKind::Packed) {
            fill_packed_head(ah, k, v);
            max_cent = std::max(max_cent, ah.n_lookup);
        } else if (kk == KKind::F16) {
            ah.k = k->rows;
            ah.k_seq_stride = (uint64_t)k->cap_alloc * k->row_stride;
            ah.row_stride = k->row_stride;
            ah.scale_stride = 4;
        } else {
            // materialise every requested sequence: [sequences][cap_alloc][D] FP32
            const size_t per_seq = (size_t)k->cap_alloc * k->D * 4;
            CK(k->materialized.ensure(per_seq * k->sequences), "materialized K allocation");
            if (k->D != k->dim) CK(cudaMemsetAsync(k->materialized.p, 0, per_seq * k->sequences, stream), "clear");
            for (uint32_t s = 0; s < seq_count; ++s) {
                const uint32_t seq = seq_first + s;
                // reconstruct writes [length][dim]; the dense kernel reads rows of D floats
                float *dst = reinterpret_cast<float *>(static_cast<unsigned char *>(k->materialized.p) + per_seq * seq);
                if (k->D == k->dim) {
                    bgtq_status st = reconstruct_into(k, seq, dst, stream);
                    if (st != BGTQ_OK) return st;
                    ++launches;
                } else {
                    return fail(BGTQ_ELAYOUT, "materialised attention needs dim 16, 32, 64 or 128");
                }
            }
            ah.k = static_cast<const uint8_t *>(k->materialized.p);
            ah.k_seq_stride = per_seq;
            ah.row_stride = k->D * 4;
            ah.scale_stride = 4;
        }
    }
    a.q = dq;
    a.qt = at->qt;
    a.positions = dpos;
    a.lengths = k0->d_lengths;
    a.out = dout;
    a.logits = dlogits;
    a.lse = (logits || probs) ? at->lse : nullptr;
    a.part = at->part;
    a.counters = at->counters + 0;
    a.rope = at->use_rope ? static_cast<const float *>(at->rope.p) : nullptr;
    a.status = device_status_word(at->device);
    a.seq_first = seq_first;
    a.seq_count = seq_count;
    a.heads = H;
    a.rows = rows;
    a.causal = causal ? 1u : 0u;
    a.logit_stride = max_len;
    uint32_t splits = 1, sk = 0, attn_launches = 2;
    cudaError_t e = launch_attention(a, kk, at->values[0]->dtype == BGTQ_F32, d, max_cent, plan_len, at->forced_splits,
                                     at->max_splits, at->schedule, &splits, &sk, stream, &attn_launches);
    if (e != cudaSuccess) return cuda_fail(e, "attention launch");
    launches += attn_launches;  // query rotation (unless fused) + attention
    if (probs) {
        e = launch_probs(dlogits, at->lse, dprobs, (uint64_t)seq_count * H * rows, max_len, max_len, stream);
        if (e != cudaSuccess) return cuda_fail(e, "probabilities launch");
        ++launches;
    }
    at->last_splits = splits;
    at->last_sk_units = sk;
    at->last_launches = launches;
    if (host) {
        CK(cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, stream), "output download");
        if (logits) CK(cudaMemcpyAsync(logits, dlogits, nl * 4, cudaMemcpyDeviceToHost, stream), "logit download");
        if (probs) CK(cudaMemcpyAsync(probs, dprobs, nl * 4, cudaMemcpyDeviceToHost, stream), "probability download");
        if (host != 2) CK(cudaStreamSynchronize(stream), "attend");  // 2: the caller waits on the stream
    }
    return BGTQ_OK;
}

bgtq_status bgtq_attend_prefill(bgtq_attention *at, const float *q, uint32_t pos_first, uint32_t n, uint32_t gqa,
                                uint32_t seq_first, uint32_t seq_count, float *out, int host, void *stream_) {
    if (!at || !q || !out) return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    if (!n || !seq_count || gqa < 1 || gqa > (uint32_t)kMaxRows || (uint64_t)seq_first + seq_count > at->sequences ||
        (uint64_t)pos_first + n > 0xffffffffull)
        return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    const uint32_t d = at->dim, H = at->heads;
    if (d > 64) return fail(BGTQ_EINVAL, "prefill needs head dim <= 64");
    for (uint32_t h = 0; h < H; ++h)
        if (at->keys[h]->kind != BGTQ_KEYS_PACKED || at->values[h]->dtype != BGTQ_F16)
            return fail(BGTQ_EINVAL, "prefill needs packed keys and FP16 values");
    // every query position must have its key appended: lengths >= pos_first + n
    for (uint32_t s = 0; s < seq_count; ++s) {
        const uint32_t seq = seq_first + s, L = at->keys[0]->lengths[seq];
        for (uint32_t h = 0; h < H; ++h)
            if (at->keys[h]->lengths[seq] != L || at->values[h]->lengths[seq] != L)
                return fail(BGTQ_EBUSY, "K/V lengths must match and be nonzero");
        if ((uint64_t)pos_first + n > L) return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    }
    const size_t nq = (size_t)seq_count * n * H * gqa * d;
    if (host && !host_finite(q, BGTQ_F32, d, seq_count * n * H * gqa, d, 1, 0))
        return fail(BGTQ_ENONFINITE, "Q: finite inputs required");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    DeviceGuard g(at->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    const float *dq = q;
    float *dout = out;
    if (host) {
        CK(at->q_dev.ensure(nq * 4), "Q staging");
        CK(at->out_dev.ensure(nq * 4), "output staging");
        CK(cudaMemcpyAsync(at->q_dev.p, q, nq * 4, cudaMemcpyHostToDevice, stream), "Q upload");
        dq = static_cast<const float *>(at->q_dev.p);
        dout = static_cast<float *>(at->out_dev.p);
    }
    CK(at->prefill_qt.ensure((size_t)seq_count * n * H * gqa * 64 * 4), "query record allocation");
    PrefillArgs a;
    std::memset(&a, 0, sizeof(a));
    uint32_t max_cent = 0;
    for (uint32_t h = 0; h < H; ++h) {
        fill_packed_head(a.head[h], at->keys[h], at->values[h]);
        max_cent = std::max(max_cent, a.head[h].n_cent);
    }
    a.q = dq;
    a.qt = static_cast<float *>(at->prefill_qt.p);
    a.out = dout;
    a.lengths = at->keys[0]->d_lengths;
    a.status = device_status_word(at->device);
    a.rope = at->use_rope ? static_cast<const float *>(at->rope.p) : nullptr;
    a.seq_first = seq_first;
    a.seq_count = seq_count;
    a.heads = H;
    a.gqa = gqa;
    a.n = n;
    a.pos_first = pos_first;
    a.d = d;
    cudaError_t e = launch_prefill(a, max_cent, at->prefill_kernel == 0 ? 1 : 0, stream);
    if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
    at->last_splits = 1;
    at->last_launches = 2;  // query rotation + prefill attention
    if (host) {
        CK(cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, stream), "output download");
        CK(cudaStreamSynchronize(stream), "prefill");
    }
    return BGTQ_OK;
}

bgtq_status bgtq_attention_last_splits(const bgtq_attention *a, uint32_t *out) {
    if (!a || !out) return fail(BGTQ_EINVAL, "null argument");
    *out = a->last_splits;
    return BGTQ_OK;
}
bgtq_status bgtq_attention_set_splits(bgtq_attention *a, uint32_t splits) {
    if (!a || splits > 64) return fail(BGTQ_EINVAL, "invalid split count");
    a->forced_splits = splits;
    return BGTQ_OK;
}
bgtq_status bgtq_attention_set_schedule(bgtq_attention *a, int mode) {
    if (!a || mode < 0 || mode > 2) return fail(BGTQ_EINVAL, "invalid schedule");
    a->schedule = mode;
    return BGTQ_OK;
}
bgtq_status bgtq_attention_last_stream_k(const bgtq_attention *a, uint32_t *units_out) {
    if (!a || !units_out) return fail(BGTQ_EINVAL, "null argument");
    *units_out = a->last_sk_units;
    return BGTQ_OK;
}
bgtq_status bgtq_attention_plan_for_capacity(bgtq_attention *a, int on) {
    if (!a) return fail(BGTQ_EINVAL, "null attention");
    a->plan_capacity = on != 0;
    return BGTQ_OK;
}

bgtq_status bgtq_keys_sync_lengths(bgtq_keys *k) {
    if (!k) return fail(BGTQ_EINVAL, "null keys");
    DeviceGuard g(k->device);
    CK(cudaMemcpy(k->lengths.data(), k->d_lengths, (size_t)k->sequences * 4, cudaMemcpyDeviceToHost), "lengths");
    return BGTQ_OK;
}

bgtq_status bgtq_values_sync_lengths(bgtq_values *v) {
    if (!v) return fail(BGTQ_EINVAL, "null values");
    DeviceGuard g(v->device);
    CK(cudaMemcpy(v->lengths.data(), v->d_lengths, (size_t)v->sequences * 4, cudaMemcpyDeviceToHost), "lengths");
    return BGTQ_OK;
}

bgtq_status bgtq_attention_set_rope(bgtq_attention *a, const float *inv_freq, uint32_t n) {
    if (!a || (n && (!inv_freq || n != a->dim / 2))) return fail(BGTQ_EINVAL, "RoPE table must hold dim/2 entries");
    if (!n) {
        a->use_rope = false;
        return BGTQ_OK;
    }
    DeviceGuard g(a->device);
    if (!g.ok) return fail(BGTQ_ECUDA, "cannot select device");
    CK(a->rope.ensure((size_t)n * 4), "RoPE table allocation");
    CK(cudaMemcpy(a->rope.p, inv_freq, (size_t)n * 4, cudaMemcpyHostToDevice), "RoPE table upload");
    a->use_rope = true;
    return BGTQ_OK;
}

bgtq_status bgtq_attention_set_prefill_kernel(bgtq_attention *a, uint32_t kernel) {
    if (!a || kernel > 1) return fail(BGTQ_EINVAL, "invalid prefill kernel");
    a->prefill_kernel = kernel;
    return BGTQ_OK;
}
bgtq_status bgtq_attention_last_launches(const bgtq_attention *a, uint32_t *out) {
    if (!a || !out) return fail(BGTQ_EINVAL, "null argument");
    *out = a->last_launches;
    return BGTQ_OK;
}

bgtq_status bgtq_device_status(int device, uint32_t *out) {
    if (!out) return fail(BGTQ_EINVAL, "null argument");
    DeviceGuard g(device);
    uint32_t *w = device_status_word(device);
    if (!w) return fail(BGTQ_ECUDA, "no status word");
    CK(cudaMemcpy(out, w, sizeof(uint32_t), cudaMemcpyDeviceToHost), "status read");
    return BGTQ_OK;
}

}  // extern "C"
