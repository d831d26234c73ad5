// Compressed-K attention that allocates no device memory: bgtq_attend_static.
//
// Who needs it: callers that run attention where they must not (or cannot) allocate -
// a serving process that hands all free device memory to its own pool once the KV
// caches exist, or a plugin whose host framework owns every device allocation and
// forbids the plugin's own cudaMalloc.  The regular path (bgtq_attention_create +
// bgtq_attend) keeps per-object workspace that is allocated when the object is created;
// this entry point needs no attention object and takes its scratch from one fixed array
// compiled into the library instead.
//
// Scratch: g_scratch below, kScratchBytes (4 MiB + 64 KiB) in every GPU that loads the
// library, held until the process exits.  It holds the split-KV partial results, the
// per-(sequence, head) completion tickets and the rotated query records.  Every call
// shares it, so calls whose kernels overlap on the GPU (different streams, or different
// host threads on one device) race and must be serialised by the caller.  The tickets
// must start at zero and are cleared with cudaMemsetAsync at the start of every call.
// Bounded-wait timeouts go to the library's device status word (bgtq_device_status),
// which exists as soon as any key or value store does.
//
// Set-up: the first call on each device (that device current) looks up the device
// address of g_scratch with cudaGetSymbolAddress and has the driver load the code of
// every kernel this entry point can launch, so later calls load nothing; both results
// are kept per device for the life of the process.  Make that first call before any
// stream capture starts, and do not keep using the library on a device across a
// cudaDeviceReset (the kept address belongs to the old context).
#include <algorithm>
#include <cstring>
#include <mutex>

#include "objects.h"

namespace {

constexpr size_t kPartFloats = 3u << 18;   // split-KV partials: 786,432 floats (3 MiB)
constexpr size_t kQtFloats = 1u << 18;     // query records: 262,144 floats (1 MiB)
constexpr size_t kTickets = 1u << 14;      // (sequence, head) tickets: 16,384 (64 KiB)
constexpr size_t kScratchBytes = (kPartFloats + kQtFloats + kTickets) * 4;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_addr[64] = {};

bgtq_status fail(bgtq_status s, const std::string &m) {
    bgtq::set_last_error(m);
    return s;
}

uint32_t dim_template(uint32_t d) { return d <= 16 ? 16u : d <= 32 ? 32u : d <= 64 ? 64u : 128u; }
uint32_t rows_pad(uint32_t r) { return r <= 1 ? 1u : r <= 2 ? 2u : r <= 4 ? 4u : 8u; }

// Set-up on `device` (which must be current), once: the device address of g_scratch, and
// the code of every generic packed-key attention kernel loaded.
cudaError_t scratch_address(int device, void **out) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess) return e;
        e = bgtq::preload_attention_kernels(bgtq::KKind::Packed);
        if (e != cudaSuccess) return e;
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return cudaSuccess;
}

}  // namespace

extern "C" bgtq_status bgtq_attend_static(uint32_t heads, bgtq_keys *const *keys, bgtq_values *const *values,
                                          const float *q, const uint32_t *positions, int causal, uint32_t rows,
                                          uint32_t seq_first, uint32_t seq_count, float *out, void *stream_) {
    using namespace bgtq;
    if (!keys || !values || !q || !out || heads < 1 || heads > (uint32_t)kMaxHeads || rows < 1 ||
        rows > (uint32_t)kMaxRows || !seq_count)
        return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    const bgtq_keys *k0 = keys[0];
    if (!k0 || k0->kind != BGTQ_KEYS_PACKED) return fail(BGTQ_EINVAL, "static-scratch attention needs packed keys");
    if ((uint64_t)seq_first + seq_count > k0->sequences) return fail(BGTQ_EINVAL, "Invalid Q/K/V shape or positions");
    for (uint32_t h = 0; h < heads; ++h) {
        const bgtq_keys *k = keys[h];
        const bgtq_values *v = values[h];
        if (!k || !v || k->kind != BGTQ_KEYS_PACKED || k->device != k0->device || v->device != k0->device ||
            k->dim != k0->dim || v->dim != k0->dim || k->capacity != k0->capacity || v->capacity != k0->capacity ||
            k->sequences != k0->sequences || v->sequences != k0->sequences || v->dtype != values[0]->dtype)
            return fail(BGTQ_EINVAL, "Incompatible attention storage");
    }
    const uint32_t d = k0->dim, D = dim_template(d), QP = rows_pad(rows);
    // the limits of the static scratch
    const uint64_t pairs = (uint64_t)seq_count * heads;
    if (pairs > kTickets || pairs * D * QP > kQtFloats)
        return fail(BGTQ_EINVAL, "static scratch holds query records for at most " + std::to_string(kQtFloats) +
                                     " floats (sequences x heads x " + std::to_string(D) + " x " +
                                     std::to_string(QP) + " requested " + std::to_string(pairs * D * QP) + ")");
    uint32_t max_len = 0;
    for (uint32_t s = 0; s < seq_count; ++s) {
        const uint32_t seq = seq_first + s, L = k0->lengths[seq];
        for (uint32_t h = 0; h < heads; ++h)
            if (keys[h]->lengths[seq] != L || values[h]->lengths[seq] != L)
                return fail(BGTQ_EBUSY, "K/V lengths must match and be nonzero");
        if (!L) return fail(BGTQ_EBUSY, "K/V lengths must match and be nonzero");
        max_len = std::max(max_len, L);
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != k0->device && cudaSetDevice(k0->device) != cudaSuccess) return fail(BGTQ_ECUDA, "cannot select device");
    struct Restore {
        int dev;
        ~Restore() {
            int cur = -1;
            if (dev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != dev) cudaSetDevice(dev);
        }
    } restore{prev};
    void *base = nullptr;
    cudaError_t e = scratch_address(k0->device, &base);
    if (e != cudaSuccess) return fail(BGTQ_ECUDA, std::string("scratch address: ") + cudaGetErrorString(e));
    float *part = static_cast<float *>(base);
    float *qt = part + kPartFloats;
    uint32_t *tickets = reinterpret_cast<uint32_t *>(qt + kQtFloats);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    e = cudaMemsetAsync(tickets, 0, pairs * sizeof(uint32_t), stream);
    if (e != cudaSuccess) return fail(BGTQ_ECUDA, std::string("ticket clear: ") + cudaGetErrorString(e));

    AttnArgs a;
    std::memset(&a, 0, sizeof(a));
    uint32_t max_cent = 0;
    for (uint32_t h = 0; h < heads; ++h) {
        fill_packed_head(a.head[h], keys[h], values[h]);
        max_cent = std::max(max_cent, a.head[h].n_lookup);
    }
    a.q = q;
    a.qt = qt;
    a.positions = positions;
    a.lengths = k0->d_lengths;
    a.out = out;
    a.part = part;
    a.counters = tickets;
    // bounded-wait timeouts go to the library's status word (bgtq_device_status), which
    // the key stores created when they were made
    a.status = device_status_word_if_present(k0->device);
    if (!a.status) return fail(BGTQ_ECUDA, "device status word missing");
    a.seq_first = seq_first;
    a.seq_count = seq_count;
    a.heads = heads;
    a.rows = rows;
    a.causal = causal ? 1u : 0u;
    a.logit_stride = max_len;
    // as many splits as the partial buffer holds (at least one: a single split writes
    // its result directly and uses no partials)
    const uint64_t per_split = pairs * rows * (d + 2);
    const uint32_t max_splits = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(64, kPartFloats / per_split));
    uint32_t splits = 1;
    jit_suppress_on_thread(1);  // generic kernel: loading a specialised one would allocate
    e = launch_attention(a, KKind::Packed, values[0]->dtype == BGTQ_F32, d, max_cent, max_len, 0, max_splits, 0, &splits,
                         nullptr, stream);
    jit_suppress_on_thread(0);
    if (e != cudaSuccess) return fail(BGTQ_ECUDA, std::string("attention launch: ") + cudaGetErrorString(e));
    return BGTQ_OK;
}
