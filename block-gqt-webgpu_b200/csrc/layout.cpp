// Host-side table parsing and validation, and the greedy bit allocator.
//
// parse_layout() accepts exactly the reference's flattened tables (src/webgpu/layout.ts:24-31)
// and applies validateLayout (layout.ts:8-23) and the PackedKeys transform-group check
// (src/runtime/packed-keys.ts:15-23), raising the same classes of error.  It additionally
// requires what the CUDA kernels rely on and every reference table satisfies: group ids
// increase along the (head-permuted) dimension order, codes are whole bytes or nibbles.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <set>
#include <string>

#include "bgtq_internal.h"

namespace bgtq {

void build_lookup_layout(Layout &L, const std::vector<uint32_t> &cb_size);

static bgtq_status fail(std::string &err, bgtq_status s, const char *msg) {
    err = msg;
    return s;
}

bgtq_status parse_layout(const uint32_t *config, size_t n_config, const float *table, size_t n_table, Layout &L,
                         std::string &err) {
    if (!config || !table || n_config < 10) return fail(err, BGTQ_ELAYOUT, "Invalid Block-GTQ layout");
    const uint32_t d = config[0], ng = config[1], rb = config[2], nstride = config[3], ns = config[4], maxc = config[5];
    // validateLayout, layout.ts:10-13
    if (d < 2 || d > 128 || d % 2 || ng < 1 || ng > 8 || nstride < ng || ns > d || ns % 2 ||
        rb < ns / 2 + d - ns || maxc < 2 || maxc > 256)
        return fail(err, BGTQ_ELAYOUT, "Invalid Block-GTQ layout");
    const uint64_t off_perm = config[6], off_grp = config[7], off_cb = config[8], off_lut = config[9];
    if (off_perm + d > n_config || off_grp + d > n_config || off_cb + d > n_config || off_lut > n_config)
        return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
    const uint64_t lut_len = n_config - off_lut;
    if (lut_len == 0 || lut_len % 256) return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
    if ((uint64_t)n_table != (uint64_t)d * d + (uint64_t)d * maxc + 2ull * d)
        return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
    L = Layout();
    L.d = d; L.ng = ng; L.row_bytes = rb; L.norm_stride = nstride; L.ns = ns; L.maxc = maxc;
    L.ncb = (uint32_t)(lut_len / 256);
    L.logical_rb = ns / 2 + d - ns;
    // an odd number of 32-bit words: lanes reading word k of 32 consecutive rows in shared
    // memory hit 32 different banks
    L.dev_row_stride = 4u * (((L.logical_rb + 3u) / 4u) | 1u);
    L.dev_scale_stride = ng <= 4 ? 4u : 8u;
    L.perm.resize(d); L.group_of.resize(d); L.pos_to_cb.resize(d);
    std::set<uint32_t> seen;
    for (uint32_t i = 0; i < d; ++i) {
        const uint32_t p = config[off_perm + i], g = config[off_grp + i], c = config[off_cb + i];
        if (p >= d) return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
        seen.insert(p);
        if (g >= ng) return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
        if ((uint64_t)c * 256 >= lut_len) return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
        L.perm[i] = (uint8_t)p; L.group_of[i] = (uint8_t)g; L.pos_to_cb[i] = (uint8_t)c;
    }
    if (seen.size() != d) return fail(err, BGTQ_ELAYOUT, "Invalid calibration table shape");
    for (size_t i = 0; i < n_table; ++i)
        if (!std::isfinite(table[i])) return fail(err, BGTQ_ELAYOUT, "Nonfinite calibration table");
    L.lut.resize(lut_len);
    for (uint64_t i = 0; i < lut_len; ++i) {
        const uint32_t v = config[off_lut + i];
        if (v > 255) return fail(err, BGTQ_ELAYOUT, "Code LUT incompatible with packing");
        L.lut[i] = (uint8_t)v;
    }
    // layout.ts:19-22: every reachable code fits the centroid table and its nibble/byte slot
    std::vector<uint32_t> cb_size(d, 1);
    for (uint32_t i = 0; i < d; ++i)
        for (uint32_t bin = 0; bin < 256; ++bin) {
            const uint32_t code = L.lut[(uint64_t)L.pos_to_cb[i] * 256 + bin];
            if (code >= maxc || (i < ns && code > 15)) return fail(err, BGTQ_ELAYOUT, "Code LUT incompatible with packing");
            if (code + 1 > cb_size[i]) cb_size[i] = code + 1;
        }
    L.rot.assign(table, table + (size_t)d * d);
    L.cent.assign(table + (size_t)d * d, table + (size_t)d * d + (size_t)d * maxc);
    L.off.assign(table + (size_t)d * d + (size_t)d * maxc, table + (size_t)d * d + (size_t)d * maxc + d);
    L.inv.assign(table + (size_t)d * d + (size_t)d * maxc + d, table + n_table);
    // packed-keys.ts:15-23: contiguous groups, zero off-group transform entries
    L.ranges.assign(2 * (size_t)d, 0);
    for (uint32_t j = 0; j < d; ++j) {
        int start = -1, end = -1;
        uint32_t members = 0;
        for (uint32_t i = 0; i < d; ++i)
            if (L.group_of[i] == L.group_of[j]) {
                if (start < 0) start = (int)i;
                end = (int)i + 1;
                ++members;
            }
        if ((uint32_t)(end - start) != members) return fail(err, BGTQ_ELAYOUT, "Non-contiguous transform group");
        for (uint32_t i = 0; i < d; ++i)
            if (((int)i < start || (int)i >= end) && L.rot[(size_t)i * d + j] != 0.0f)
                return fail(err, BGTQ_ELAYOUT, "Off-group transform is nonzero");
        L.ranges[2 * j] = (uint32_t)start;
        L.ranges[2 * j + 1] = (uint32_t)end;
    }
    // kernel requirement: groups appear in ascending id order along the dimensions and
    // every group id is used
    for (uint32_t i = 1; i < d; ++i)
        if (L.group_of[i] < L.group_of[i - 1] || L.group_of[i] > L.group_of[i - 1] + 1)
            return fail(err, BGTQ_ELAYOUT, "Groups must occupy ascending dimension ranges in id order");
    if (L.group_of[0] != 0 || L.group_of[d - 1] != ng - 1)
        return fail(err, BGTQ_ELAYOUT, "Groups must occupy ascending dimension ranges in id order");
    for (uint32_t g = 0; g <= ng; ++g) L.group_off[g] = d;
    for (int i = (int)d - 1; i >= 0; --i) L.group_off[L.group_of[i]] = (uint32_t)i;
    L.group_off[ng] = d;
    for (uint32_t g = 1; g < ng; ++g) {
        const uint32_t j = L.group_off[g];
        L.bound_mask[j >> 5] |= 1u << (j & 31);
    }
    // kernel requirement: groups hold whole RoPE pairs and the nibble/byte split falls
    // on a group boundary (groups are width classes, so every reference table does)
    bool ns_on_boundary = ns == 0 || ns == d;
    for (uint32_t g = 0; g <= ng; ++g) {
        if (L.group_off[g] % 2) return fail(err, BGTQ_ELAYOUT, "Groups must hold whole dimension pairs");
        ns_on_boundary |= L.group_off[g] == ns;
    }
    if (!ns_on_boundary) return fail(err, BGTQ_ELAYOUT, "Nibble/byte split must fall on a group boundary");
    // compact per-dimension codebooks (entries 0..max reachable code)
    L.cb_base.resize(d);
    uint32_t total = 0;
    for (uint32_t i = 0; i < d; ++i) {
        L.cb_base[i] = (uint16_t)total;
        total += cb_size[i];
    }
    L.cent_compact.resize(total);
    for (uint32_t i = 0; i < d; ++i)
        for (uint32_t c = 0; c < cb_size[i]; ++c) L.cent_compact[L.cb_base[i] + c] = L.cent[(size_t)i * maxc + c];
    build_lookup_layout(L, cb_size);
    return BGTQ_OK;
}

// The decode-attention kernel walks each group's dimension pairs in runs of four (one
// 32-bit word of nibble codes, two words of byte codes) and forms a lookup address without
// a separate add:
//  - nibble groups: run b (numbered over all groups, each group starting a new run) owns the
//    512-byte slot b; the even dimension of its pair p has its 16-entry codebook at float
//    128 b + 16 p, the odd one at 128 b + 64 + 16 p.  With the slot 256-byte aligned, one
//    byte permute of (code * 4, slot address) is the address, and p's offset is a constant.
//  - byte groups: each dimension gets a slot of P = next power of two >= its group's largest
//    codebook, aligned to P floats (groups placed in descending P, after the nibble slots),
//    so slot | code * 4 is the address.
// Slots are zero past each codebook's reachable codes.
void build_lookup_layout(Layout &L, const std::vector<uint32_t> &cb_size) {
    const uint32_t d = L.d;
    L.lookup_off.assign(d, 0);
    uint32_t runs = 0, g_first_run[kMaxGroups] = {}, pmax = 1, pg[kMaxGroups] = {};
    for (uint32_t g = 0; g < L.ng; ++g) {
        const uint32_t a = L.group_off[g], b = L.group_off[g + 1];
        g_first_run[g] = runs;
        if (a < L.ns) {
            runs += ((b - a) / 2 + 3) / 4;
        } else {
            uint32_t m = 1;
            for (uint32_t j = a; j < b; ++j) m = std::max(m, cb_size[j]);
            uint32_t p = 1;
            while (p < m) p *= 2;
            pg[g] = p;
            pmax = std::max(pmax, p);
        }
    }
    uint32_t cursor = runs * 128u;
    cursor = (cursor + pmax - 1) / pmax * pmax;
    for (uint32_t g = 0; g < L.ng; ++g) {
        const uint32_t a = L.group_off[g], b = L.group_off[g + 1];
        if (a >= L.ns) continue;
        for (uint32_t j = a; j < b; ++j) {
            const uint32_t q = j / 2 - a / 2;
            L.lookup_off[j] = (uint16_t)((g_first_run[g] + q / 4) * 128u + (j & 1u) * 64u + (q % 4) * 16u);
        }
    }
    for (uint32_t p = pmax; p >= 1; p /= 2)
        for (uint32_t g = 0; g < L.ng; ++g) {
            if (L.group_off[g] < L.ns || pg[g] != p) continue;
            for (uint32_t j = L.group_off[g]; j < L.group_off[g + 1]; ++j) {
                L.lookup_off[j] = (uint16_t)cursor;
                cursor += p;
            }
        }
    L.lookup.assign(cursor, 0.0f);
    for (uint32_t j = 0; j < d; ++j)
        for (uint32_t c = 0; c < cb_size[j]; ++c) L.lookup[L.lookup_off[j] + c] = L.cent_compact[L.cb_base[j] + c];
}

}  // namespace bgtq

extern "C" bgtq_status bgtq_allocate_bits(const float *scores, uint32_t n, int64_t budget, int32_t min_bits,
                                          int32_t max_bits, int64_t *widths_out) {
    if ((!scores && n) || !widths_out || min_bits > max_bits) return BGTQ_EINVAL;
    for (uint32_t i = 0; i < n; ++i) widths_out[i] = min_bits;
    int64_t remaining = budget - (int64_t)min_bits * (int64_t)n;
    // allocator.py:9-16: priorities = float32(score) * 4.0**-width in float64; first max wins
    while (remaining > 0 && n > 0) {
        uint32_t best = 0;
        double best_p = 0.0;
        bool have = false;
        for (uint32_t i = 0; i < n; ++i) {
            double p = (double)scores[i] * std::pow(4.0, -(double)widths_out[i]);
            if (widths_out[i] >= max_bits) p = -1.0;
            if (!have || p > best_p) { best_p = p; best = i; have = true; }
        }
        if (best_p <= 0.0) break;
        widths_out[best] += 1;
        remaining -= 1;
    }
    return BGTQ_OK;
}
