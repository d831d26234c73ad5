// Block-GTQ table builder (host C++): per-pair bit widths -> the flattened config / table
// arrays the runtime consumes (src/webgpu/layout.ts:24-31), without Python.
//
// Restates, step for step, the reference's table construction:
//   - dimension order, groups, block-diagonal rotation, Lloyd-Max centroids
//     (BlockGTQPipeline._post_allocation_setup, vendor/blockgtq/block_gtq_pipeline.py:151-246;
//     _optimal_centroids_torch :24-78; _random_rotation_dense_torch :81-92),
//   - the 256-bin code LUT, offsets and inverse scales (build_code_lut,
//     vendor/blockgtq/quant_kernels.py:276-364),
//   - the nibble / byte split (build_pack_meta, vendor/blockgtq/quantizer.py:34-106).
//
// Numerics, and where they can differ from the reference:
//   - The Haar rotation of a width class is NumPy's: Generator(PCG64(SeedSequence(42 + w)))
//     .standard_normal((n, n)), QR, columns signed by diag(R), first column negated when
//     det < 0.  PCG64 and SeedSequence are reproduced exactly (M. O'Neill's PCG XSL-RR
//     128/64 and NumPy's published SeedSequence hash).  Normals use the 256-layer
//     Marsaglia-Tsang ziggurat (r = 3.6541528853610088) with tables computed here from the
//     method's recurrence in long double: they agree with NumPy's to a few ulps, so an
//     accept/reject decision could in principle differ (never observed).  QR is unblocked
//     Householder (LAPACK dgeqr2/dorg2r order of operations) in double; the rotation is
//     stored in FP32, which absorbs the last-ulp differences of double arithmetic.
//   - Centroids iterate Lloyd-Max exactly as the reference (100 passes from quantile
//     boundaries) with the normal CDF from erfc (Cephes ndtr form) and the quantile from
//     Acklam's rational approximation refined by two Halley steps; stored in FP32.
//   - Bin centres follow torch.linspace in FP32 (step = (end - start) / 255 rounded to
//     FP32, each value one fused multiply-add from the nearer end); bins map to centroids by
//     a left binary search over the FP32 boundaries, like torch.searchsorted.
//   - Pairs are ordered like the reference's torch.argsort, which is not stable: torch's
//     CPU sort is std::sort over (width, index) pairs compared by width, and so is this
//     (libstdc++ introsort).  Ties can order differently under another sort implementation.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <utility>
#include <string>
#include <vector>

#include "bgtq_internal.h"

namespace bgtq {
namespace builder {

// ---- NumPy SeedSequence (pool of 4 words) and PCG64 ----
static void seed_sequence_u64(uint64_t seed, uint64_t (&out)[4]) {
    const uint32_t INIT_A = 0x43b0d7e5u, MULT_A = 0x931e8875u, INIT_B = 0x8b51f9ddu, MULT_B = 0x58f38dedu;
    const uint32_t MIX_L = 0xca01f9ddu, MIX_R = 0x4973f715u;
    std::vector<uint32_t> ent;
    ent.push_back((uint32_t)seed);
    if (seed >> 32) ent.push_back((uint32_t)(seed >> 32));
    uint32_t hc = INIT_A;
    auto hashmix = [&](uint32_t v) {
        v ^= hc;
        hc *= MULT_A;
        v *= hc;
        return v ^ (v >> 16);
    };
    auto mix = [&](uint32_t x, uint32_t y) {
        uint32_t r = MIX_L * x - MIX_R * y;
        return r ^ (r >> 16);
    };
    uint32_t pool[4];
    for (int i = 0; i < 4; ++i) pool[i] = hashmix(i < (int)ent.size() ? ent[i] : 0u);
    for (int s = 0; s < 4; ++s)
        for (int d = 0; d < 4; ++d)
            if (s != d) pool[d] = mix(pool[d], hashmix(pool[s]));
    for (size_t s = 4; s < ent.size(); ++s)
        for (int d = 0; d < 4; ++d) pool[d] = mix(pool[d], hashmix(ent[s]));
    uint32_t h = INIT_B, words[8];
    for (int i = 0; i < 8; ++i) {
        uint32_t v = pool[i % 4];
        v ^= h;
        h *= MULT_B;
        v *= h;
        v ^= v >> 16;
        words[i] = v;
    }
    for (int i = 0; i < 4; ++i) out[i] = (uint64_t)words[2 * i] | ((uint64_t)words[2 * i + 1] << 32);
}

struct Pcg64 {
    unsigned __int128 state = 0, inc = 0;
    static constexpr unsigned __int128 kMult =
        ((unsigned __int128)2549297995355413924ull << 64) | (unsigned __int128)4865540595714422341ull;
    explicit Pcg64(uint64_t seed) {
        uint64_t v[4];
        seed_sequence_u64(seed, v);
        const unsigned __int128 s = ((unsigned __int128)v[0] << 64) | v[1];
        const unsigned __int128 q = ((unsigned __int128)v[2] << 64) | v[3];
        inc = (q << 1) | 1u;
        state = 0;
        step();
        state += s;
        step();
    }
    void step() { state = state * kMult + inc; }
    uint64_t next64() {
        step();
        const uint64_t x = (uint64_t)(state >> 64) ^ (uint64_t)state;
        const unsigned r = (unsigned)(state >> 122);
        return (x >> r) | (x << ((64u - r) & 63u));
    }
    double next_double() { return (double)(next64() >> 11) * (1.0 / 9007199254740992.0); }
};

// ---- 256-layer ziggurat for the standard normal (Marsaglia & Tsang 2000) ----
struct Ziggurat {
    uint64_t ki[256];
    double wi[256], fi[256];
    static constexpr double kR = 3.6541528853610088;
    Ziggurat() {
        typedef long double ld;
        const ld R = 3.6541528853610087963519472518L;
        // layer area: r f(r) + the tail integral, f(x) = exp(-x^2/2)
        const ld V = R * expl(-0.5L * R * R) + sqrtl(acosl(-1.0L) / 2.0L) * erfcl(R / sqrtl(2.0L));
        const ld m1 = 4503599627370496.0L;  // 2^52
        ld dn = R, tn = R;
        const ld q = V / expl(-0.5L * dn * dn);
        ki[0] = (uint64_t)((dn / q) * m1);
        ki[1] = 0;
        wi[0] = (double)(q / m1);
        wi[255] = (double)(dn / m1);
        fi[0] = 1.0;
        fi[255] = (double)expl(-0.5L * dn * dn);
        for (int i = 254; i >= 1; --i) {
            dn = sqrtl(-2.0L * logl(V / dn + expl(-0.5L * dn * dn)));
            ki[i + 1] = (uint64_t)((dn / tn) * m1);
            tn = dn;
            fi[i] = (double)expl(-0.5L * dn * dn);
            wi[i] = (double)(dn / m1);
        }
    }
    double normal(Pcg64 &g) const {
        for (;;) {
            uint64_t r = g.next64();
            const int idx = (int)(r & 0xffu);
            r >>= 8;
            const int sign = (int)(r & 1u);
            const uint64_t rabs = (r >> 1) & 0x000fffffffffffffull;
            double x = (double)rabs * wi[idx];
            if (sign) x = -x;
            if (rabs < ki[idx]) return x;
            if (idx == 0) {
                for (;;) {
                    const double xx = -(1.0 / kR) * std::log1p(-g.next_double());
                    const double yy = -std::log1p(-g.next_double());
                    if (yy + yy > xx * xx) return ((rabs >> 8) & 1u) ? -(kR + xx) : kR + xx;
                }
            } else if ((fi[idx - 1] - fi[idx]) * g.next_double() + fi[idx] < std::exp(-0.5 * x * x)) {
                return x;
            }
        }
    }
};

// ---- Householder QR (LAPACK dgeqr2 / dorg2r order), column-major n x n ----
static double lapy2(double x, double y) {
    const double xa = std::fabs(x), ya = std::fabs(y), w = std::max(xa, ya), z = std::min(xa, ya);
    if (z == 0.0) return w;
    const double t = z / w;
    return w * std::sqrt(1.0 + t * t);
}
static double nrm2(const double *x, int n) {
    double scale = 0.0, ssq = 1.0;
    for (int i = 0; i < n; ++i) {
        if (x[i] != 0.0) {
            const double a = std::fabs(x[i]);
            if (scale < a) {
                ssq = 1.0 + ssq * (scale / a) * (scale / a);
                scale = a;
            } else {
                ssq += (a / scale) * (a / scale);
            }
        }
    }
    return scale * std::sqrt(ssq);
}
// apply H = I - tau v v^T (v[0] = 1 implied by the caller's storage) to columns c0..n-1 of
// the trailing block rows r0..n-1
static void apply_reflector(std::vector<double> &A, int n, int r0, int c0, const double *v, double tau) {
    if (tau == 0.0) return;
    const int m = n - r0;
    for (int c = c0; c < n; ++c) {
        double *col = &A[(size_t)c * n + r0];
        double w = 0.0;
        for (int i = 0; i < m; ++i) w += v[i] * col[i];
        w *= tau;
        for (int i = 0; i < m; ++i) col[i] -= w * v[i];
    }
}

// Haar rotation of size n from NumPy's generator seeded with `seed`; row-major FP32 out[n*n].
void haar_rotation(int n, uint64_t seed, float *out) {
    static const Ziggurat zig;
    Pcg64 g(seed);
    std::vector<double> A((size_t)n * n);  // column-major: A[c*n + r] = G[r][c]
    for (int r = 0; r < n; ++r)
        for (int c = 0; c < n; ++c) A[(size_t)c * n + r] = zig.normal(g);
    std::vector<double> tau(n, 0.0), rdiag(n, 0.0);
    // dgeqr2
    for (int i = 0; i < n; ++i) {
        double *col = &A[(size_t)i * n + i];
        const int m = n - i;
        double alpha = col[0];
        double t = 0.0;
        if (m > 1) {
            const double xnorm = nrm2(col + 1, m - 1);
            if (xnorm != 0.0) {
                const double beta = -std::copysign(lapy2(alpha, xnorm), alpha);
                t = (beta - alpha) / beta;
                const double s = 1.0 / (alpha - beta);
                for (int k = 1; k < m; ++k) col[k] *= s;
                alpha = beta;
            }
        }
        tau[i] = t;
        rdiag[i] = alpha;
        if (i < n - 1) {
            const double keep = col[0];
            col[0] = 1.0;
            apply_reflector(A, n, i, i + 1, col, t);
            col[0] = keep;
        }
        col[0] = alpha;
    }
    // dorg2r: Q from the reflectors, last to first
    for (int i = n - 1; i >= 0; --i) {
        double *col = &A[(size_t)i * n + i];
        if (i < n - 1) {
            col[0] = 1.0;
            apply_reflector(A, n, i, i + 1, col, tau[i]);
        }
        for (int k = 1; k < n - i; ++k) col[k] *= -tau[i];
        col[0] = 1.0 - tau[i];
        for (int k = 0; k < i; ++k) A[(size_t)i * n + k] = 0.0;
    }
    // columns signed by diag(R); det(Q) = prod over reflectors (-1 each) * prod(signs)
    int det_neg = 0;
    for (int i = 0; i < n; ++i) {
        const double sg = rdiag[i] > 0.0 ? 1.0 : rdiag[i] < 0.0 ? -1.0 : 1.0;
        if (sg < 0.0) {
            det_neg ^= 1;
            for (int r = 0; r < n; ++r) A[(size_t)i * n + r] = -A[(size_t)i * n + r];
        }
        if (tau[i] != 0.0) det_neg ^= 1;
    }
    if (det_neg)
        for (int r = 0; r < n; ++r) A[r] = -A[r];
    for (int r = 0; r < n; ++r)
        for (int c = 0; c < n; ++c) out[(size_t)r * n + c] = (float)A[(size_t)c * n + r];
}

// ---- normal distribution helpers ----
static double ndtr(double a) {
    const double x = a * 0.70710678118654752440, z = std::fabs(x);
    double y;
    if (z < 0.70710678118654752440) {
        y = 0.5 + 0.5 * std::erf(x);
    } else {
        y = 0.5 * std::erfc(z);
        if (x > 0) y = 1.0 - y;
    }
    return y;
}
static double norm_pdf(double x) {
    if (std::isinf(x)) return 0.0;
    return std::exp(-x * x / 2.0) / std::sqrt(2.0 * M_PI);
}
// inverse standard normal CDF: Acklam's rational approximation + two Halley steps
static double ndtri(double p) {
    static const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                                1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
    static const double b[5] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                                6.680131188771972e+01, -1.328068155288572e+01};
    static const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                                -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
    static const double d[4] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                                3.754408661907416e+00};
    double x;
    if (p < 0.02425) {
        const double q = std::sqrt(-2 * std::log(p));
        x = (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
            ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    } else if (p > 1 - 0.02425) {
        const double q = std::sqrt(-2 * std::log(1 - p));
        x = -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
            ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1);
    } else {
        const double q = p - 0.5, r = q * q;
        x = (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
            (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1);
    }
    for (int it = 0; it < 2; ++it) {
        const double e = ndtr(x) - p, u = e * std::sqrt(2 * M_PI) * std::exp(x * x / 2);
        x = x - u / (1 + x * u / 2);
    }
    return x;
}

// E[X | a < X < b] for X ~ N(0, sig^2) (_cond_exp of the reference)
static double cond_exp(double sig, double a, double b) {
    const double a_std = std::isfinite(a) ? a / sig : a, b_std = std::isfinite(b) ? b / sig : b;
    double prob;
    if (!std::isfinite(a_std)) prob = ndtr(b_std);
    else if (!std::isfinite(b_std)) prob = ndtr(-a_std);
    else prob = ndtr(b_std) - ndtr(a_std);
    if (prob < 1e-15) {
        if (std::isfinite(a) && !std::isfinite(b)) return a + sig;
        if (!std::isfinite(a) && std::isfinite(b)) return b - sig;
        if (std::isfinite(a) && std::isfinite(b)) return (a + b) / 2.0;
        return 0.0;
    }
    const double pdf_diff = norm_pdf(a_std) - norm_pdf(b_std);
    return sig * pdf_diff / prob;
}

// MSE-optimal centroids of `bits` for N(0, 1/n) (the reference's _optimal_centroids_torch).
std::vector<float> optimal_centroids(int bits, int n) {
    const int nc = 1 << bits;
    if (bits == 1) {
        const double c = std::sqrt(2.0 / (M_PI * n));
        return {(float)-c, (float)c};
    }
    if (bits == 2) {
        const double s = std::sqrt((double)n);
        return {(float)(-1.51 / s), (float)(-0.453 / s), (float)(0.453 / s), (float)(1.51 / s)};
    }
    const double sigma = 1.0 / std::sqrt((double)n);
    std::vector<double> bnd(nc - 1), cen(nc);
    const double step = 1.0 / nc;
    for (int i = 1; i < nc; ++i) bnd[i - 1] = ndtri(i * step) * sigma;
    const double inf = INFINITY;
    auto refresh = [&]() {
        cen[0] = cond_exp(sigma, -inf, bnd[0]);
        for (int i = 1; i < nc - 1; ++i) cen[i] = cond_exp(sigma, bnd[i - 1], bnd[i]);
        cen[nc - 1] = cond_exp(sigma, bnd[nc - 2], inf);
    };
    refresh();
    for (int it = 0; it < 100; ++it) {
        for (int i = 0; i < nc - 1; ++i) bnd[i] = (cen[i] + cen[i + 1]) / 2.0;
        refresh();
    }
    std::sort(cen.begin(), cen.end());
    std::vector<float> out(nc);
    for (int i = 0; i < nc; ++i) out[i] = (float)cen[i];
    return out;
}

}  // namespace builder
}  // namespace bgtq

using namespace bgtq;

extern "C" {

bgtq_status bgtq_haar_rotation(uint32_t n, uint64_t seed, float *out) {
    if (!out || n < 1 || n > 256) {
        set_last_error("bgtq_haar_rotation: invalid size");
        return BGTQ_EINVAL;
    }
    builder::haar_rotation((int)n, seed, out);
    return BGTQ_OK;
}

bgtq_status bgtq_optimal_centroids(uint32_t bits, uint32_t n, float *out) {
    if (!out || bits < 1 || bits > 8 || n < 1) {
        set_last_error("bgtq_optimal_centroids: invalid bit width or dimension");
        return BGTQ_EINVAL;
    }
    const std::vector<float> c = builder::optimal_centroids((int)bits, (int)n);
    std::memcpy(out, c.data(), c.size() * sizeof(float));
    return BGTQ_OK;
}

bgtq_status bgtq_tables_build(uint32_t dim, const int64_t *widths, const int64_t *pair_order,
                              uint32_t rotation_threshold, uint32_t row_pad, uint32_t norm_stride, uint32_t *config,
                              size_t config_capacity, size_t *config_len, float *table, size_t table_capacity,
                              size_t *table_len) {
    if (!widths || !config_len || !table_len || dim < 2 || dim > 128 || dim % 2) {
        set_last_error("bgtq_tables_build: invalid arguments");
        return BGTQ_EINVAL;
    }
    const int L = (int)dim / 2, hd = (int)dim;
    for (int i = 0; i < L; ++i)
        if (widths[i] < 1 || widths[i] > 8) {
            set_last_error("bgtq_tables_build: widths must be 1..8");
            return BGTQ_EINVAL;
        }
    // pairs ordered by width; position 2p / 2p+1 <- dims f / f + L of pair f.  The order of
    // equal widths is the reference's torch.argsort (not stable): torch's CPU sort runs
    // std::sort over (key, index) pairs compared by key, which is what this does.
    std::vector<std::pair<int64_t, int64_t>> kv(L);
    for (int i = 0; i < L; ++i) kv[i] = {widths[i], i};
    std::sort(kv.begin(), kv.end(),
              [](const std::pair<int64_t, int64_t> &a, const std::pair<int64_t, int64_t> &b) { return a.first < b.first; });
    std::vector<int> order(L);
    for (int i = 0; i < L; ++i) order[i] = (int)kv[i].second;
    if (pair_order) {  // a given order (e.g. an existing calibration's): a width-sorted permutation
        std::vector<char> seen(L, 0);
        for (int i = 0; i < L; ++i) {
            const int64_t f = pair_order[i];
            if (f < 0 || f >= L || seen[f] || (i && widths[f] < widths[order[i - 1]])) {
                set_last_error("bgtq_tables_build: pair_order must be a width-ascending permutation");
                return BGTQ_EINVAL;
            }
            seen[f] = 1;
            order[i] = (int)f;
        }
    }
    std::vector<uint32_t> perm(hd), group_of(hd);
    std::vector<int> bits_sorted(L);
    for (int p = 0; p < L; ++p) {
        perm[2 * p] = (uint32_t)order[p];
        perm[2 * p + 1] = (uint32_t)(order[p] + L);
        bits_sorted[p] = (int)widths[order[p]];
    }
    // one group per width present, in ascending width
    std::vector<int> gbits, gstart, gend;
    for (int p = 0; p < L; ++p) {
        if (gbits.empty() || gbits.back() != bits_sorted[p]) {
            gbits.push_back(bits_sorted[p]);
            gstart.push_back(2 * p);
            gend.push_back(2 * p);
        }
        gend.back() = 2 * p + 2;
    }
    const int ng = (int)gbits.size();
    if (ng > kMaxGroups) {
        set_last_error("bgtq_tables_build: more than 8 width classes");
        return BGTQ_EINVAL;
    }
    int maxc = 2;
    for (int b : gbits) maxc = std::max(maxc, 1 << b);
    std::vector<float> rot((size_t)hd * hd, 0.0f), cent((size_t)hd * maxc, 0.0f), bnd((size_t)hd * (maxc - 1), INFINITY);
    for (int g = 0; g < ng; ++g) {
        const int s = gstart[g], e = gend[g], n = e - s;
        group_of.resize(hd);
        for (int j = s; j < e; ++j) group_of[j] = (uint32_t)g;
        if (gbits[g] < (int)rotation_threshold) {
            for (int j = s; j < e; ++j) rot[(size_t)j * hd + j] = 1.0f;
        } else {
            std::vector<float> q((size_t)n * n);
            builder::haar_rotation(n, 42u + (uint64_t)gbits[g], q.data());
            for (int r = 0; r < n; ++r)
                for (int c = 0; c < n; ++c) rot[(size_t)(s + r) * hd + s + c] = q[(size_t)r * n + c];
        }
        const std::vector<float> c = builder::optimal_centroids(gbits[g], n);
        for (int j = s; j < e; ++j) {
            for (size_t k = 0; k < c.size(); ++k) cent[(size_t)j * maxc + k] = c[k];
            for (size_t k = 0; k + 1 < c.size(); ++k) bnd[(size_t)j * (maxc - 1) + k] = (c[k] + c[k + 1]) / 2.0f;
        }
    }
    // build_code_lut: per-position offsets / inverse scales; codebooks by centroid signature
    std::vector<float> off(hd), inv(hd);
    std::vector<uint32_t> pos_to_cb(hd);
    std::map<std::vector<float>, uint32_t> sig;
    std::vector<int> reps;
    for (int j = 0; j < hd; ++j) {
        int nvb = 0;
        for (int k = 0; k < maxc - 1; ++k) nvb += bnd[(size_t)j * (maxc - 1) + k] < 1e30f ? 1 : 0;
        const int nc = std::max(nvb + 1, 2);
        const float *cj = &cent[(size_t)j * maxc];
        double cmin = cj[0], cmax = cj[0];
        for (int k = 1; k < nc; ++k) { cmin = std::min(cmin, (double)cj[k]); cmax = std::max(cmax, (double)cj[k]); }
        const double spacing = (cmax - cmin) / std::max(nc - 1, 1), margin = spacing * 0.5;
        const double rmin = cmin - margin, rmax = cmax + margin, bw = (rmax - rmin) / 256;
        off[j] = (float)rmin;
        inv[j] = (float)(1.0 / bw);
        std::vector<float> key(cj, cj + nc);
        key.push_back((float)nc);
        auto it = sig.find(key);
        if (it == sig.end()) {
            it = sig.emplace(key, (uint32_t)reps.size()).first;
            reps.push_back(j);
        }
        pos_to_cb[j] = it->second;
    }
    std::vector<uint32_t> lut(reps.size() * 256);
    for (size_t cb = 0; cb < reps.size(); ++cb) {
        const int j = reps[cb];
        int nvb = 0;
        for (int k = 0; k < maxc - 1; ++k) nvb += bnd[(size_t)j * (maxc - 1) + k] < 1e30f ? 1 : 0;
        const int nc = std::max(nvb + 1, 2);
        const float *cj = &cent[(size_t)j * maxc];
        double cmin = cj[0], cmax = cj[0];
        for (int k = 1; k < nc; ++k) { cmin = std::min(cmin, (double)cj[k]); cmax = std::max(cmax, (double)cj[k]); }
        const double spacing = (cmax - cmin) / std::max(nc - 1, 1), margin = spacing * 0.5;
        const double rmin = cmin - margin, rmax = cmax + margin, bw = (rmax - rmin) / 256;
        // torch.linspace(rmin + bw/2, rmax - bw/2, 256) in FP32
        const float s0 = (float)(rmin + bw / 2), s1 = (float)(rmax - bw / 2);
        const float stp = (s1 - s0) / 255.0f;
        const float *bj = &bnd[(size_t)j * (maxc - 1)];
        for (int i = 0; i < 256; ++i) {
            const float x = i < 128 ? std::fmaf(stp, (float)i, s0) : std::fmaf(-stp, (float)(255 - i), s1);
            uint32_t idx;
            if (nvb > 0) {
                idx = (uint32_t)(std::lower_bound(bj, bj + nvb, x) - bj);  // first boundary >= x
                idx = std::min(idx, (uint32_t)(nc - 1));
            } else {
                const float mid = (cj[0] + cj[1]) / 2.0f;
                idx = x > mid ? 1u : 0u;
            }
            lut[cb * 256 + i] = idx;
        }
    }
    // build_pack_meta: widths >= 5 are raw bytes, the rest nibbles
    int ns = hd, nl = 0;
    for (int j = 0; j < hd; ++j)
        if (bits_sorted[j / 2] >= 5) {
            if (ns == hd) ns = j;
            ++nl;
        }
    const uint32_t row_bytes = (uint32_t)(ns / 2 + nl) + row_pad;
    const uint32_t nstride = norm_stride ? norm_stride : (uint32_t)ng;
    if (nstride < (uint32_t)ng) {
        set_last_error("bgtq_tables_build: norm_stride below the group count");
        return BGTQ_EINVAL;
    }
    // flatten (layout.ts:24-31)
    std::vector<uint32_t> cfg = {dim, (uint32_t)ng, row_bytes, nstride, (uint32_t)ns, (uint32_t)maxc, 0, 0, 0, 0};
    const std::vector<uint32_t> *parts[4] = {&perm, &group_of, &pos_to_cb, &lut};
    for (int k = 0; k < 4; ++k) {
        cfg[6 + k] = (uint32_t)cfg.size();
        cfg.insert(cfg.end(), parts[k]->begin(), parts[k]->end());
    }
    std::vector<float> tab;
    tab.reserve(rot.size() + cent.size() + 2 * hd);
    tab.insert(tab.end(), rot.begin(), rot.end());
    tab.insert(tab.end(), cent.begin(), cent.end());
    tab.insert(tab.end(), off.begin(), off.end());
    tab.insert(tab.end(), inv.begin(), inv.end());
    *config_len = cfg.size();
    *table_len = tab.size();
    if (!config || !table) return BGTQ_OK;  // size query
    if (config_capacity < cfg.size() || table_capacity < tab.size()) {
        set_last_error("bgtq_tables_build: output buffers too small");
        return BGTQ_EINVAL;
    }
    std::memcpy(config, cfg.data(), cfg.size() * sizeof(uint32_t));
    std::memcpy(table, tab.data(), tab.size() * sizeof(float));
    return BGTQ_OK;
}

}  // extern "C"
