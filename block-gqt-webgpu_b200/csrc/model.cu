// Decode-step kernels of the model path (batch of a few sequences, one token each): the
// reference's per-token matmul / RMSNorm / SiLU-gate shaders (src/model/kernels.wgsl:11-54,
// driven by src/model/decoder.ts:31-81) fused into weight-streaming GEMVs.
//
// A decode step reads every weight once for a handful of activation rows, so these are
// HBM-latency kernels: FP16 weights (the checkpoint's precision, converted to FP32 in
// registers; FP32 arithmetic throughout, as the reference's shaders compute) streamed with
// 16-byte loads, each warp owning whole output rows and issuing all of its loads before
// the first FMA.  The activation rows sit in shared memory; when the layer's RMSNorm comes
// first, every CTA computes it in its prologue (a few hundred floats from L2), so no
// separate normalisation launch and no normalised copy in global memory are needed.
//   GEMV_NORM         y[b][r]  = W[r] . rmsnorm(x[b]) (+ bias[r])        Q/K/V, lm_head
//   GEMV_RESIDUAL     y[b][r] += W[r] . x[b]                            o_proj, down_proj
//   GEMV_NORM_SILU    y[b][r]  = silu(W[r] . n) * (W[out + r] . n)      gate/up, n = rmsnorm(x[b])
#include <cuda_fp16.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxBatch = 8;
constexpr int kChunks = 4;      // 16-byte weight chunks per lane and row in flight per pass

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// FP16 x 8 (one 16-byte chunk) dotted with 8 FP32 activations.
__device__ __forceinline__ float dot8(const uint4 w, const float *x) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        acc = fmaf(f.x, x[2 * k], acc);
        acc = fmaf(f.y, x[2 * k + 1], acc);
    }
    return acc;
}

template <int MODE, int B, int RPW>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const float *__restrict__ x, uint64_t x_stride, uint32_t in,
                                                            const float *__restrict__ norm_w, float eps,
                                                            const __half *__restrict__ w, const float *__restrict__ bias,
                                                            uint32_t out, float *y, uint64_t y_stride) {
    extern __shared__ __align__(16) float xs[];       // [B][in] activations (normalised for the NORM modes)
    __shared__ float red[kGemvWarps][B];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t chunks = in / 8;
    const uint32_t r0 = (blockIdx.x * kGemvWarps + warp) * RPW;
    constexpr int NW = MODE == 2 ? 2 : 1;   // gate and up rows
    // the weights do not depend on the kernel before this one: their first pass is loaded
    // while that kernel finishes (programmatic launch), the activations after the wait
    uint4 wv[RPW][NW][kChunks];
    auto load_pass = [&](uint32_t base) {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int u = 0; u < NW; ++u)
#pragma unroll
                for (int c = 0; c < kChunks; ++c) {
                    const uint32_t row = r0 + r, ch = base + lane + 32u * c;
                    wv[r][u][c] = row < out && ch < chunks
                                      ? __ldg(reinterpret_cast<const uint4 *>(w + (uint64_t)(row + u * out) * in) + ch)
                                      : make_uint4(0, 0, 0, 0);
                }
    };
    load_pass(0);
    pdl_wait();
    pdl_trigger();
    // ---- the activation rows into shared memory (and their RMSNorm) ----
    for (uint32_t e = tid; e < (uint32_t)B * in; e += kGemvThreads) {
        const uint32_t b = e / in, i = e - b * in;
        xs[e] = x[b * x_stride + i];
    }
    __syncthreads();
    if (MODE != 1) {
        float ss[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float s = 0.0f;
            for (uint32_t i = tid; i < in; i += kGemvThreads) s = fmaf(xs[b * in + i], xs[b * in + i], s);
            ss[b] = warp_sum(s);
        }
        if (lane == 0)
#pragma unroll
            for (int b = 0; b < B; ++b) red[warp][b] = ss[b];
        __syncthreads();
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < kGemvWarps; ++k) s += red[k][b];
            ss[b] = rsqrtf(s / (float)in + eps);
        }
#pragma unroll
        for (int b = 0; b < B; ++b)
            for (uint32_t i = tid; i < in; i += kGemvThreads) xs[b * in + i] = xs[b * in + i] * ss[b] * norm_w[i];
        __syncthreads();
    }
    // ---- rows: each pass has kChunks weight chunks per lane and row in flight, then the dots ----
    float acc[RPW][NW][B];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int u = 0; u < NW; ++u)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][u][b] = 0.0f;
    for (uint32_t base = 0; base < chunks; base += 32u * kChunks) {
        if (base) load_pass(base);
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const uint32_t ch = base + lane + 32u * c;
            if (ch < chunks) {
#pragma unroll
                for (int r = 0; r < RPW; ++r)
#pragma unroll
                    for (int u = 0; u < NW; ++u)
#pragma unroll
                        for (int b = 0; b < B; ++b) acc[r][u][b] += dot8(wv[r][u][c], xs + b * in + 8u * ch);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const uint32_t row = r0 + r;
#pragma unroll
        for (int u = 0; u < NW; ++u)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][u][b] = warp_sum(acc[r][u][b]);
        if (lane == 0 && row < out) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float v = acc[r][0][b];
                if constexpr (MODE == 0) {
                    y[b * y_stride + row] = bias ? v + bias[row] : v;
                } else if constexpr (MODE == 1) {
                    y[b * y_stride + row] += v;
                } else {
                    y[b * y_stride + row] = v / (1.0f + expf(-v)) * acc[r][NW - 1][b];
                }
            }
        }
    }
}

template <int MODE, int B>
cudaError_t run_gemv(const float *x, uint64_t xs, uint32_t in, const float *nw, float eps, const __half *w,
                     const float *bias, uint32_t out, float *y, uint64_t ys, cudaStream_t s) {
    // one output row per warp covers the SMs for the layer matrices; the long lm_head takes
    // four rows per warp (more loads in flight per warp, fewer CTAs)
    const size_t smem = sizeof(float) * (size_t)B * in;
    if (smem > 48u * 1024u) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MODE, B, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_kernel<MODE, B, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    if (out >= 16384u) {
        const uint32_t per = kGemvWarps * 4;
        return launch_pdl(gemv_kernel<MODE, B, 4>, dim3((out + per - 1) / per), dim3(kGemvThreads), smem, s, x, xs, in,
                          nw, eps, w, bias, out, y, ys);
    }
    const uint32_t per = kGemvWarps;
    return launch_pdl(gemv_kernel<MODE, B, 1>, dim3((out + per - 1) / per), dim3(kGemvThreads), smem, s, x, xs, in, nw,
                      eps, w, bias, out, y, ys);
}

template <int MODE>
cudaError_t dispatch_batch(uint32_t batch, const float *x, uint64_t xs, uint32_t in, const float *nw, float eps,
                           const __half *w, const float *bias, uint32_t out, float *y, uint64_t ys, cudaStream_t s) {
    switch (batch) {
        case 1: return run_gemv<MODE, 1>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 2: return run_gemv<MODE, 2>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 3: return run_gemv<MODE, 3>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 4: return run_gemv<MODE, 4>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 5: return run_gemv<MODE, 5>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 6: return run_gemv<MODE, 6>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        case 7: return run_gemv<MODE, 7>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
        default: return run_gemv<MODE, 8>(x, xs, in, nw, eps, w, bias, out, y, ys, s);
    }
}

}  // namespace
}  // namespace bgtq

extern "C" bgtq_status bgtq_model_gemv(int mode, const float *x, uint32_t batch, uint64_t x_stride, uint32_t in,
                                       const float *norm_w, float eps, const uint16_t *w, const float *bias,
                                       uint32_t out, float *y, uint64_t y_stride, void *stream) {
    using namespace bgtq;
    if (mode < 0 || mode > 2 || !x || !w || !y || batch < 1 || batch > (uint32_t)kMaxBatch || in < 8 || in % 8 ||
        (uint64_t)batch * in * sizeof(float) > 200u * 1024u || out < 1 || (mode != 1 && !norm_w) || x_stride < in ||
        y_stride < out || (reinterpret_cast<uintptr_t>(w) & 15u)) {
        set_last_error("Invalid model GEMV shape");
        return BGTQ_EINVAL;
    }
    const __half *wh = reinterpret_cast<const __half *>(w);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e =
        mode == 0   ? dispatch_batch<0>(batch, x, x_stride, in, norm_w, eps, wh, bias, out, y, y_stride, s)
        : mode == 1 ? dispatch_batch<1>(batch, x, x_stride, in, norm_w, eps, wh, bias, out, y, y_stride, s)
                    : dispatch_batch<2>(batch, x, x_stride, in, norm_w, eps, wh, bias, out, y, y_stride, s);
    if (e != cudaSuccess) {
        set_last_error(std::string("model GEMV launch: ") + cudaGetErrorString(e));
        return BGTQ_ECUDA;
    }
    return BGTQ_OK;
}
