// Row appends for the FP16 key store and the value stores, and the test/debug
// reconstruction of FP32 keys from packed rows.
//
//   copy_rows   FP16Keys.append (src/runtime/keys.ts:24-26), Values.append
//               (src/runtime/values.ts:9-14) and the model's FP32 -> FP16 V append
//               (src/model/append.wgsl:6-10, RNE via __float2half_rn = half.wgsl:2-12).
//   reconstruct CompressedKeys.prepare / mixed.wgsl:43-56: k[perm[j]] = sum_i
//               cent[i][code_i] * scale_{g(i)} * R[i][j], sequential FMA in ascending i,
//               the same order as the CPU oracle (compiled with -fmad=false).
#include <cuda_fp16.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace {

// swizzle: FP16 rows of 64 or 128 halves store 16-byte chunk c of row t at chunk
// (c & ~7) | ((c ^ t) & 7), so that a tile of rows copied verbatim into shared memory can
// be read column-wise (ldmatrix) without bank conflicts.
__global__ void copy_rows_kernel(void *dst, uint64_t dst_seq_stride, uint32_t dst_row_elems, int dst_f32,
                                 const void *src, uint64_t src_row_stride, uint64_t src_seq_stride, int src_f32,
                                 const uint32_t *row0, uint32_t row0_scalar, uint32_t count, uint32_t seq_first,
                                 uint32_t seq_count, uint32_t d, uint32_t *lengths, int swizzle) {
    const uint64_t total = (uint64_t)seq_count * count * d;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t e = (uint32_t)(i % d);
        const uint64_t rowi = i / d;
        const uint32_t r = (uint32_t)(rowi % count), s = (uint32_t)(rowi / count);
        const uint64_t si = (uint64_t)s * src_seq_stride + (uint64_t)r * src_row_stride + e;
        const uint32_t drow = (row0 ? row0[s] : row0_scalar) + r;
        uint32_t de = e;
        if (swizzle) {
            const uint32_t c = e >> 3;
            de = (((c & ~7u) | ((c ^ drow) & 7u)) << 3) | (e & 7u);
        }
        const uint64_t di = (uint64_t)(seq_first + s) * dst_seq_stride + (uint64_t)drow * dst_row_elems + de;
        if (dst_f32) {
            const float v = src_f32 ? static_cast<const float *>(src)[si]
                                    : __half2float(__ushort_as_half(static_cast<const uint16_t *>(src)[si]));
            static_cast<float *>(dst)[di] = v;
        } else {
            const uint16_t v = src_f32 ? __half_as_ushort(__float2half_rn(static_cast<const float *>(src)[si]))
                                       : static_cast<const uint16_t *>(src)[si];
            static_cast<uint16_t *>(dst)[di] = v;
        }
    }
    if (blockIdx.x == 0 && lengths) {
        for (uint32_t s = threadIdx.x; s < seq_count; s += blockDim.x)
            lengths[seq_first + s] = (row0 ? row0[s] : row0_scalar) + count;
    }
}

template <int D>
__global__ void __launch_bounds__(128) reconstruct_kernel(const __grid_constant__ ReconArgs a, uint32_t n_cent) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *rt_s = reinterpret_cast<float *>(smem);  // [D][D]: rt_s[j][i] = R[i][j]
    float *cent_s = rt_s + D * D;
    const uint32_t d = a.d;
    for (uint32_t k = threadIdx.x; k < (uint32_t)(D * D); k += blockDim.x) {
        const uint32_t j = k / D, i = k % D;
        rt_s[k] = (i < d && j < d) ? a.t.rot[i * d + j] : 0.0f;
    }
    for (uint32_t k = threadIdx.x; k < n_cent; k += blockDim.x) cent_s[k] = a.t.cent[k];
    __syncthreads();
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.rows) return;
    const uint8_t *row = a.packed + (uint64_t)r * a.row_stride;
    const uint16_t *sc = a.scales + (uint64_t)r * a.scale_stride;
    float val[D];
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float v = 0.0f;
        if ((uint32_t)i < d) {
            uint32_t code;
            if ((uint32_t)i < a.ns) code = (row[i >> 1] >> ((i & 1) * 4)) & 15u;
            else code = row[(a.ns >> 1) + i - a.ns];
            v = cent_s[a.t.cb_base[i] + code] * __half2float(__ushort_as_half(sc[a.t.group_of[i]]));
        }
        val[i] = v;
    }
    for (uint32_t j = 0; j < d; ++j) {
        const float *cj = rt_s + j * D;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < D; i += 4) {
            const float4 c = *reinterpret_cast<const float4 *>(cj + i);
            acc = fmaf(val[i + 0], c.x, acc);
            acc = fmaf(val[i + 1], c.y, acc);
            acc = fmaf(val[i + 2], c.z, acc);
            acc = fmaf(val[i + 3], c.w, acc);
        }
        a.out[(uint64_t)r * d + a.t.perm[j]] = acc;
    }
}

template <int D>
cudaError_t run_reconstruct(const ReconArgs &a, uint32_t n_cent, cudaStream_t s) {
    const size_t smem = sizeof(float) * ((size_t)D * D + n_cent);
    cudaError_t e = cudaFuncSetAttribute(reconstruct_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const uint32_t blocks = (a.rows + 127) / 128;
    reconstruct_kernel<D><<<blocks, 128, smem, s>>>(a, n_cent);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_copy_rows(void *dst, uint64_t dst_seq_stride, uint32_t dst_row_elems, int dst_f32, const void *src,
                             uint64_t src_row_stride, uint64_t src_seq_stride, int src_f32, const uint32_t *row0,
                             uint32_t row0_scalar, uint32_t count, uint32_t seq_first, uint32_t seq_count,
                             uint32_t *lengths, uint32_t d, int swizzle, cudaStream_t s) {
    if (count == 0 || seq_count == 0) return cudaSuccess;
    const uint64_t total = (uint64_t)seq_count * count * d;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 148u * 16u) blocks = 148u * 16u;
    copy_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(dst, dst_seq_stride, dst_row_elems, dst_f32, src, src_row_stride,
                                                       src_seq_stride, src_f32, row0, row0_scalar, count, seq_first,
                                                       seq_count, d, lengths, swizzle);
    return cudaGetLastError();
}

cudaError_t launch_reconstruct(const ReconArgs &a, uint32_t n_cent, cudaStream_t s) {
    if (a.rows == 0) return cudaSuccess;
    if (a.d <= 16) return run_reconstruct<16>(a, n_cent, s);
    if (a.d <= 32) return run_reconstruct<32>(a, n_cent, s);
    if (a.d <= 64) return run_reconstruct<64>(a, n_cent, s);
    return run_reconstruct<128>(a, n_cent, s);
}

}  // namespace bgtq
