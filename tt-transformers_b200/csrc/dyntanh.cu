// Dynamic Tanh around sub-layers, fused with the residual add, and the operand of a pass's mixing product.
//
// add_dyntanh: x += mult * (after ? tanh(a_alpha d) * a_w + a_b : d)   (d optional, float32 or bfloat16; x float32, in place)
//              out = tanh(alpha x) * w + b                             (optional, float32 or bfloat16)
// Every element by itself: no row statistic, so the kernel is one pass over the stream (read, add, write, norm).
// Accurate tanhf; everything in float32. One launch per sub-layer boundary.
// concat_cast: out[t] = [a[t] | b[t]] for two float32 [rows, width] tensors, in the output's type.
#include "common.cuh"

__device__ __forceinline__ float dt_load(const void* p, int dtype, size_t i) {
    return dtype == TTB_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                                   : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void dt_store(void* p, int dtype, size_t i, float v) {
    if (dtype == TTB_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}

// four columns a thread; `width` a multiple of 4 takes 16-byte loads of the stream and of the weight vectors
template <bool VEC>
__global__ void __launch_bounds__(256)
add_dyntanh_kernel(float* __restrict__ x, const void* __restrict__ delta, int delta_dtype, int delta_stride,
                   const float* __restrict__ a_w, const float* __restrict__ a_b, float a_alpha, float mult,
                   const float* __restrict__ n_w, const float* __restrict__ n_b, float n_alpha, void* __restrict__ out,
                   int out_dtype, int rows, int width) {
    pdl_wait();
    pdl_launch_dependents();
    const int quads = (width + 3) / 4;
    const size_t total = (size_t)rows * quads;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / quads;
        const int c0 = (int)(i % quads) * 4;
        float v[4];
        const int n = min(4, width - c0);
        if (VEC) {
            const float4 q = *reinterpret_cast<const float4*>(x + r * width + c0);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        } else {
            for (int j = 0; j < n; ++j) v[j] = x[r * width + c0 + j];
        }
        if (delta != nullptr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j >= n) break;
                float d = dt_load(delta, delta_dtype, r * delta_stride + c0 + j);
                if (a_w != nullptr) d = tanhf(a_alpha * d) * a_w[c0 + j] + a_b[c0 + j];
                v[j] = fmaf(mult, d, v[j]);
            }
            if (VEC) *reinterpret_cast<float4*>(x + r * width + c0) = make_float4(v[0], v[1], v[2], v[3]);
            else for (int j = 0; j < n; ++j) x[r * width + c0 + j] = v[j];
        }
        if (out != nullptr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j >= n) break;
                dt_store(out, out_dtype, r * width + c0 + j, tanhf(n_alpha * v[j]) * n_w[c0 + j] + n_b[c0 + j]);
            }
        }
    }
}

TTB_EXPORT int ttb_add_dyntanh(float* x, const void* delta, int delta_dtype, int delta_stride, const float* after_w,
                               const float* after_b, float after_alpha, float mult, const float* norm_w, const float* norm_b,
                               float norm_alpha, void* out, int out_dtype, int rows, int width, cudaStream_t stream) {
    if (rows == 0 || width == 0) return TTB_OK;
    if (!x || (after_w && !after_b) || (out && (!norm_w || !norm_b))) return TTB_ERR_ARGUMENT;
    if (delta == nullptr && out == nullptr) return TTB_OK;
    const size_t total = (size_t)rows * ((width + 3) / 4);
    const int blocks = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
    const bool vec = (width & 3) == 0 && aligned16(x);
    if (vec)
        ttb_launch(add_dyntanh_kernel<true>, blocks, 256, 0, stream, x, delta, delta_dtype, delta_stride, after_w, after_b,
                   after_alpha, mult, norm_w, norm_b, norm_alpha, out, out_dtype, rows, width);
    else
        ttb_launch(add_dyntanh_kernel<false>, blocks, 256, 0, stream, x, delta, delta_dtype, delta_stride, after_w, after_b,
                   after_alpha, mult, norm_w, norm_b, norm_alpha, out, out_dtype, rows, width);
    return ttb_launch_status();
}

__global__ void __launch_bounds__(256)
concat_cast_kernel(const float* __restrict__ a, const float* __restrict__ b, void* __restrict__ out, int out_dtype, int rows,
                   int width) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)rows * 2 * width;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / (2 * width);
        const int c = (int)(i % (2 * width));
        dt_store(out, out_dtype, i, c < width ? a[r * width + c] : b[r * width + c - width]);
    }
}

TTB_EXPORT int ttb_concat_cast(const float* a, const float* b, void* out, int out_dtype, int rows, int width,
                               cudaStream_t stream) {
    if (rows == 0 || width == 0) return TTB_OK;
    if (!a || !b || !out) return TTB_ERR_ARGUMENT;
    const size_t total = (size_t)rows * 2 * width;
    const int blocks = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
    ttb_launch(concat_cast_kernel, blocks, 256, 0, stream, a, b, out, out_dtype, rows, width);
    return ttb_launch_status();
}
