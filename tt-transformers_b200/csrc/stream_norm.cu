// Norm kernels around the float32 residual stream that the plain add_rmsnorm does not cover.
//
// stream_add_norm: residual[r, :] += d1[r, :] + d2[r, :] + vec[:] (each optional; d1 and d2 float32 or bfloat16 by
//   themselves; vec float32, the same for every row), then, with a weight, out = residual / sqrt(mean(residual^2) +
//   eps) * (offset + w) in the output type (offset 1 for weights stored around zero). Without a weight nothing is
//   normed (the kernel is then the addition alone). One block per row; the summed row waits in shared memory.
// gated_rmsnorm: out = x / sqrt(mean(x^2) + eps) * w * sigmoid(gate), x float32, gate of the compute type with a row
//   stride of its own (a slice of a wider product).
// mean_rmsnorm_pair: out = (rms(a) * wa + rms(b) * wb) / 2 in float32, a and b of the compute type.
// All sums, means and scalings are float32; 1 / sqrt by the correctly rounded sqrtf and a division.
#include "common.cuh"

#define SN_THREADS 256

__device__ __forceinline__ float sn_load(const void* p, int dtype, size_t i) {
    return dtype == TTB_DTYPE_F32 ? reinterpret_cast<const float*>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void sn_store(void* p, int dtype, size_t i, float v) {
    if (dtype == TTB_DTYPE_F32) reinterpret_cast<float*>(p)[i] = v;
    else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__global__ void __launch_bounds__(SN_THREADS)
stream_add_norm_kernel(float* __restrict__ residual, const void* __restrict__ d1, int d1_dtype, const void* __restrict__ d2,
                       int d2_dtype, const float* __restrict__ vec, const void* __restrict__ weight, int w_dtype,
                       float offset, float eps, void* __restrict__ out, int out_dtype, int width) {
    extern __shared__ float sn_row[];
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const size_t base = (size_t)blockIdx.x * width;
    const bool adds = d1 != nullptr || d2 != nullptr || vec != nullptr;
    float sumsq = 0.f;
    for (int c = threadIdx.x; c < width; c += SN_THREADS) {
        float v = residual[base + c];
        if (adds) {
            float d = 0.f;
            if (d1 != nullptr) d = sn_load(d1, d1_dtype, base + c);
            if (d2 != nullptr) d += sn_load(d2, d2_dtype, base + c);
            if (vec != nullptr) d += vec[c];
            v += d;
            residual[base + c] = v;
        }
        sn_row[c] = v;
        sumsq += v * v;
    }
    if (out == nullptr) return;
    sumsq = block_sum(sumsq, scratch);
    const float scale = 1.f / sqrtf(sumsq / (float)width + eps);
    for (int c = threadIdx.x; c < width; c += SN_THREADS)
        sn_store(out, out_dtype, base + c, sn_row[c] * scale * (offset + sn_load(weight, w_dtype, c)));
}

TTB_EXPORT int ttb_stream_add_norm(float* residual, const void* d1, int d1_dtype, const void* d2, int d2_dtype, const float* vec,
                                   const void* weight, int w_dtype, float offset, float eps, void* out, int out_dtype,
                                   int rows, int width, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!residual || width < 1 || ((out != nullptr) != (weight != nullptr))) return TTB_ERR_ARGUMENT;
    const size_t smem = (size_t)width * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    ttb_launch(stream_add_norm_kernel, rows, SN_THREADS, smem, stream, residual, d1, d1_dtype, d2, d2_dtype, vec, weight,
               w_dtype, offset, eps, out, out_dtype, width);
    return ttb_launch_status();
}

__global__ void __launch_bounds__(SN_THREADS)
gated_rmsnorm_kernel(const float* __restrict__ x, const void* __restrict__ gate, int gate_dtype, int gate_stride,
                     const float* __restrict__ weight, float eps, void* __restrict__ out, int out_dtype, int width) {
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const size_t base = (size_t)blockIdx.x * width;
    float sumsq = 0.f;
    for (int c = threadIdx.x; c < width; c += SN_THREADS) {
        const float v = x[base + c];
        sumsq += v * v;
    }
    sumsq = block_sum(sumsq, scratch);
    const float scale = 1.f / sqrtf(sumsq / (float)width + eps);
    for (int c = threadIdx.x; c < width; c += SN_THREADS) {
        const float g = sn_load(gate, gate_dtype, (size_t)blockIdx.x * gate_stride + c);
        sn_store(out, out_dtype, base + c, x[base + c] * scale * weight[c] / (1.f + expf(-g)));
    }
}

TTB_EXPORT int ttb_gated_rmsnorm(const float* x, const void* gate, int gate_dtype, int gate_stride, const float* weight,
                                 float eps, void* out, int out_dtype, int rows, int width, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!x || !gate || !weight || !out || width < 1) return TTB_ERR_ARGUMENT;
    ttb_launch(gated_rmsnorm_kernel, rows, SN_THREADS, 0, stream, x, gate, gate_dtype, gate_stride, weight, eps, out, out_dtype, width);
    return ttb_launch_status();
}

__global__ void __launch_bounds__(SN_THREADS)
mean_rmsnorm_pair_kernel(const void* __restrict__ a, const void* __restrict__ b, int dtype, const float* __restrict__ wa,
                         const float* __restrict__ wb, float eps, float* __restrict__ out, int width) {
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const size_t base = (size_t)blockIdx.x * width;
    float sa = 0.f, sb = 0.f;
    for (int c = threadIdx.x; c < width; c += SN_THREADS) {
        const float va = sn_load(a, dtype, base + c), vb = sn_load(b, dtype, base + c);
        sa += va * va;
        sb += vb * vb;
    }
    sa = block_sum(sa, scratch);
    sb = block_sum(sb, scratch);
    const float ka = 1.f / sqrtf(sa / (float)width + eps), kb = 1.f / sqrtf(sb / (float)width + eps);
    for (int c = threadIdx.x; c < width; c += SN_THREADS)
        out[base + c] = 0.5f * (sn_load(a, dtype, base + c) * ka * wa[c] + sn_load(b, dtype, base + c) * kb * wb[c]);
}

TTB_EXPORT int ttb_mean_rmsnorm_pair(const void* a, const void* b, int dtype, const float* wa, const float* wb, float eps,
                                     float* out, int rows, int width, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!a || !b || !wa || !wb || !out || width < 1) return TTB_ERR_ARGUMENT;
    ttb_launch(mean_rmsnorm_pair_kernel, rows, SN_THREADS, 0, stream, a, b, dtype, wa, wb, eps, out, width);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- activations on a product's output
// kind 0: silu(g) * u, 1: gelu_tanh(g) * u, 4: relu(g) * u over [rows, gate | up] -> [rows, cols]; 2: relu(z)^2, 3: the erf GELU over [rows, cols].
__device__ __forceinline__ float gelu_tanh(float z) {
    return 0.5f * z * (1.f + tanhf(0.7978845608028654f * (z + 0.044715f * z * z * z)));
}

__global__ void activation_kernel(const void* __restrict__ in, int in_dtype, int in_stride, void* __restrict__ out, int out_dtype,
                                  int rows, int cols, int kind) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)rows * cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        const float g = sn_load(in, in_dtype, r * in_stride + c);
        float v;
        if (kind == 2) {
            const float p = fmaxf(g, 0.f);
            v = p * p;
        } else if (kind == 3) {                       // the exact GELU: 0.5 z (1 + erf(z / sqrt 2))
            v = 0.5f * g * (1.f + erff(g * 0.70710678118654752f));
        } else {
            const float u = sn_load(in, in_dtype, r * in_stride + cols + c);
            v = (kind == 0 ? g / (1.f + expf(-g)) : (kind == 4 ? fmaxf(g, 0.f) : gelu_tanh(g))) * u;
        }
        sn_store(out, out_dtype, i, v);
    }
}

TTB_EXPORT int ttb_activation(const void* in, int in_dtype, int in_stride, void* out, int out_dtype, int rows, int cols, int kind,
                              cudaStream_t stream) {
    if (rows == 0 || cols == 0) return TTB_OK;
    if (!in || !out || kind < 0 || kind > 4) return TTB_ERR_ARGUMENT;
    const size_t total = (size_t)rows * cols;
    const int blocks = (int)((total + 255) / 256 > 148 * 16 ? 148 * 16 : (total + 255) / 256);
    ttb_launch(activation_kernel, blocks, 256, 0, stream, in, in_dtype, in_stride, out, out_dtype, rows, cols, kind);
    return ttb_launch_status();
}
