// Layer norm with weight and bias around sub-layers, fused with the residual add between them.
//   residual += mult * after(delta)      (after: a layer norm of the sub-layer's output; absent: delta itself)
//   out = norm(residual)                 (norm: the layer norm before the next sub-layer; absent: nothing is written)
// y = (x - mean) / sqrt(var + eps) * w + b, var = mean((x - mean)^2); the residual stream, both means, both
// variances and the scaling are float32. One block per row; the row stays in shared memory between the passes, so
// the variance is the mean of squared deviations from the exact mean (no E[x^2] - E[x]^2 cancellation).
#include "common.cuh"

#define LN_THREADS 256

__device__ __forceinline__ void ln_stats(const float* row, int width, float eps, float* scratch, float& mean, float& rstd) {
    float s = 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) s += row[c];
    mean = block_sum(s, scratch) / (float)width;
    float q = 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        const float d = row[c] - mean;
        q += d * d;
    }
    rstd = rsqrtf(block_sum(q, scratch) / (float)width + eps);
}

template <typename TD, typename TO>
__global__ void __launch_bounds__(LN_THREADS)
add_layernorm_kernel(float* __restrict__ residual, const TD* __restrict__ delta, int ld_delta,
                     const float* __restrict__ after_w, const float* __restrict__ after_b, float after_eps, float mult,
                     const float* __restrict__ norm_w, const float* __restrict__ norm_b, float norm_eps,
                     TO* __restrict__ out, int width) {
    extern __shared__ float row[];
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    float* res = residual + (size_t)blockIdx.x * width;
    if (delta != nullptr) {
        const TD* d = delta + (size_t)blockIdx.x * ld_delta;
        for (int c = threadIdx.x; c < width; c += blockDim.x) row[c] = to_float(d[c]);
        __syncthreads();
        float mean = 0.f, rstd = 1.f;
        if (after_w != nullptr) ln_stats(row, width, after_eps, scratch, mean, rstd);
        __syncthreads();
        for (int c = threadIdx.x; c < width; c += blockDim.x) {
            float y = row[c];
            if (after_w != nullptr) y = (y - mean) * rstd * after_w[c] + (after_b != nullptr ? after_b[c] : 0.f);
            const float v = res[c] + mult * y;
            res[c] = v;
            row[c] = v;
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) row[c] = res[c];
    }
    if (norm_w == nullptr) return;
    __syncthreads();
    float mean, rstd;
    ln_stats(row, width, norm_eps, scratch, mean, rstd);
    TO* o = out + (size_t)blockIdx.x * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x)
        o[c] = from_float<TO>((row[c] - mean) * rstd * norm_w[c] + (norm_b != nullptr ? norm_b[c] : 0.f));
}


// Rows of up to LN_THREADS * 8 elements (a multiple of 8): a thread keeps its eight values in registers through both
// norms, and the four weight vectors, which no kernel writes, are fetched before the wait for the kernel in front.
template <typename TD, typename TO>
__global__ void __launch_bounds__(LN_THREADS)
add_layernorm_regs_kernel(float* __restrict__ residual, const TD* __restrict__ delta, int ld_delta,
                          const float* __restrict__ after_w, const float* __restrict__ after_b, float after_eps, float mult,
                          const float* __restrict__ norm_w, const float* __restrict__ norm_b, float norm_eps,
                          TO* __restrict__ out, int width) {
    __shared__ float scratch[32];
    const int c = threadIdx.x * 8;
    const bool mine = c < width;
    float aw[8], ab[8], nw[8], nb[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) { aw[e] = 1.f; ab[e] = 0.f; nw[e] = 1.f; nb[e] = 0.f; }
    if (mine) {
        if (delta != nullptr && after_w != nullptr) {
            load8(after_w + c, aw);
            if (after_b != nullptr) load8(after_b + c, ab);
        }
        if (norm_w != nullptr) {
            load8(norm_w + c, nw);
            if (norm_b != nullptr) load8(norm_b + c, nb);
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    float* res = residual + (size_t)blockIdx.x * width;
    float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (mine) load8(res + c, r);
    const float inv_width = 1.f / (float)width;
    if (delta != nullptr) {
        float d[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (mine) load8(delta + (size_t)blockIdx.x * ld_delta + c, d);
        if (after_w != nullptr) {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) s += d[e];
            const float mean = block_sum(s, scratch) * inv_width;
            float q = 0.f;
            if (mine) {
#pragma unroll
                for (int e = 0; e < 8; ++e) { d[e] -= mean; q += d[e] * d[e]; }
            }
            const float rstd = rsqrtf(block_sum(q, scratch) * inv_width + after_eps);
#pragma unroll
            for (int e = 0; e < 8; ++e) d[e] = d[e] * rstd * aw[e] + ab[e];
        }
        if (mine) {
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] += mult * d[e];
            store8(res + c, r);
        }
    }
    if (norm_w == nullptr) return;
    float s = 0.f;
    if (mine) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s += r[e];
    }
    const float mean = block_sum(s, scratch) * inv_width;
    float q = 0.f;
    if (mine) {
#pragma unroll
        for (int e = 0; e < 8; ++e) { r[e] -= mean; q += r[e] * r[e]; }
    }
    const float rstd = rsqrtf(block_sum(q, scratch) * inv_width + norm_eps);
    if (mine) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = r[e] * rstd * nw[e] + nb[e];
        store8(out + (size_t)blockIdx.x * width + c, o);
    }
}

// delta: null, float32 or bfloat16 [rows, ld_delta]; weights and biases float32; out: float32 or bfloat16 (null with norm_w null).
TTB_EXPORT int ttb_add_layernorm(float* residual, const void* delta, int delta_dtype, int ld_delta, const float* after_w,
                                 const float* after_b, float after_eps, float mult, const float* norm_w,
                                 const float* norm_b, float norm_eps, void* out, int out_dtype, int rows, int width,
                                 cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!residual || width < 1 || (norm_w && !out)) return TTB_ERR_ARGUMENT;
    const size_t smem = (size_t)width * sizeof(float);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    // rows that fit a thread's registers: width a multiple of 8 up to LN_THREADS * 8, everything 16-byte aligned
    const bool regs = (width & 7) == 0 && width <= LN_THREADS * 8 && aligned16(residual) && (!delta || (aligned16(delta) && (ld_delta & 7) == 0)) &&
                      (!after_w || aligned16(after_w)) && (!after_b || aligned16(after_b)) && (!norm_w || aligned16(norm_w)) &&
                      (!norm_b || aligned16(norm_b)) && (!out || aligned16(out));
#define LN_LAUNCH(TD, TO)                                                                                            \
    do {                                                                                                             \
        if (regs) {                                                                                                  \
            ttb_launch(add_layernorm_regs_kernel<TD, TO>, rows, LN_THREADS, 0, stream, residual, (const TD*)delta, ld_delta, \
                       after_w, after_b, after_eps, mult, norm_w, norm_b, norm_eps, (TO*)out, width);                \
            break;                                                                                                   \
        }                                                                                                            \
        if (smem > 48 * 1024)                                                                                        \
            cudaFuncSetAttribute(add_layernorm_kernel<TD, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        ttb_launch(add_layernorm_kernel<TD, TO>, rows, LN_THREADS, smem, stream, residual, (const TD*)delta, ld_delta,    \
                   after_w, after_b, after_eps, mult, norm_w, norm_b, norm_eps, (TO*)out, width);                    \
    } while (0)
    const bool d_bf16 = delta && delta_dtype == TTB_DTYPE_BF16;
    if (delta && delta_dtype != TTB_DTYPE_BF16 && delta_dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    if (out_dtype == TTB_DTYPE_BF16) {
        if (d_bf16) LN_LAUNCH(__nv_bfloat16, __nv_bfloat16); else LN_LAUNCH(float, __nv_bfloat16);
    } else if (out_dtype == TTB_DTYPE_F32) {
        if (d_bf16) LN_LAUNCH(__nv_bfloat16, float); else LN_LAUNCH(float, float);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
#undef LN_LAUNCH
    return ttb_launch_status();
}

// Several sub-layer outputs at once, each with a factor, and a vector that is the same for every row:
//   residual += sum_i scale_i * term_i + row_scale * row_vector;   out = norm(residual)  (norm absent: nothing is written)
// Terms are float32 or bfloat16 [rows, width], contiguous. One block per row, the row in shared memory between the passes.
#define LN_MAX_TERMS 4
struct LnTerms {
    const void* ptr[LN_MAX_TERMS];
    int dtype[LN_MAX_TERMS];
    float scale[LN_MAX_TERMS];
    int count;
};

template <typename TO>
__global__ void __launch_bounds__(LN_THREADS)
add_layernorm_sum_kernel(float* __restrict__ residual, const LnTerms terms, const float* __restrict__ row_vector, float row_scale,
                         const float* __restrict__ norm_w, const float* __restrict__ norm_b, float norm_eps,
                         TO* __restrict__ out, int width) {
    extern __shared__ float row[];
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    float* res = residual + (size_t)blockIdx.x * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        float v = res[c];
        for (int i = 0; i < terms.count; ++i) {
            const size_t at = (size_t)blockIdx.x * width + c;
            const float d = terms.dtype[i] == TTB_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(terms.ptr[i])[at])
                                                             : reinterpret_cast<const float*>(terms.ptr[i])[at];
            v = fmaf(terms.scale[i], d, v);
        }
        if (row_vector != nullptr) v = fmaf(row_scale, row_vector[c], v);
        if (terms.count > 0 || row_vector != nullptr) res[c] = v;
        row[c] = v;
    }
    if (norm_w == nullptr) return;
    __syncthreads();
    float mean, rstd;
    ln_stats(row, width, norm_eps, scratch, mean, rstd);
    TO* o = out + (size_t)blockIdx.x * width;
    for (int c = threadIdx.x; c < width; c += blockDim.x)
        o[c] = from_float<TO>((row[c] - mean) * rstd * norm_w[c] + (norm_b != nullptr ? norm_b[c] : 0.f));
}

// Rows of up to LN_THREADS * 8 elements (a multiple of 8), everything 16-byte aligned: a thread keeps its eight values in
// registers through the sum and the norm, and every load is issued before the first is used.
template <typename TO>
__global__ void __launch_bounds__(LN_THREADS)
add_layernorm_sum_regs_kernel(float* __restrict__ residual, const LnTerms terms, const float* __restrict__ row_vector, float row_scale,
                              const float* __restrict__ norm_w, const float* __restrict__ norm_b, float norm_eps,
                              TO* __restrict__ out, int width) {
    __shared__ float scratch[32];
    const int c = threadIdx.x * 8;
    const bool mine = c < width;
    float nw[8], nb[8], rv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) { nw[e] = 1.f; nb[e] = 0.f; rv[e] = 0.f; }
    if (mine) {                                   // weights, which no kernel writes, before the wait for the kernel in front
        if (norm_w != nullptr) {
            load8(norm_w + c, nw);
            if (norm_b != nullptr) load8(norm_b + c, nb);
        }
        if (row_vector != nullptr) load8(row_vector + c, rv);
    }
    pdl_wait();
    pdl_launch_dependents();
    const size_t at = (size_t)blockIdx.x * width + c;
    float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float d[LN_MAX_TERMS][8];
    if (mine) {
        load8(residual + at, r);
#pragma unroll
        for (int i = 0; i < LN_MAX_TERMS; ++i) {
            if (i < terms.count) {
                if (terms.dtype[i] == TTB_DTYPE_BF16) load8(reinterpret_cast<const __nv_bfloat16*>(terms.ptr[i]) + at, d[i]);
                else load8(reinterpret_cast<const float*>(terms.ptr[i]) + at, d[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < LN_MAX_TERMS; ++i) {
            if (i < terms.count) {
#pragma unroll
                for (int e = 0; e < 8; ++e) r[e] = fmaf(terms.scale[i], d[i][e], r[e]);
            }
        }
        if (row_vector != nullptr) {
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = fmaf(row_scale, rv[e], r[e]);
        }
        if (terms.count > 0 || row_vector != nullptr) store8(residual + at, r);
    }
    if (norm_w == nullptr) return;
    const float inv_width = 1.f / (float)width;
    float s = 0.f;
    if (mine) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s += r[e];
    }
    const float mean = block_sum(s, scratch) * inv_width;
    float q = 0.f;
    if (mine) {
#pragma unroll
        for (int e = 0; e < 8; ++e) { r[e] -= mean; q += r[e] * r[e]; }
    }
    const float rstd = rsqrtf(block_sum(q, scratch) * inv_width + norm_eps);
    if (mine) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = r[e] * rstd * nw[e] + nb[e];
        store8(out + at, o);
    }
}

TTB_EXPORT int ttb_add_layernorm_sum(float* residual, const void* const* term_ptrs, const int* term_dtypes, const float* term_scales,
                                     int count, const float* row_vector, float row_scale, const float* norm_w, const float* norm_b,
                                     float norm_eps, void* out, int out_dtype, int rows, int width, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!residual || width < 1 || count < 0 || count > LN_MAX_TERMS || (norm_w && !out)) return TTB_ERR_ARGUMENT;
    LnTerms terms = {};
    terms.count = count;
    for (int i = 0; i < count; ++i) {
        if (!term_ptrs[i] || (term_dtypes[i] != TTB_DTYPE_BF16 && term_dtypes[i] != TTB_DTYPE_F32)) return TTB_ERR_ARGUMENT;
        terms.ptr[i] = term_ptrs[i]; terms.dtype[i] = term_dtypes[i]; terms.scale[i] = term_scales[i];
    }
    const size_t smem = (size_t)width * sizeof(float);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    bool regs = (width & 7) == 0 && width <= LN_THREADS * 8 && aligned16(residual) && (!row_vector || aligned16(row_vector)) &&
                (!norm_w || aligned16(norm_w)) && (!norm_b || aligned16(norm_b)) && (!out || aligned16(out));
    for (int i = 0; i < count; ++i) regs = regs && aligned16(term_ptrs[i]);
    if (regs && (out_dtype == TTB_DTYPE_BF16 || out_dtype == TTB_DTYPE_F32 || !norm_w)) {
        if (out_dtype == TTB_DTYPE_F32 && norm_w)
            ttb_launch(add_layernorm_sum_regs_kernel<float>, rows, LN_THREADS, 0, stream, residual, terms, row_vector, row_scale, norm_w,
                       norm_b, norm_eps, (float*)out, width);
        else
            ttb_launch(add_layernorm_sum_regs_kernel<__nv_bfloat16>, rows, LN_THREADS, 0, stream, residual, terms, row_vector, row_scale,
                       norm_w, norm_b, norm_eps, (__nv_bfloat16*)out, width);
        return ttb_launch_status();
    }
    if (out_dtype == TTB_DTYPE_BF16 || !norm_w) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(add_layernorm_sum_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        ttb_launch(add_layernorm_sum_kernel<__nv_bfloat16>, rows, LN_THREADS, smem, stream, residual, terms, row_vector, row_scale,
                   norm_w, norm_b, norm_eps, (__nv_bfloat16*)out, width);
    } else if (out_dtype == TTB_DTYPE_F32) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(add_layernorm_sum_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        ttb_launch(add_layernorm_sum_kernel<float>, rows, LN_THREADS, smem, stream, residual, terms, row_vector, row_scale, norm_w,
                   norm_b, norm_eps, (float*)out, width);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
    return ttb_launch_status();
}
