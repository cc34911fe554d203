// Per-head RMS norm of queries and keys, rotation by position, and the write of keys and values into cache pages,
// for attention whose keys and values may differ in size.
//
// qkv [tokens, heads * dim | kv_heads * dim | kv_heads * vdim] of the compute type. One warp per (token, head unit),
// four of them a block:
//   query head:  q = rms(q) * w_q (optional), rotated, written back in place
//   key head:    k = rms(k) * w_k (optional), rotated, written back in place and into its page row
//   value head:  copied into its page row
// The norm is over `dim` with eps inside the root and one weight vector shared by all heads; the rotation pairs
// element i with i + rotary_dim / 2 for i < rotary_dim / 2 (angle = position * inv_freq[i], sincosf on float32) and
// leaves the other elements alone. Pages: keys [pages, kv_heads, page_size, dim], values [.., vdim].
#include "common.cuh"

#define QN_THREADS 128

template <typename T>
__global__ void __launch_bounds__(QN_THREADS)
qk_norm_rope_write_kernel(T* __restrict__ qkv, int ld, const int* __restrict__ positions, const int* __restrict__ seg_of_token,
                          const float* __restrict__ q_weight, const float* __restrict__ k_weight, float eps,
                          const float* __restrict__ inv_freq, int rotary_dim, int heads, int kv_heads, int dim, int vdim,
                          T* __restrict__ key_pages, T* __restrict__ value_pages, const int* __restrict__ block_table,
                          int table_width, int page_size, int num_pages, int write_kv, int* __restrict__ status,
                          const float* __restrict__ bias, float temp_coef, int temp_every) {
    extern __shared__ float qn_rows[];         // [warps][dim]
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x, unit = blockIdx.y * (QN_THREADS / 32) + warp;
    if (unit >= heads + 2 * kv_heads) return;
    float* qn_row = qn_rows + warp * dim;
    const int pos = positions[t];
    const bool is_q = unit < heads, is_k = !is_q && unit < heads + kv_heads;
    const int g = is_q ? unit : (is_k ? unit - heads : unit - heads - kv_heads);
    T* dst_page = nullptr;
    if (!is_q) {
        if (!write_kv) {
            if (!is_k) return;
        } else {
            const int page_index = pos / page_size;
            int page = -1;
            if (page_index >= table_width) {
                if (lane == 0) atomicExch(status, 0x1000000 + t);
            } else {
                page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
                if ((unsigned)page >= (unsigned)num_pages) {
                    if (lane == 0) atomicExch(status, 0x2000000 + t);
                    page = -1;
                }
            }
            if (page >= 0) {
                const size_t row = ((size_t)page * kv_heads + g) * page_size + pos % page_size;
                dst_page = is_k ? key_pages + row * dim : value_pages + row * vdim;
            }
        }
    }
    if (!is_q && !is_k) {                       // a value head: a copy
        const T* src = qkv + (size_t)t * ld + (size_t)(heads + kv_heads) * dim + (size_t)g * vdim;
        if (dst_page != nullptr) {
            if (bias != nullptr) {
                const float* b = bias + (size_t)(heads + kv_heads) * dim + (size_t)g * vdim;
                for (int d = lane; d < vdim; d += 32) dst_page[d] = from_float<T>(to_float(src[d]) + b[d]);
            } else {
                for (int d = lane; d < vdim; d += 32) dst_page[d] = src[d];
            }
        }
        return;
    }
    T* row = qkv + (size_t)t * ld + (size_t)(is_q ? g : heads + g) * dim;
    const float* weight = is_q ? q_weight : k_weight;
    const float* row_bias = bias != nullptr ? bias + (size_t)(is_q ? g : heads + g) * dim : nullptr;
    float sumsq = 0.f;
    for (int d = lane; d < dim; d += 32) {
        const float v = to_float(row[d]) + (row_bias != nullptr ? row_bias[d] : 0.f);
        qn_row[d] = v;
        sumsq += v * v;
    }
    // a query's temperature: 1 + c ln(floor((position + 1) / n) + 1)
    const float temperature = (is_q && temp_coef != 0.f) ? 1.f + temp_coef * logf((float)((pos + 1) / temp_every) + 1.f) : 1.f;
    if (weight != nullptr) {
        sumsq = warp_sum(sumsq);
        const float scale = temperature / sqrtf(sumsq / (float)dim + eps);
        for (int d = lane; d < dim; d += 32) qn_row[d] = qn_row[d] * scale * weight[d];
    } else if (temperature != 1.f) {
        for (int d = lane; d < dim; d += 32) qn_row[d] *= temperature;
    }
    __syncwarp();
    const int half = rotary_dim / 2;
    for (int d = lane; d < dim; d += 32) {
        float v = qn_row[d];
        if (d < rotary_dim) {
            const int i = d < half ? d : d - half;
            float sn, cs;
            sincosf((float)pos * inv_freq[i], &sn, &cs);
            v = d < half ? qn_row[d] * cs - qn_row[d + half] * sn : qn_row[d] * cs + qn_row[d - half] * sn;
        }
        const T rounded = from_float<T>(v);
        row[d] = rounded;
        if (dst_page != nullptr) dst_page[d] = rounded;
    }
}

// bias: float32 [heads * dim | kv_heads * dim | kv_heads * vdim] added to q, k and v before anything else (or null);
// temp_coef, temp_every: the queries' temperature by position (coef 0: none).
TTB_EXPORT int ttb_qk_norm_rope_write_ext(void* qkv, int dtype, int ld, const int* positions, const int* seg_of_token,
                                      const float* q_weight, const float* k_weight, float eps, const float* inv_freq,
                                      int rotary_dim, int tokens, int heads, int kv_heads, int dim, int vdim, void* key_pages,
                                      void* value_pages, const int* block_table, int table_width, int page_size, int num_pages,
                                      int write_kv, int* status, const float* bias, float temp_coef, int temp_every,
                                      cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!qkv || !positions || !seg_of_token || !status) return TTB_ERR_ARGUMENT;
    if (write_kv && (!key_pages || !value_pages || !block_table || page_size < 1)) return TTB_ERR_ARGUMENT;
    if (rotary_dim < 0 || (rotary_dim & 1) || rotary_dim > dim || (rotary_dim > 0 && !inv_freq)) return TTB_ERR_ARGUMENT;
    if (dim < 1 || vdim < 1 || heads + 2 * kv_heads > 65535) return TTB_ERR_UNSUPPORTED;
    dim3 grid(tokens, (heads + 2 * kv_heads + QN_THREADS / 32 - 1) / (QN_THREADS / 32));
    const size_t smem = (size_t)(QN_THREADS / 32) * dim * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(qk_norm_rope_write_kernel<__nv_bfloat16>, grid, QN_THREADS, smem, stream, (__nv_bfloat16*)qkv, ld, positions,
                   seg_of_token, q_weight, k_weight, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, (__nv_bfloat16*)key_pages,
                   (__nv_bfloat16*)value_pages, block_table, table_width, page_size, num_pages, write_kv, status, bias, temp_coef,
                   temp_every);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(qk_norm_rope_write_kernel<float>, grid, QN_THREADS, smem, stream, (float*)qkv, ld, positions, seg_of_token,
                   q_weight, k_weight, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, (float*)key_pages, (float*)value_pages,
                   block_table, table_width, page_size, num_pages, write_kv, status, bias, temp_coef, temp_every);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

TTB_EXPORT int ttb_qk_norm_rope_write(void* qkv, int dtype, int ld, const int* positions, const int* seg_of_token,
                                      const float* q_weight, const float* k_weight, float eps, const float* inv_freq,
                                      int rotary_dim, int tokens, int heads, int kv_heads, int dim, int vdim, void* key_pages,
                                      void* value_pages, const int* block_table, int table_width, int page_size, int num_pages,
                                      int write_kv, int* status, cudaStream_t stream) {
    return ttb_qk_norm_rope_write_ext(qkv, dtype, ld, positions, seg_of_token, q_weight, k_weight, eps, inv_freq, rotary_dim, tokens,
                                      heads, kv_heads, dim, vdim, key_pages, value_pages, block_table, table_width, page_size,
                                      num_pages, write_kv, status, nullptr, 0.f, 1, stream);
}

// ---------------------------------------------------------------- the norm over the whole projection
// The same step with the RMS norm taken over ALL of a token's query elements at once (heads * dim numbers, one
// root mean square) and over all of its key elements (kv_heads * dim), before the heads are split; the weights have
// one entry per element of the projection. The rotation's cosines and sines are multiplied by `amplitude`. One
// block per token: both sums of squares first (float32, a fixed order), then every element once.
#define QW_THREADS 256

template <typename T>
__global__ void __launch_bounds__(QW_THREADS)
qk_whole_norm_rope_write_kernel(T* __restrict__ qkv, int ld, const int* __restrict__ positions, const int* __restrict__ seg_of_token,
                                const float* __restrict__ q_weight, const float* __restrict__ k_weight, float eps,
                                const float* __restrict__ inv_freq, int rotary_dim, float amplitude, int heads, int kv_heads, int dim,
                                int vdim, T* __restrict__ key_pages, T* __restrict__ value_pages,
                                const int* __restrict__ block_table, int table_width, int page_size, int num_pages, int write_kv,
                                int* __restrict__ status) {
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int pos = positions[t];
    T* row = qkv + (size_t)t * ld;
    const int nq = heads * dim, nk = kv_heads * dim, nv = kv_heads * vdim;
    float scale_q = 1.f, scale_k = 1.f;
    if (q_weight != nullptr) {
        float sq = 0.f, sk = 0.f;
        for (int c = threadIdx.x; c < nq; c += QW_THREADS) { const float v = to_float(row[c]); sq += v * v; }
        for (int c = threadIdx.x; c < nk; c += QW_THREADS) { const float v = to_float(row[nq + c]); sk += v * v; }
        sq = block_sum(sq, scratch);
        sk = block_sum(sk, scratch);
        scale_q = 1.f / sqrtf(sq / (float)nq + eps);
        scale_k = 1.f / sqrtf(sk / (float)nk + eps);
    }
    long long page_row = -1;                                  // the token's row in its page, before the KV head's offset
    if (write_kv) {
        const int page_index = pos / page_size;
        if (page_index >= table_width) {
            if (threadIdx.x == 0) atomicExch(status, 0x1000000 + t);
        } else {
            const int page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
            if ((unsigned)page >= (unsigned)num_pages) {
                if (threadIdx.x == 0) atomicExch(status, 0x2000000 + t);
            } else {
                page_row = (long long)page;
            }
        }
    }
    const int half = rotary_dim / 2;
    // a thread owns a rotated pair (both of its elements) or one unrotated element, so nothing is read after it is written
    const int per_head = dim - half;                          // work items of one head: `half` pairs, then dim - rotary_dim singles
    for (int w = threadIdx.x; w < (heads + kv_heads) * per_head; w += QW_THREADS) {
        const int unit = w / per_head, i = w % per_head;
        const bool is_q = unit < heads;
        const int g = is_q ? unit : unit - heads;
        const int base = is_q ? g * dim : nq + g * dim;
        const float* weight = is_q ? q_weight : k_weight;
        const int wbase = g * dim;
        const float scale = is_q ? scale_q : scale_k;
        T* dst = nullptr;
        if (!is_q && page_row >= 0)
            dst = key_pages + (((size_t)page_row * kv_heads + g) * page_size + pos % page_size) * dim;
        if (i < half) {
            float a = to_float(row[base + i]) * scale, b = to_float(row[base + i + half]) * scale;
            if (weight != nullptr) { a *= weight[wbase + i]; b *= weight[wbase + i + half]; }
            float sn, cs;
            sincosf((float)pos * inv_freq[i], &sn, &cs);
            sn *= amplitude;
            cs *= amplitude;
            const T ra = from_float<T>(a * cs - b * sn), rb = from_float<T>(b * cs + a * sn);
            row[base + i] = ra;
            row[base + i + half] = rb;
            if (dst != nullptr) { dst[i] = ra; dst[i + half] = rb; }
        } else {
            const int d = i + half;                           // rotary_dim .. dim - 1
            float a = to_float(row[base + d]) * scale;
            if (weight != nullptr) a *= weight[wbase + d];
            const T ra = from_float<T>(a);
            row[base + d] = ra;
            if (dst != nullptr) dst[d] = ra;
        }
    }
    if (page_row >= 0) {
        for (int c = threadIdx.x; c < nv; c += QW_THREADS) {
            const int g = c / vdim, d = c % vdim;
            value_pages[(((size_t)page_row * kv_heads + g) * page_size + pos % page_size) * vdim + d] = row[nq + nk + c];
        }
    }
}

TTB_EXPORT int ttb_qk_whole_norm_rope_write(void* qkv, int dtype, int ld, const int* positions, const int* seg_of_token,
                                            const float* q_weight, const float* k_weight, float eps, const float* inv_freq,
                                            int rotary_dim, float amplitude, int tokens, int heads, int kv_heads, int dim, int vdim,
                                            void* key_pages, void* value_pages, const int* block_table, int table_width,
                                            int page_size, int num_pages, int write_kv, int* status, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!qkv || !positions || !seg_of_token || !status) return TTB_ERR_ARGUMENT;
    if ((q_weight == nullptr) != (k_weight == nullptr)) return TTB_ERR_ARGUMENT;
    if (write_kv && (!key_pages || !value_pages || !block_table || page_size < 1)) return TTB_ERR_ARGUMENT;
    if (rotary_dim < 0 || (rotary_dim & 1) || rotary_dim > dim || (rotary_dim > 0 && !inv_freq)) return TTB_ERR_ARGUMENT;
    if (dim < 1 || vdim < 1) return TTB_ERR_UNSUPPORTED;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(qk_whole_norm_rope_write_kernel<__nv_bfloat16>, tokens, QW_THREADS, 0, stream, (__nv_bfloat16*)qkv, ld, positions,
                   seg_of_token, q_weight, k_weight, eps, inv_freq, rotary_dim, amplitude, heads, kv_heads, dim, vdim,
                   (__nv_bfloat16*)key_pages, (__nv_bfloat16*)value_pages, block_table, table_width, page_size, num_pages, write_kv,
                   status);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(qk_whole_norm_rope_write_kernel<float>, tokens, QW_THREADS, 0, stream, (float*)qkv, ld, positions, seg_of_token,
                   q_weight, k_weight, eps, inv_freq, rotary_dim, amplitude, heads, kv_heads, dim, vdim, (float*)key_pages,
                   (float*)value_pages, block_table, table_width, page_size, num_pages, write_kv, status);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
