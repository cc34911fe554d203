// Paged causal attention for any head size, head count and group count, in float32 or
// bfloat16 storage with float32 arithmetic. One block per (token, head): it walks the
// keys of its request from the cache pages in tiles of TILE keys with a running
// maximum and sum (softmax in float32). This kernel is the path of the 32-bit mode and
// the fallback for sizes that the tensor-core kernels do not take.
//
// Query t of segment r sits at absolute position p = positions[t] and sees the keys at
// positions lo..p, lo = 0 or p - window + 1 with a window. Keys and values come from
// pages [num_pages, kv_heads, page_size, head_dim] through block_table[r, position / page_size].
// Tiles start at multiples of TILE from position 0, so that the order of summation for a
// query does not depend on how its request was cut into steps.
//
// Options, all off by default: values of another size than keys (value_dim); a cap on the scores,
// score = cap * tanh(score / cap); chunks (lo = the first position of the chunk of `chunk` positions that
// holds p); a sink per head, one more term exp(sink_h) of the softmax's denominator without a value; a bias by
// distance, dist_bias[h, min(p - key, far)] (float32 [heads, far + 1]), added to the capped score.
#include "common.cuh"

#define ATT_TILE 128
#define ATT_THREADS 128
#define ATT_MAX_ACC 4   // head_dim <= ATT_MAX_ACC * ATT_THREADS

template <typename T>
__global__ void __launch_bounds__(ATT_THREADS)
paged_attention_generic_kernel(const T* __restrict__ qkv, int q_row_stride, T* __restrict__ out,
                               const int* __restrict__ positions, const int* __restrict__ seg_of_token,
                               const T* __restrict__ key_pages, const T* __restrict__ value_pages,
                               const int* __restrict__ block_table, int table_width, int page_size,
                               int heads, int kv_heads, int head_dim, float scale, int window, int num_pages,
                               int* __restrict__ status, int value_dim, float softcap, int chunk,
                               const float* __restrict__ sinks, const float* __restrict__ dist_bias, int far) {
    extern __shared__ float smem[];
    float* q = smem;                                   // [head_dim, padded to an even count]
    float* prob = smem + ((head_dim + 1) & ~1);        // [ATT_TILE]
    size_t* row_offset = reinterpret_cast<size_t*>(prob + ATT_TILE);  // [ATT_TILE] element offset of each key row
    __shared__ float scratch[32];

    const int t = blockIdx.x, h = blockIdx.y;
    const int g = h / (heads / kv_heads);
    const int pos = positions[t];
    const int seg = seg_of_token[t];
    int lo = (window > 0 && pos - window + 1 > 0) ? pos - window + 1 : 0;
    if (chunk > 0 && pos / chunk * chunk > lo) lo = pos / chunk * chunk;
    const int* table = block_table + (size_t)seg * table_width;

    const T* q_src = qkv + (size_t)t * q_row_stride + (size_t)h * head_dim;
    for (int d = threadIdx.x; d < head_dim; d += ATT_THREADS) q[d] = to_float(q_src[d]);

    float acc[ATT_MAX_ACC];
#pragma unroll
    for (int a = 0; a < ATT_MAX_ACC; ++a) acc[a] = 0.f;
    float run_max = -INFINITY, run_sum = 0.f;
    const bool vec_ok = (head_dim & 7) == 0;

    const int first_tile = lo / ATT_TILE;
    const int last_tile = pos / ATT_TILE;
    for (int tile = first_tile; tile <= last_tile; ++tile) {
        __syncthreads();   // q ready (first pass); prob and row_offset free (later passes)
        const int key = tile * ATT_TILE + threadIdx.x;
        float score = -INFINITY;
        int page = (key >= lo && key <= pos) ? table[key / page_size] : -1;
        if (key >= lo && key <= pos && (unsigned)page >= (unsigned)num_pages) {
            atomicExch(status, 0x2000000 + t);     // a page id outside the pool: the key is left out
            row_offset[threadIdx.x] = 0;
            page = -1;
        }
        if (page >= 0) {
            const size_t row = ((size_t)page * kv_heads + g) * page_size + (key % page_size);
            row_offset[threadIdx.x] = row * value_dim;
            const T* k = key_pages + row * head_dim;
            float dot = 0.f;
            if (vec_ok) {
                for (int d = 0; d < head_dim; d += 8) {
                    float kv[8];
                    load8(k + d, kv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) dot += q[d + e] * kv[e];
                }
            } else {
                for (int d = 0; d < head_dim; ++d) dot += q[d] * to_float(k[d]);
            }
            score = dot * scale;
            if (softcap > 0.f) score = softcap * tanhf(score / softcap);
            if (dist_bias != nullptr) score += dist_bias[(size_t)h * (far + 1) + min(pos - key, far)];   // not scaled, not capped
        }
        const float tile_max = block_max(score, scratch);
        const float new_max = fmaxf(run_max, tile_max);       // finite: every tile holds at least one visible key
        const float p = (score == -INFINITY) ? 0.f : expf(score - new_max);
        prob[threadIdx.x] = p;
        const float tile_sum = block_sum(p, scratch);         // syncs inside: prob and row_offset are visible after it
        const float correction = (run_max == -INFINITY) ? 0.f : expf(run_max - new_max);
        run_sum = run_sum * correction + tile_sum;
        run_max = new_max;

        const int k_begin = (tile * ATT_TILE < lo) ? lo - tile * ATT_TILE : 0;
        const int k_end = (tile * ATT_TILE + ATT_TILE - 1 > pos) ? pos - tile * ATT_TILE + 1 : ATT_TILE;
#pragma unroll
        for (int a = 0; a < ATT_MAX_ACC; ++a) {
            const int d = threadIdx.x + a * ATT_THREADS;
            if (d < value_dim) {
                float sum = 0.f;
                for (int j = k_begin; j < k_end; ++j) sum += prob[j] * to_float(value_pages[row_offset[j] + d]);
                acc[a] = acc[a] * correction + sum;
            }
        }
    }
    float shrink = 1.f;
    if (sinks != nullptr) {                                  // one more term of the denominator; it has no value
        const float sink = sinks[h];
        const float top = fmaxf(run_max, sink);
        shrink = expf(run_max - top);
        run_sum = run_sum * shrink + expf(sink - top);
    }
    const float inv = shrink / run_sum;
    T* dst = out + ((size_t)t * heads + h) * value_dim;
#pragma unroll
    for (int a = 0; a < ATT_MAX_ACC; ++a) {
        const int d = threadIdx.x + a * ATT_THREADS;
        if (d < value_dim) dst[d] = from_float<T>(acc[a] * inv);
    }
}

TTB_EXPORT int ttb_paged_attention_generic_bias(const void* qkv, int q_row_stride, void* out, int dtype,
                                           const int* positions, const int* seg_of_token, const void* key_pages,
                                           const void* value_pages, const int* block_table, int table_width,
                                           int page_size, int tokens, int heads, int kv_heads, int head_dim,
                                           float scale, int window, int num_pages, int* status, int value_dim, float softcap,
                                           int chunk, const float* sinks, const float* dist_bias, int far, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!qkv || !out || !positions || !seg_of_token || !key_pages || !value_pages || !block_table || !status)
        return TTB_ERR_ARGUMENT;
    if (head_dim < 1 || value_dim < 1 || value_dim > ATT_MAX_ACC * ATT_THREADS || head_dim > 4096) return TTB_ERR_UNSUPPORTED;
    if (softcap < 0.f || chunk < 0 || (dist_bias && far < 0)) return TTB_ERR_ARGUMENT;
    if (kv_heads < 1 || heads % kv_heads != 0) return TTB_ERR_UNSUPPORTED;
    if (heads > 65535) return TTB_ERR_UNSUPPORTED;
    const size_t smem = (size_t)(((head_dim + 1) & ~1) + ATT_TILE) * sizeof(float) + ATT_TILE * sizeof(size_t);
    dim3 grid(tokens, heads);
    if (dtype == TTB_DTYPE_BF16) {
        if ((head_dim & 7) == 0 && (!aligned16(key_pages))) return TTB_ERR_ARGUMENT;
        paged_attention_generic_kernel<<<grid, ATT_THREADS, smem, stream>>>(
            (const __nv_bfloat16*)qkv, q_row_stride, (__nv_bfloat16*)out, positions, seg_of_token,
            (const __nv_bfloat16*)key_pages, (const __nv_bfloat16*)value_pages, block_table, table_width, page_size,
            heads, kv_heads, head_dim, scale, window, num_pages, status, value_dim, softcap, chunk, sinks, dist_bias, far);
    } else if (dtype == TTB_DTYPE_F32) {
        if ((head_dim & 7) == 0 && (!aligned16(key_pages))) return TTB_ERR_ARGUMENT;
        paged_attention_generic_kernel<<<grid, ATT_THREADS, smem, stream>>>(
            (const float*)qkv, q_row_stride, (float*)out, positions, seg_of_token, (const float*)key_pages,
            (const float*)value_pages, block_table, table_width, page_size, heads, kv_heads, head_dim, scale, window, num_pages, status, value_dim, softcap, chunk, sinks, dist_bias, far);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
    return ttb_launch_status();
}

TTB_EXPORT int ttb_paged_attention_generic_ext(const void* qkv, int q_row_stride, void* out, int dtype,
                                           const int* positions, const int* seg_of_token, const void* key_pages,
                                           const void* value_pages, const int* block_table, int table_width,
                                           int page_size, int tokens, int heads, int kv_heads, int head_dim,
                                           float scale, int window, int num_pages, int* status, int value_dim, float softcap,
                                           int chunk, const float* sinks, cudaStream_t stream) {
    return ttb_paged_attention_generic_bias(qkv, q_row_stride, out, dtype, positions, seg_of_token, key_pages, value_pages, block_table,
                                            table_width, page_size, tokens, heads, kv_heads, head_dim, scale, window, num_pages, status,
                                            value_dim, softcap, chunk, sinks, nullptr, 0, stream);
}

TTB_EXPORT int ttb_paged_attention_generic(const void* qkv, int q_row_stride, void* out, int dtype,
                                           const int* positions, const int* seg_of_token, const void* key_pages,
                                           const void* value_pages, const int* block_table, int table_width,
                                           int page_size, int tokens, int heads, int kv_heads, int head_dim,
                                           float scale, int window, int num_pages, int* status, cudaStream_t stream) {
    return ttb_paged_attention_generic_ext(qkv, q_row_stride, out, dtype, positions, seg_of_token, key_pages, value_pages, block_table,
                                           table_width, page_size, tokens, heads, kv_heads, head_dim, scale, window, num_pages, status,
                                           head_dim, 0.f, 0, nullptr, stream);
}
