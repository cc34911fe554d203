// Attention over a paged cache of latents: one row per token, [latent | extra], from which every head's key and
// value are linear maps. Queries arrive already carried into the latent space (q' = W_uk^T q), so all heads read
// the same rows: score_h(i, j) = (q'_h(i) . c(j) + R(i) q_rot,h(i) . extra(j)) * scale, the weighted sum of the
// latents leaves as [tokens, heads, latent] and goes through W_uv afterwards.
//
// latent_prepare: RMS norm of the query latent; RMS norm of the key/value latent and rotation of the shared
//   rotated key part by the token's position, written into the token's page row. Norms and angles are float32.
// latent_attention_generic: float32 arithmetic on float32 or bfloat16 storage; any sizes. One block per token
//   and group of up to LA_HEADS heads; key tiles start at multiples of LA_TILE from position 0, so the order of
//   summation for a query does not depend on how its request was cut into steps or what else the batch holds.
//   An optional sink per head joins the softmax's denominator (no key, no value, not scaled).
// gate_heads: out[t, h, v] * sigmoid(gate) with one gate number per head or per element, into [tokens, heads * v].
#include "common.cuh"

#define LA_TILE 128
#define LA_THREADS 128
#define LA_HEADS 8
#define LA_MAX_ACC 4   // output columns per block: LA_MAX_ACC * LA_THREADS

// ---------------------------------------------------------------- latent_prepare
// A warp per token (eight tokens a block): both sums of squares are warp reductions, nothing waits on the block.
#define LP_WARPS 8
template <typename TO>
__global__ void __launch_bounds__(LP_WARPS * 32)
latent_prepare_kernel(const float* __restrict__ down, int ld_down, int q_rank, int kv_rank, int rot_dim,
                      const float* __restrict__ q_norm, const float* __restrict__ kv_norm, float eps,
                      const float* __restrict__ inv_freq, int rotary_dim, const int* __restrict__ positions,
                      const int* __restrict__ seg_of_token, TO* __restrict__ cq, TO* __restrict__ rows,
                      const int* __restrict__ block_table, int table_width, int page_size, int num_pages, int write,
                      int tokens, int* __restrict__ status, float amplitude) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * LP_WARPS + (threadIdx.x >> 5);
    if (t >= tokens) return;
    const float* src = down + (size_t)t * ld_down;
    const float* c_src = src + q_rank;
    // where the token's row goes (looked up while the sums are formed)
    int pos = 0, page = -1;
    if (write) {
        pos = positions[t];
        const int page_index = pos / page_size;
        if (page_index < table_width) {
            page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
            if ((unsigned)page >= (unsigned)num_pages) {
                if (lane == 0) atomicExch(status, 0x2000000 + t);         // a page id outside the pool
                page = -1;
            }
        } else if (lane == 0) {
            atomicExch(status, 0x1000000 + t);                             // a position beyond the block table
        }
    }
    float sq = 0.f, sc = 0.f;
    for (int c = lane; c < q_rank; c += 32) sq = fmaf(src[c], src[c], sq);
    for (int c = lane; c < kv_rank; c += 32) sc = fmaf(c_src[c], c_src[c], sc);
    const float q_scale = rsqrtf(warp_sum(sq) / (float)q_rank + eps);
    const float c_scale = rsqrtf(warp_sum(sc) / (float)kv_rank + eps);
    for (int c = lane; c < q_rank; c += 32) cq[(size_t)t * q_rank + c] = from_float<TO>(src[c] * q_scale * q_norm[c]);
    if (page < 0) return;
    TO* dst = rows + ((size_t)page * page_size + (pos % page_size)) * (kv_rank + rot_dim);
    for (int c = lane; c < kv_rank; c += 32) dst[c] = from_float<TO>(c_src[c] * c_scale * kv_norm[c]);
    const float* r_src = c_src + kv_rank;
    const int half = rotary_dim / 2;
    for (int i = lane; i < half; i += 32) {
        float sn, cs;
        sincosf((float)pos * inv_freq[i], &sn, &cs);
        sn *= amplitude;
        cs *= amplitude;
        const float u = r_src[i], v = r_src[i + half];
        dst[kv_rank + i] = from_float<TO>(u * cs - v * sn);
        dst[kv_rank + i + half] = from_float<TO>(v * cs + u * sn);
    }
    for (int i = rotary_dim + lane; i < rot_dim; i += 32) dst[kv_rank + i] = from_float<TO>(r_src[i]);
}

// q_rank 0: no query latent (q_norm and cq may be null); amplitude: what the rotation's cosines and sines are multiplied by.
TTB_EXPORT int ttb_latent_prepare_ext(const float* down, int ld_down, int q_rank, int kv_rank, int rot_dim,
                                  const float* q_norm, const float* kv_norm, float eps, const float* inv_freq,
                                  int rotary_dim, const int* positions, const int* seg_of_token, void* cq, void* rows,
                                  int dtype, const int* block_table, int table_width, int page_size, int num_pages,
                                  int write, int tokens, int* status, float amplitude, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!down || !positions || !seg_of_token || !status || q_rank < 0) return TTB_ERR_ARGUMENT;
    if (q_rank > 0 && (!q_norm || !cq)) return TTB_ERR_ARGUMENT;
    if (write && (!rows || !block_table || !kv_norm)) return TTB_ERR_ARGUMENT;
    if (rot_dim < 0 || rotary_dim < 0 || rotary_dim > rot_dim || (rotary_dim & 1) || (rotary_dim > 0 && !inv_freq))
        return TTB_ERR_ARGUMENT;
    const int blocks = (tokens + LP_WARPS - 1) / LP_WARPS;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(latent_prepare_kernel<__nv_bfloat16>, blocks, LP_WARPS * 32, 0, stream, down, ld_down, q_rank, kv_rank, rot_dim,
                   q_norm, kv_norm, eps, inv_freq, rotary_dim, positions, seg_of_token, (__nv_bfloat16*)cq,
                   (__nv_bfloat16*)rows, block_table, table_width, page_size, num_pages, write, tokens, status, amplitude);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(latent_prepare_kernel<float>, blocks, LP_WARPS * 32, 0, stream, down, ld_down, q_rank, kv_rank, rot_dim, q_norm,
                   kv_norm, eps, inv_freq, rotary_dim, positions, seg_of_token, (float*)cq, (float*)rows, block_table,
                   table_width, page_size, num_pages, write, tokens, status, amplitude);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

TTB_EXPORT int ttb_latent_prepare(const float* down, int ld_down, int q_rank, int kv_rank, int rot_dim,
                                  const float* q_norm, const float* kv_norm, float eps, const float* inv_freq,
                                  int rotary_dim, const int* positions, const int* seg_of_token, void* cq, void* rows,
                                  int dtype, const int* block_table, int table_width, int page_size, int num_pages,
                                  int write, int tokens, int* status, cudaStream_t stream) {
    return ttb_latent_prepare_ext(down, ld_down, q_rank, kv_rank, rot_dim, q_norm, kv_norm, eps, inv_freq, rotary_dim, positions,
                                  seg_of_token, cq, rows, dtype, block_table, table_width, page_size, num_pages, write, tokens,
                                  status, 1.f, stream);
}

// ---------------------------------------------------------------- latent_attention_generic
template <typename T>
__global__ void __launch_bounds__(LA_THREADS)
latent_attention_generic_kernel(const T* __restrict__ q_lat, long long ql_stride_t, long long ql_stride_h,
                                const T* __restrict__ q_rot, long long qr_stride_t, long long qr_stride_h,
                                T* __restrict__ out, const int* __restrict__ positions,
                                const int* __restrict__ seg_of_token, const T* __restrict__ rows,
                                const int* __restrict__ block_table, int table_width, int page_size, int heads,
                                int latent, int extra, float scale, const float* __restrict__ sinks,
                                const float* __restrict__ inv_freq, int rotary_dim, int window, int num_pages,
                                int* __restrict__ status, float amplitude) {
    extern __shared__ __align__(16) float smem[];
    const int dk = latent + extra, dk_pad = (dk + 3) & ~3;
    float* q = smem;                                       // [LA_HEADS, dk_pad]
    float* prob = q + LA_HEADS * dk_pad;                   // [LA_HEADS, LA_TILE]
    size_t* row_offset = reinterpret_cast<size_t*>(prob + LA_HEADS * LA_TILE);   // [LA_TILE]
    __shared__ float scratch[32];

    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, h0 = blockIdx.y * LA_HEADS;
    const int nh = min(LA_HEADS, heads - h0);
    const int col_base = blockIdx.z * LA_MAX_ACC * LA_THREADS;      // this block's share of the output columns
    const int pos = positions[t];
    const int lo = (window > 0 && pos - window + 1 > 0) ? pos - window + 1 : 0;
    const int* table = block_table + (size_t)seg_of_token[t] * table_width;

    for (int i = threadIdx.x; i < nh * latent; i += LA_THREADS) {
        const int h = i / latent, d = i % latent;
        q[h * dk_pad + d] = to_float(q_lat[(size_t)t * ql_stride_t + (size_t)(h0 + h) * ql_stride_h + d]);
    }
    if (extra > 0) {
        const int half = rotary_dim / 2;
        for (int i = threadIdx.x; i < nh * extra; i += LA_THREADS) {
            const int h = i / extra, d = i % extra;
            const T* src = q_rot + (size_t)t * qr_stride_t + (size_t)(h0 + h) * qr_stride_h;
            float v = to_float(src[d]);
            if (d < rotary_dim) {                        // rotated by this token's position: pairs (i, i + rotary_dim/2)
                const int f = d < half ? d : d - half;
                float sn, cs;
                sincosf((float)pos * inv_freq[f], &sn, &cs);
                const float other = to_float(src[d < half ? d + half : d - half]);
                v = (d < half ? v * cs - other * sn : v * cs + other * sn) * amplitude;
            }
            q[h * dk_pad + latent + d] = v;
        }
    }

    float acc[LA_MAX_ACC][LA_HEADS];
#pragma unroll
    for (int a = 0; a < LA_MAX_ACC; ++a)
#pragma unroll
        for (int h = 0; h < LA_HEADS; ++h) acc[a][h] = 0.f;
    float run_max[LA_HEADS], run_sum[LA_HEADS];
#pragma unroll
    for (int h = 0; h < LA_HEADS; ++h) { run_max[h] = -INFINITY; run_sum[h] = 0.f; }
    const bool vec_ok = (dk & 7) == 0;

    for (int tile = lo / LA_TILE; tile <= pos / LA_TILE; ++tile) {
        __syncthreads();   // q ready (first pass); prob and row_offset free (later passes)
        const int key = tile * LA_TILE + threadIdx.x;
        const bool visible = key >= lo && key <= pos;
        int page = visible ? table[key / page_size] : -1;
        if (visible && (unsigned)page >= (unsigned)num_pages) {
            atomicExch(status, 0x2000000 + t);         // a page id outside the pool: the key is left out
            page = -1;
        }
        float dot[LA_HEADS];
#pragma unroll
        for (int h = 0; h < LA_HEADS; ++h) dot[h] = 0.f;
        row_offset[threadIdx.x] = 0;
        if (page >= 0) {
            const size_t off = ((size_t)page * page_size + (key % page_size)) * dk;
            row_offset[threadIdx.x] = off;
            const T* k = rows + off;
            if (vec_ok) {
                for (int d = 0; d < dk; d += 8) {
                    float kv[8];
                    load8(k + d, kv);
#pragma unroll
                    for (int h = 0; h < LA_HEADS; ++h) {
                        if (h < nh) {
                            const float4 a = *reinterpret_cast<const float4*>(q + h * dk_pad + d);
                            const float4 b = *reinterpret_cast<const float4*>(q + h * dk_pad + d + 4);
                            dot[h] += a.x * kv[0] + a.y * kv[1] + a.z * kv[2] + a.w * kv[3] + b.x * kv[4] + b.y * kv[5] +
                                      b.z * kv[6] + b.w * kv[7];
                        }
                    }
                }
            } else {
                for (int d = 0; d < dk; ++d) {
                    const float kv = to_float(k[d]);
#pragma unroll
                    for (int h = 0; h < LA_HEADS; ++h)
                        if (h < nh) dot[h] += q[h * dk_pad + d] * kv;
                }
            }
        }
        float correction[LA_HEADS];
#pragma unroll
        for (int h = 0; h < LA_HEADS; ++h) {
            correction[h] = 1.f;
            if (h < nh) {                                  // nh is the same for every thread of the block
                const float score = page >= 0 ? dot[h] * scale : -INFINITY;
                const float new_max = fmaxf(run_max[h], block_max(score, scratch));   // finite: a tile holds a visible key
                const float p = page >= 0 ? expf(score - new_max) : 0.f;
                prob[h * LA_TILE + threadIdx.x] = p;
                const float tile_sum = block_sum(p, scratch);
                correction[h] = run_max[h] == -INFINITY ? 0.f : expf(run_max[h] - new_max);
                run_sum[h] = run_sum[h] * correction[h] + tile_sum;
                run_max[h] = new_max;
            }
        }
        __syncthreads();
        const int k_begin = (tile * LA_TILE < lo) ? lo - tile * LA_TILE : 0;
        const int k_end = (tile * LA_TILE + LA_TILE - 1 > pos) ? pos - tile * LA_TILE + 1 : LA_TILE;
#pragma unroll
        for (int a = 0; a < LA_MAX_ACC; ++a) {
            const int d = col_base + threadIdx.x + a * LA_THREADS;
            if (d < latent) {
                float sum[LA_HEADS];
#pragma unroll
                for (int h = 0; h < LA_HEADS; ++h) sum[h] = 0.f;
                for (int j = k_begin; j < k_end; ++j) {
                    const float c = to_float(rows[row_offset[j] + d]);
#pragma unroll
                    for (int h = 0; h < LA_HEADS; ++h) sum[h] += prob[h * LA_TILE + j] * c;
                }
#pragma unroll
                for (int h = 0; h < LA_HEADS; ++h) acc[a][h] = acc[a][h] * correction[h] + sum[h];
            }
        }
    }
#pragma unroll
    for (int h = 0; h < LA_HEADS; ++h) {
        if (h < nh) {
            float denom = run_sum[h];
            if (sinks != nullptr) denom += expf(sinks[h0 + h] - run_max[h]);    // the sink: in the denominator only
            const float inv = 1.f / denom;
            T* dst = out + ((size_t)t * heads + h0 + h) * latent;
#pragma unroll
            for (int a = 0; a < LA_MAX_ACC; ++a) {
                const int d = col_base + threadIdx.x + a * LA_THREADS;
                if (d < latent) dst[d] = from_float<T>(acc[a][h] * inv);
            }
        }
    }
}

TTB_EXPORT int ttb_latent_attention_generic_ext(const void* q_lat, long long ql_stride_t, long long ql_stride_h,
                                            const void* q_rot, long long qr_stride_t, long long qr_stride_h, void* out,
                                            int dtype, const int* positions, const int* seg_of_token, const void* rows,
                                            const int* block_table, int table_width, int page_size, int tokens,
                                            int heads, int latent, int extra, float scale, const float* sinks,
                                            const float* inv_freq, int rotary_dim, int window, int num_pages,
                                            int* status, float amplitude, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!q_lat || !out || !positions || !seg_of_token || !rows || !block_table || !status) return TTB_ERR_ARGUMENT;
    if (extra > 0 && (!q_rot || (rotary_dim > 0 && !inv_freq))) return TTB_ERR_ARGUMENT;
    if (latent < 1 || extra < 0 || rotary_dim > extra || (rotary_dim & 1))
        return TTB_ERR_UNSUPPORTED;
    if (heads < 1 || (heads + LA_HEADS - 1) / LA_HEADS > 65535) return TTB_ERR_UNSUPPORTED;
    const int dk = latent + extra, dk_pad = (dk + 3) & ~3;
    if ((dk & 7) == 0 && !aligned16(rows)) return TTB_ERR_ARGUMENT;
    const size_t smem = (size_t)LA_HEADS * (dk_pad + LA_TILE) * sizeof(float) + LA_TILE * sizeof(size_t);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    // output columns beyond LA_MAX_ACC * LA_THREADS go to further blocks (blockIdx.z), which compute the scores again
    dim3 grid(tokens, (heads + LA_HEADS - 1) / LA_HEADS, (latent + LA_MAX_ACC * LA_THREADS - 1) / (LA_MAX_ACC * LA_THREADS));
#define LA_LAUNCH(T)                                                                                                 \
    do {                                                                                                             \
        if (smem > 48 * 1024)                                                                                        \
            cudaFuncSetAttribute(latent_attention_generic_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        ttb_launch(latent_attention_generic_kernel<T>, grid, LA_THREADS, smem, stream, (const T*)q_lat, ql_stride_t,  \
                   ql_stride_h, (const T*)q_rot, qr_stride_t, qr_stride_h, (T*)out, positions, seg_of_token,         \
                   (const T*)rows, block_table, table_width, page_size, heads, latent, extra, scale, sinks, inv_freq, \
                   rotary_dim, window, num_pages, status, amplitude);                                                \
    } while (0)
    if (dtype == TTB_DTYPE_BF16) LA_LAUNCH(__nv_bfloat16);
    else if (dtype == TTB_DTYPE_F32) LA_LAUNCH(float);
    else return TTB_ERR_UNSUPPORTED;
#undef LA_LAUNCH
    return ttb_launch_status();
}

TTB_EXPORT int ttb_latent_attention_generic(const void* q_lat, long long ql_stride_t, long long ql_stride_h,
                                            const void* q_rot, long long qr_stride_t, long long qr_stride_h, void* out,
                                            int dtype, const int* positions, const int* seg_of_token, const void* rows,
                                            const int* block_table, int table_width, int page_size, int tokens,
                                            int heads, int latent, int extra, float scale, const float* sinks,
                                            const float* inv_freq, int rotary_dim, int window, int num_pages,
                                            int* status, cudaStream_t stream) {
    return ttb_latent_attention_generic_ext(q_lat, ql_stride_t, ql_stride_h, q_rot, qr_stride_t, qr_stride_h, out, dtype, positions,
                                            seg_of_token, rows, block_table, table_width, page_size, tokens, heads, latent, extra,
                                            scale, sinks, inv_freq, rotary_dim, window, num_pages, status, 1.f, stream);
}

// ---------------------------------------------------------------- gate_heads
template <typename T>
__global__ void gate_heads_kernel(const T* __restrict__ in, long long stride_t, long long stride_h,
                                  const float* __restrict__ gate, int ld_gate, int per_head, T* __restrict__ out,
                                  int heads, int vdim) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, n = heads * vdim;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int h = i / vdim, v = i % vdim;
        float x = to_float(in[(size_t)t * stride_t + (size_t)h * stride_h + v]);
        if (gate != nullptr) {
            const float g = gate[(size_t)t * ld_gate + (per_head ? h : i)];
            x *= 1.f / (1.f + expf(-g));
        }
        out[(size_t)t * n + i] = from_float<T>(x);
    }
}

// in: [tokens, heads, vdim] with element strides (stride_t, stride_h, 1); gate: float32 logits, one per head
// (per_head) or per element, or null; out: contiguous [tokens, heads * vdim].
TTB_EXPORT int ttb_gate_heads(const void* in, long long stride_t, long long stride_h, const float* gate, int ld_gate,
                              int per_head, void* out, int dtype, int tokens, int heads, int vdim, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!in || !out) return TTB_ERR_ARGUMENT;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(gate_heads_kernel<__nv_bfloat16>, tokens, 256, 0, stream, (const __nv_bfloat16*)in, stride_t, stride_h,
                   gate, ld_gate, per_head, (__nv_bfloat16*)out, heads, vdim);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(gate_heads_kernel<float>, tokens, 256, 0, stream, (const float*)in, stride_t, stride_h, gate, ld_gate,
                   per_head, (float*)out, heads, vdim);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// ---------------------------------------------------------------- latent_out (a handful of tokens)
// The end of the mixer for decode steps in one kernel: the key splits' partial sums are merged (or the finished
// weighted sum of latents is read), carried through the head's W_uv and gated:
//   out[t, h, v] = sigmoid(gate) * sum_r W_uv[h, v, r] * c[t, h, r].
// One block per (token, head); c is float32 in shared memory; a warp works on four rows of W_uv at a time.
#define LO_THREADS 128

template <typename T, bool VEC>
__global__ void __launch_bounds__(LO_THREADS)
latent_out_kernel(const T* __restrict__ mixed, long long in_stride_t, long long in_stride_h,
                  const float* __restrict__ partial_o, const float* __restrict__ partial_ml, int splits,
                  const T* __restrict__ w_uv, const float* __restrict__ gate, int ld_gate, int per_head,
                  T* __restrict__ out, int heads, int latent, int vdim) {
    extern __shared__ __align__(16) float lo_c[];          // [latent]
    __shared__ float wt[64];
    {   // this head's W_uv on its way into L2 while the attention kernel finishes
        const char* w = reinterpret_cast<const char*>(w_uv + (size_t)blockIdx.y * vdim * latent);
        const size_t bytes = (size_t)vdim * latent * sizeof(T);
        for (size_t off = (size_t)threadIdx.x * 128; off < bytes; off += (size_t)LO_THREADS * 128) prefetch_l2(w + off);
    }
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, h = blockIdx.y;
    const size_t row = (size_t)t * heads + h;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (splits > 1) {
        if (warp == 0) {
            const float2* ml = reinterpret_cast<const float2*>(partial_ml) + row * splits;
            const float2 a = lane < splits ? ml[lane] : make_float2(-INFINITY, 0.f);
            const float2 b = lane + 32 < splits ? ml[lane + 32] : make_float2(-INFINITY, 0.f);
            const float M = warp_max(fmaxf(a.x, b.x));
            const float wa = a.x == -INFINITY ? 0.f : exp2f(a.x - M), wb = b.x == -INFINITY ? 0.f : exp2f(b.x - M);
            wt[lane] = wa * a.y;
            wt[lane + 32] = wb * b.y;
            __syncwarp();
            float denom = 0.f;
            for (int s = 0; s < splits; ++s) denom += wt[s];        // in the order of the splits
            const float inv = denom > 0.f ? 1.f / denom : 0.f;
            __syncwarp();
            wt[lane] = wa * inv;
            wt[lane + 32] = wb * inv;
        }
        __syncthreads();
        for (int c = threadIdx.x; c < latent; c += LO_THREADS) {
            const float* src = partial_o + row * splits * latent + c;
            float acc = 0.f;
#pragma unroll 8
            for (int s = 0; s < splits; ++s) acc = fmaf(wt[s], src[(size_t)s * latent], acc);
            lo_c[c] = acc;
        }
    } else {
        const T* src = mixed + (size_t)t * in_stride_t + (size_t)h * in_stride_h;
        for (int c = threadIdx.x; c < latent; c += LO_THREADS) lo_c[c] = to_float(src[c]);
    }
    __syncthreads();
    const T* W = w_uv + (size_t)h * vdim * latent;
    for (int v0 = warp * 4; v0 < vdim; v0 += (LO_THREADS / 32) * 4) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const T* rows[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rows[i] = W + (size_t)min(v0 + i, vdim - 1) * latent;
        if (VEC) {
#pragma unroll 2
            for (int k = lane * 8; k < latent; k += 256) {
                float w[4][8];
#pragma unroll
                for (int i = 0; i < 4; ++i) load8(rows[i] + k, w[i]);
                const float4 xa = *reinterpret_cast<const float4*>(lo_c + k), xb = *reinterpret_cast<const float4*>(lo_c + k + 4);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    d[i] += w[i][0] * xa.x + w[i][1] * xa.y + w[i][2] * xa.z + w[i][3] * xa.w + w[i][4] * xb.x + w[i][5] * xb.y +
                            w[i][6] * xb.z + w[i][7] * xb.w;
            }
        } else {
            for (int k = lane; k < latent; k += 32) {
                const float x = lo_c[k];
#pragma unroll
                for (int i = 0; i < 4; ++i) d[i] = fmaf(to_float(rows[i][k]), x, d[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = warp_sum(d[i]);
        if (lane < 4 && v0 + lane < vdim) {
            float y = lane == 0 ? d[0] : lane == 1 ? d[1] : lane == 2 ? d[2] : d[3];
            const int v = v0 + lane;
            if (gate != nullptr) y *= 1.f / (1.f + expf(-gate[(size_t)t * ld_gate + (per_head ? h : h * vdim + v)]));
            out[row * vdim + v] = from_float<T>(y);
        }
    }
}

// mixed: [tokens, heads, latent] with element strides (in_stride_t, in_stride_h, 1) (splits == 1), or null with
// partial_o / partial_ml as the attention kernel's key splits left them (2 <= splits <= 64); w_uv: [heads, vdim, latent];
// out: [tokens, heads * vdim]. Without a gate and with one split this is a per-head matrix-vector product of any use.
TTB_EXPORT int ttb_latent_out(const void* mixed, long long in_stride_t, long long in_stride_h, const float* partial_o, const float* partial_ml, int splits, const void* w_uv,
                              const float* gate, int ld_gate, int per_head, void* out, int dtype, int tokens, int heads,
                              int latent, int vdim, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!w_uv || !out || splits < 1 || splits > 64) return TTB_ERR_ARGUMENT;
    if (splits == 1 ? !mixed : (!partial_o || !partial_ml)) return TTB_ERR_ARGUMENT;
    if (heads > 65535 || (size_t)latent * 4 > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    const bool vec = (latent & 7) == 0 && aligned16(w_uv);
    dim3 grid(tokens, heads);
    const size_t smem = (size_t)latent * sizeof(float);
#define LO_LAUNCH(T, VEC)                                                                                            \
    ttb_launch(latent_out_kernel<T, VEC>, grid, LO_THREADS, smem, stream, (const T*)mixed, in_stride_t, in_stride_h, partial_o, partial_ml, splits,  \
               (const T*)w_uv, gate, ld_gate, per_head, (T*)out, heads, latent, vdim)
    if (dtype == TTB_DTYPE_BF16) { if (vec) LO_LAUNCH(__nv_bfloat16, true); else LO_LAUNCH(__nv_bfloat16, false); }
    else if (dtype == TTB_DTYPE_F32) { if (vec) LO_LAUNCH(float, true); else LO_LAUNCH(float, false); }
    else return TTB_ERR_UNSUPPORTED;
#undef LO_LAUNCH
    return ttb_launch_status();
}
