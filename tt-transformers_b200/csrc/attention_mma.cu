// Paged causal flash attention on the tensor cores (bfloat16 operands, float32 scores,
// running maximum, sum and output in float32), for head sizes 64 and 128.
//
// A query tile holds 16 * WM rows; a row is one (token, query head of the KV group) pair,
// token-major, so the heads that share a KV head share every key and value that is loaded.
// Keys and values stream from the cache pages in tiles of 64 keys through a cp.async pipeline
// of STAGES tiles into swizzled shared memory; the block-table entries of the block's key range
// are copied to shared memory first, so that no load of a tile waits for a load of its page id. Two shapes of the same code:
//   prefill:  WM = 4, WN = 1   four warps, 16 rows each, every warp sees all 64 keys of a tile
//   decode:   WM = 1, WN = 4   one 16-row tile (a single token's heads), the four warps take
//                              16 keys each of every tile and merge at the end
// With num_splits > 1 the keys of a tile's range are cut into num_splits chunks, one block
// each; the blocks write unnormalised partial results to scratch memory and a second kernel
// merges them (flash decoding).
//
// Query t of segment r sits at position seg_pos0[r] + (t - cu_seqlens[r]) and sees the keys at
// positions <= its own (and > its own - window, with a window).
#include "common.cuh"

#define AM_BN 64
#define AM_TABLE_CACHE 1024      // block-table entries kept in shared memory per block

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 2^x by the special-function unit (two units in the last place are plenty for probabilities
// that are rounded to bfloat16 next); 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile whose rows hold HD bfloat16 values.
template <int HD> __device__ __forceinline__ uint32_t tile_offset(int row, int chunk) {
    return (uint32_t)(row * HD * 2 + ((chunk ^ (row & 7)) << 4));
}

template <int HD, int WM, int WN, int STAGES>
__global__ void __launch_bounds__(WM * WN * 32)
attention_mma_kernel(const __nv_bfloat16* __restrict__ qkv, int q_row_stride, __nv_bfloat16* __restrict__ out,
                     const int* __restrict__ cu_seqlens, const int* __restrict__ seg_pos0,
                     const __nv_bfloat16* __restrict__ key_pages, const __nv_bfloat16* __restrict__ value_pages,
                     const int* __restrict__ block_table, int table_width, int page_size, int page_shift,
                     const int* __restrict__ qtile_seg, const int* __restrict__ qtile_tok0,
                     int heads, int kv_heads, float scale_log2, int window, int num_splits,
                     float* __restrict__ partial_o, float* __restrict__ partial_ml, int num_pages,
                     int* __restrict__ status, float softcap, float softcap_scale, int chunk_size,
                     const float* __restrict__ sinks, const float* __restrict__ dist_bias, int far, float bias_mult) {
    // Options, all off at zero / null: softcap c: score = c * tanh(q.k * softcap_scale) with softcap_scale = scale / c
    // (scale_log2 is then log2(e) alone); chunk_size n: position p sees the keys from floor(p / n) * n on only;
    // sinks: one more term 2^(sink_h * log2(e)) of every row's denominator, with no value (it joins in split 0);
    // dist_bias [heads, far + 1]: dist_bias[h, min(p - key, far)] joins the (capped) score, as it is: bias_mult is 1
    // with a cap and 1 / scale without one, where the scores stay unscaled until the exponent.
    constexpr int BM = 16 * WM;
    constexpr int THREADS = WM * WN * 32;
    constexpr int CHUNKS = HD / 8;              // 16-byte chunks per row
    constexpr int WARP_KEYS = AM_BN / WN;       // keys of a tile that one warp handles
    constexpr int NB = WARP_KEYS / 8;           // score n-blocks per warp
    constexpr int KS = HD / 16;                 // k-steps of Q K^T
    constexpr int OB = HD / 8;                  // output n-blocks
    constexpr int TILE_BYTES = AM_BN * HD * 2;

    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* q_tile = smem;                               // [BM][HD]
    unsigned char* k_stage = smem + BM * HD * 2;                // [STAGES][BN][HD]
    unsigned char* v_stage = k_stage + STAGES * TILE_BYTES;     // [STAGES][BN][HD]
    int* page_cache = reinterpret_cast<int*>(v_stage + STAGES * TILE_BYTES);   // [AM_TABLE_CACHE]

    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int warp_m = warp / WN, warp_n = warp % WN;
    // the tile list comes sorted, most keys first; blocks are handed out in the order of their linear index
    const int linear = blockIdx.x + gridDim.x * blockIdx.y, split = blockIdx.z;
    const int qt = linear / gridDim.y, g = linear % gridDim.y;
    const int rep = heads / kv_heads;
    const int seg = qtile_seg ? qtile_seg[qt] : qt;
    const int tok0 = qtile_tok0 ? qtile_tok0[qt] : 0;
    const int seg_start = cu_seqlens[seg];
    const int seg_tokens = cu_seqlens[seg + 1] - seg_start;
    if (tok0 >= seg_tokens) return;                             // a padded tile of a captured step
    const int pos0 = seg_pos0[seg];
    const int tokens_per_tile = BM / rep;
    const int tile_tokens = min(tokens_per_tile, seg_tokens - tok0);
    const int valid_rows = tile_tokens * rep;
    const int q_first = pos0 + tok0, q_last = q_first + tile_tokens - 1;
    int lo = (window > 0 && q_first - window + 1 > 0) ? q_first - window + 1 : 0;
    if (chunk_size > 0 && q_first / chunk_size * chunk_size > lo) lo = q_first / chunk_size * chunk_size;
    const int total = q_last - lo + 1;
    const int chunk = ((total + num_splits - 1) / num_splits + AM_BN - 1) / AM_BN * AM_BN;
    const int k_begin = lo + split * chunk;
    const int k_end = min(q_last + 1, k_begin + chunk);
    const int* table = block_table + (size_t)seg * table_width;

    // the two rows of the score fragment that this thread holds
    const int r0 = warp_m * 16 + (lane >> 2), r1 = r0 + 8;
    const int qpos0 = q_first + r0 / rep, qpos1 = q_first + r1 / rep;
    const int warp_qpos_min = q_first + (warp_m * 16) / rep;          // over the 16 rows of this warp
    const int warp_qpos_max = q_first + (warp_m * 16 + 15) / rep;

    float o_acc[OB][4];
#pragma unroll
    for (int i = 0; i < OB; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o_acc[i][j] = 0.f;
    float row_max[2] = {-INFINITY, -INFINITY}, row_sum[2] = {0.f, 0.f};

    if (k_begin < k_end) {
        // ---- load the query tile (rows beyond valid_rows are zero)
        for (int idx = tid; idx < BM * CHUNKS; idx += THREADS) {
            const int r = idx / CHUNKS, c = idx % CHUNKS;
            const bool ok = r < valid_rows;
            const int token = tok0 + (ok ? r / rep : 0), head = g * rep + (ok ? r % rep : 0);
            const __nv_bfloat16* src = qkv + (size_t)(seg_start + token) * q_row_stride + (size_t)head * HD + c * 8;
            cp_async16(smem_u32(q_tile + tile_offset<HD>(r, c)), src, ok ? 16 : 0);
        }
        // block-table entries of this block's keys, first page index `page_base`
        const int page_base = (page_shift >= 0) ? (k_begin >> page_shift) : (k_begin / page_size);
        {
            const int last_page = (page_shift >= 0) ? ((k_end - 1) >> page_shift) : ((k_end - 1) / page_size);
            const int count = min(last_page - page_base + 1, AM_TABLE_CACHE);
            for (int i = tid; i < count; i += THREADS) page_cache[i] = table[page_base + i];
        }
        __syncthreads();
        auto load_tile = [&](int tile, int stage) {
            const int kb = k_begin + tile * AM_BN;
#pragma unroll
            for (int it = 0; it < (AM_BN * CHUNKS + THREADS - 1) / THREADS; ++it) {
                const int idx = tid + it * THREADS;
                if ((AM_BN * CHUNKS) % THREADS != 0 && idx >= AM_BN * CHUNKS) break;
                const int r = idx / CHUNKS, c = idx % CHUNKS;
                const int key = kb + r;
                bool ok = key < k_end;
                size_t off = 0;
                if (ok) {
                    int page_index, in_page;
                    if (page_shift >= 0) {
                        page_index = key >> page_shift;
                        in_page = key & (page_size - 1);
                    } else {
                        page_index = key / page_size;
                        in_page = key - page_index * page_size;
                    }
                    const int rel = page_index - page_base;
                    const int page = rel < AM_TABLE_CACHE ? page_cache[rel] : table[page_index];
                    if ((unsigned)page < (unsigned)num_pages) {
                        off = (((size_t)page * kv_heads + g) * page_size + in_page) * HD + c * 8;
                    } else {                      // a page id outside the pool: read nothing, say so
                        if (status != nullptr) atomicExch(status, 0x2000000 + seg);
                        ok = false;
                    }
                }
                const uint32_t dst = tile_offset<HD>(r, c) + stage * TILE_BYTES;
                cp_async16(smem_u32(k_stage + dst), key_pages + off, ok ? 16 : 0);
                cp_async16(smem_u32(v_stage + dst), value_pages + off, ok ? 16 : 0);
            }
        };
        const int num_tiles = (k_end - k_begin + AM_BN - 1) / AM_BN;
#pragma unroll
        for (int st = 0; st < STAGES - 1; ++st) {       // the first group also carries the query tile
            if (st < num_tiles) load_tile(st, st);
            cp_async_commit();
        }

        uint32_t q_frag[KS][4];
        for (int tile = 0; tile < num_tiles; ++tile) {
            const int stage = tile % STAGES;
            if (tile + STAGES - 1 < num_tiles) load_tile(tile + STAGES - 1, (tile + STAGES - 1) % STAGES);
            cp_async_commit();
            cp_async_wait<STAGES - 1>();
            __syncthreads();
            if (tile == 0) {
#pragma unroll
                for (int ks = 0; ks < KS; ++ks)
                    ldmatrix_x4(q_frag[ks], smem_u32(q_tile + tile_offset<HD>(warp_m * 16 + (lane & 15), ks * 2 + (lane >> 4))));
            }
            const unsigned char* k_tile = k_stage + stage * TILE_BYTES;
            const unsigned char* v_tile = v_stage + stage * TILE_BYTES;
            const int key_base = k_begin + tile * AM_BN + warp_n * WARP_KEYS;   // first key of this warp's part

            // ---- scores: S = Q K^T for this warp's keys
            float s[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[nb][j] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                for (int nb = 0; nb < NB; nb += 2) {
                    uint32_t b[4];
                    const int key_row = warp_n * WARP_KEYS + nb * 8 + (lane & 7) + ((lane >> 4) << 3);
                    ldmatrix_x4(b, smem_u32(k_tile + tile_offset<HD>(key_row, ks * 2 + ((lane >> 3) & 1))));
                    mma_bf16(s[nb], q_frag[ks], b[0], b[1]);
                    mma_bf16(s[nb + 1], q_frag[ks], b[2], b[3]);
                }
            }
            // ---- mask (only in tiles that the causal edge, a window or the end of the range cuts),
            //      running maximum and sum. Scores stay unscaled; the scale goes into the exponent's
            //      multiply-add: p = 2^(s * scale_log2 - max * scale_log2).
            if (softcap > 0.f) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                    for (int j = 0; j < 4; ++j) s[nb][j] = softcap * tanhf(s[nb][j] * softcap_scale);
            }
            const int last_key = key_base + WARP_KEYS - 1;
            if (dist_bias != nullptr) {
                const float* b0 = dist_bias + (size_t)(g * rep + r0 % rep) * (far + 1);
                const float* b1 = dist_bias + (size_t)(g * rep + r1 % rep) * (far + 1);
                if (warp_qpos_min - last_key >= far) {          // every key of the part lies beyond `far` for every row
                    const float c0 = b0[far] * bias_mult, c1 = b1[far] * bias_mult;
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) { s[nb][0] += c0; s[nb][1] += c0; s[nb][2] += c1; s[nb][3] += c1; }
                } else {
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int key = key_base + nb * 8 + ((lane & 3) << 1) + (j & 1);
                            const int d = ((j < 2) ? qpos0 : qpos1) - key;
                            s[nb][j] += ((j < 2) ? b0 : b1)[d < 0 ? 0 : (d > far ? far : d)] * bias_mult;
                        }
                    }
                }
            }
            const bool cut = last_key > warp_qpos_min || last_key >= k_end ||
                             (window > 0 && key_base <= warp_qpos_max - window) ||
                             (chunk_size > 0 && key_base < warp_qpos_max / chunk_size * chunk_size);
            float tile_max[2] = {-INFINITY, -INFINITY};
            if (cut) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int key = key_base + nb * 8 + ((lane & 3) << 1) + (j & 1);
                        const int qpos = (j < 2) ? qpos0 : qpos1;
                        const bool visible = key < k_end && key <= qpos && (window <= 0 || key > qpos - window) &&
                                             (chunk_size <= 0 || key >= qpos / chunk_size * chunk_size);
                        if (!visible) s[nb][j] = -INFINITY;
                    }
                }
            }
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                tile_max[0] = fmaxf(tile_max[0], fmaxf(s[nb][0], s[nb][1]));
                tile_max[1] = fmaxf(tile_max[1], fmaxf(s[nb][2], s[nb][3]));
            }
            float alpha[2], neg_max_scaled[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                tile_max[h] = fmaxf(tile_max[h], __shfl_xor_sync(0xffffffffu, tile_max[h], 1));
                tile_max[h] = fmaxf(tile_max[h], __shfl_xor_sync(0xffffffffu, tile_max[h], 2));
                const float new_max = fmaxf(row_max[h], tile_max[h]);        // unscaled
                alpha[h] = (row_max[h] == -INFINITY) ? 0.f : fast_exp2((row_max[h] - new_max) * scale_log2);
                row_max[h] = new_max;
                row_sum[h] *= alpha[h];
                neg_max_scaled[h] = (new_max == -INFINITY) ? 0.f : -new_max * scale_log2;
            }
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                s[nb][0] = fast_exp2(fmaf(s[nb][0], scale_log2, neg_max_scaled[0]));
                s[nb][1] = fast_exp2(fmaf(s[nb][1], scale_log2, neg_max_scaled[0]));
                s[nb][2] = fast_exp2(fmaf(s[nb][2], scale_log2, neg_max_scaled[1]));
                s[nb][3] = fast_exp2(fmaf(s[nb][3], scale_log2, neg_max_scaled[1]));
                row_sum[0] += s[nb][0] + s[nb][1];
                row_sum[1] += s[nb][2] + s[nb][3];
            }
            if (alpha[0] != 1.f || alpha[1] != 1.f) {       // the maximum moved: rescale what was gathered
#pragma unroll
                for (int ob = 0; ob < OB; ++ob) {
                    o_acc[ob][0] *= alpha[0];
                    o_acc[ob][1] *= alpha[0];
                    o_acc[ob][2] *= alpha[1];
                    o_acc[ob][3] *= alpha[1];
                }
            }
            // ---- output: O += P V
#pragma unroll
            for (int kk = 0; kk < WARP_KEYS / 16; ++kk) {
                uint32_t p[4];
                p[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
                p[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
                p[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
                p[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
                for (int ob = 0; ob < OB; ob += 2) {
                    uint32_t b[4];
                    const int key_row = warp_n * WARP_KEYS + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
                    ldmatrix_x4_trans(b, smem_u32(v_tile + tile_offset<HD>(key_row, ob + (lane >> 4))));
                    mma_bf16(o_acc[ob], p, b[0], b[1]);
                    mma_bf16(o_acc[ob + 1], p, b[2], b[3]);
                }
            }
            __syncthreads();     // the stage is free for the load after next
        }
        cp_async_wait<0>();
    }

    pdl_launch_dependents();     // the streaming part is over: the next kernel may move in
    // from here on the running maxima are in the exponent's units (scaled, base 2)
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (row_max[h] != -INFINITY) row_max[h] *= scale_log2;
    // ---- row sums over the four lanes of a quad
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        row_sum[h] += __shfl_xor_sync(0xffffffffu, row_sum[h], 1);
        row_sum[h] += __shfl_xor_sync(0xffffffffu, row_sum[h], 2);
    }

    // ---- the warps of one row tile merge what they saw of the keys
    if constexpr (WN > 1) {
        __syncthreads();
        float* merge_o = reinterpret_cast<float*>(k_stage);                     // [WN][16][HD]
        float* merge_ml = merge_o + WN * 16 * HD;                               // [WN][16][2]
        const int lr0 = lane >> 2, lr1 = lr0 + 8;
        if ((lane & 3) == 0) {
            merge_ml[(warp_n * 16 + lr0) * 2] = row_max[0];
            merge_ml[(warp_n * 16 + lr0) * 2 + 1] = row_sum[0];
            merge_ml[(warp_n * 16 + lr1) * 2] = row_max[1];
            merge_ml[(warp_n * 16 + lr1) * 2 + 1] = row_sum[1];
        }
#pragma unroll
        for (int ob = 0; ob < OB; ++ob) {
            const int col = ob * 8 + ((lane & 3) << 1);
            float* a = merge_o + ((size_t)(warp_n * 16 + lr0)) * HD + col;
            float* b = merge_o + ((size_t)(warp_n * 16 + lr1)) * HD + col;
            a[0] = o_acc[ob][0]; a[1] = o_acc[ob][1];
            b[0] = o_acc[ob][2]; b[1] = o_acc[ob][3];
        }
        __syncthreads();
        // every thread now owns elements of the merged tile: 16 rows x HD columns over WM*WN*32 threads
        for (int idx = tid; idx < 16 * HD; idx += THREADS) {
            const int r = idx / HD, c = idx % HD;
            float m = -INFINITY;
#pragma unroll
            for (int w = 0; w < WN; ++w) m = fmaxf(m, merge_ml[(w * 16 + r) * 2]);
            float sum = 0.f, o = 0.f;
#pragma unroll
            for (int w = 0; w < WN; ++w) {
                const float mw = merge_ml[(w * 16 + r) * 2];
                const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - m);
                sum += f * merge_ml[(w * 16 + r) * 2 + 1];
                o += f * merge_o[((size_t)(w * 16 + r)) * HD + c];
            }
            if (r >= valid_rows) continue;
            const int token = tok0 + r / rep, head = g * rep + r % rep;
            if (sinks != nullptr && split == 0) {
                const float sk = sinks[head] * 1.4426950408889634f, top = fmaxf(m, sk);
                const float f = (m == -INFINITY) ? 0.f : exp2f(m - top);
                sum = sum * f + exp2f(sk - top);
                o *= f;
                m = top;
            }
            if (num_splits > 1) {
                const size_t slot = ((size_t)(seg_start + token) * heads + head) * num_splits + split;
                partial_o[slot * HD + c] = o;
                if (c == 0) { partial_ml[slot * 2] = m; partial_ml[slot * 2 + 1] = sum; }
            } else {
                out[((size_t)(seg_start + token) * heads + head) * HD + c] = __float2bfloat16_rn(sum > 0.f ? o / sum : 0.f);
            }
        }
    } else {
    // ---- WN == 1: every warp writes its own 16 rows
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int r = h == 0 ? r0 : r1;
        if (r >= valid_rows) continue;
        const int token = tok0 + r / rep, head = g * rep + r % rep;
        const size_t row_index = (size_t)(seg_start + token) * heads + head;
        if (sinks != nullptr && split == 0) {
            const float sk = sinks[head] * 1.4426950408889634f, top = fmaxf(row_max[h], sk);
            const float f = (row_max[h] == -INFINITY) ? 0.f : exp2f(row_max[h] - top);
            row_sum[h] = row_sum[h] * f + exp2f(sk - top);
            row_max[h] = top;
#pragma unroll
            for (int ob = 0; ob < OB; ++ob) {
                o_acc[ob][2 * h] *= f;
                o_acc[ob][2 * h + 1] *= f;
            }
        }
        if (num_splits > 1) {
            const size_t slot = row_index * num_splits + split;
#pragma unroll
            for (int ob = 0; ob < OB; ++ob) {
                const int col = ob * 8 + ((lane & 3) << 1);
                *reinterpret_cast<float2*>(partial_o + slot * HD + col) = make_float2(o_acc[ob][2 * h], o_acc[ob][2 * h + 1]);
            }
            if ((lane & 3) == 0) { partial_ml[slot * 2] = row_max[h]; partial_ml[slot * 2 + 1] = row_sum[h]; }
        } else {
            const float inv = row_sum[h] > 0.f ? 1.f / row_sum[h] : 0.f;
#pragma unroll
            for (int ob = 0; ob < OB; ++ob) {
                const int col = ob * 8 + ((lane & 3) << 1);
                *reinterpret_cast<uint32_t*>(out + row_index * HD + col) = pack_bf16(o_acc[ob][2 * h] * inv, o_acc[ob][2 * h + 1] * inv);
            }
        }
    }
    }
}

// out[row, :] = sum_s w_s O_s / sum_s w_s l_s with w_s = 2^(m_s - max m); one warp per (token, head) row.
// Lane s holds split s's maximum and sum (splits beyond 32 in further rounds), so that the weights of all
// splits come from two loads and a few shuffles; the partial outputs are then read eight splits at a time.
template <int HD>
__global__ void attention_merge_kernel(const float* __restrict__ partial_o, const float* __restrict__ partial_ml,
                                       __nv_bfloat16* __restrict__ out, int rows, int num_splits) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float2* ml = reinterpret_cast<const float2*>(partial_ml) + (size_t)row * num_splits;
    float m = -INFINITY;
    for (int s0 = 0; s0 < num_splits; s0 += 32) {
        const float mine = s0 + lane < num_splits ? ml[s0 + lane].x : -INFINITY;
        m = fmaxf(m, warp_max(mine));
    }
    float acc[HD / 32];
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) acc[i] = 0.f;
    float sum = 0.f;
    for (int s0 = 0; s0 < num_splits; s0 += 32) {
        float2 mine = make_float2(-INFINITY, 0.f);
        if (s0 + lane < num_splits) mine = ml[s0 + lane];
        const float f_mine = mine.x == -INFINITY ? 0.f : exp2f(mine.x - m);
        sum += warp_sum(f_mine * mine.y);
        const int count = min(32, num_splits - s0);
        for (int j0 = 0; j0 < count; j0 += 8) {
            float v[8][HD / 32];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float* o = partial_o + ((size_t)row * num_splits + s0 + min(j0 + j, count - 1)) * HD;
#pragma unroll
                for (int i = 0; i < HD / 32; ++i) v[j][i] = o[lane + 32 * i];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = __shfl_sync(0xffffffffu, f_mine, min(j0 + j, count - 1));
                if (j0 + j < count) {
#pragma unroll
                    for (int i = 0; i < HD / 32; ++i) acc[i] += f * v[j][i];
                }
            }
        }
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) out[(size_t)row * HD + lane + 32 * i] = __float2bfloat16_rn(acc[i] * inv);
}

template <int HD, int WM, int WN, int STAGES>
static int launch_attention(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens, const int* seg_pos0,
                            const void* key_pages, const void* value_pages, const int* block_table, int table_width,
                            int page_size, const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int tokens,
                            int heads, int kv_heads, float scale, int window, int num_splits, float* partial_o,
                            float* partial_ml, int num_pages, int* status, float softcap, int chunk_size, const float* sinks,
                            cudaStream_t stream, const float* dist_bias, int far) {
    constexpr int BM = 16 * WM;
    const size_t stage_bytes = (size_t)BM * HD * 2 + 2 * (size_t)STAGES * AM_BN * HD * 2 + AM_TABLE_CACHE * sizeof(int);
    const size_t merge_bytes = (size_t)BM * HD * 2 + (size_t)WN * 16 * (HD + 2) * sizeof(float);
    const size_t smem = stage_bytes > merge_bytes ? stage_bytes : merge_bytes;
    auto kernel = attention_mma_kernel<HD, WM, WN, STAGES>;
    int page_shift = -1;
    for (int b = 0; b < 31; ++b)
        if (page_size == (1 << b)) page_shift = b;
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    dim3 grid(n_qtiles, kv_heads, num_splits);
    const float scale_log2 = (softcap > 0.f ? 1.f : scale) * 1.4426950408889634f;
    const float softcap_scale = softcap > 0.f ? scale / softcap : 0.f;
    ttb_launch(kernel, grid, dim3(WM * WN * 32), smem, stream,
        (const __nv_bfloat16*)qkv, q_row_stride, (__nv_bfloat16*)out, cu_seqlens, seg_pos0,
        (const __nv_bfloat16*)key_pages, (const __nv_bfloat16*)value_pages, block_table, table_width, page_size,
        page_shift, qtile_seg, qtile_tok0, heads, kv_heads, scale_log2, window, num_splits, partial_o, partial_ml,
        num_pages, status, softcap, softcap_scale, chunk_size, sinks, dist_bias, far, softcap > 0.f ? 1.f : 1.f / scale);
    int launch = ttb_launch_status();
    if (launch != TTB_OK || num_splits == 1) return launch;
    const int rows = tokens * heads;
    ttb_launch(attention_merge_kernel<HD>, dim3((rows + 3) / 4), dim3(128), 0, stream, (const float*)partial_o,
               (const float*)partial_ml, (__nv_bfloat16*)out, rows, num_splits);
    return ttb_launch_status();
}

// Merge of split partial results by itself (the tcgen05 attention kernel writes the same format).
TTB_EXPORT int ttb_attention_merge(const float* partial_o, const float* partial_ml, void* out, int rows, int num_splits,
                                   int head_dim, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!partial_o || !partial_ml || !out || num_splits < 1) return TTB_ERR_ARGUMENT;
    if (head_dim == 64)
        ttb_launch(attention_merge_kernel<64>, dim3((rows + 3) / 4), dim3(128), 0, stream, partial_o, partial_ml,
                   (__nv_bfloat16*)out, rows, num_splits);
    else if (head_dim == 128)
        ttb_launch(attention_merge_kernel<128>, dim3((rows + 3) / 4), dim3(128), 0, stream, partial_o, partial_ml,
                   (__nv_bfloat16*)out, rows, num_splits);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// Rows of a query tile in each shape: the host cuts segments into tiles of rows / (heads / kv_heads) tokens.
TTB_EXPORT int ttb_attention_mma_tile_rows(int decode_shape) { return decode_shape ? 16 : 64; }

// Blocks of a shape that fit one SM at a time (by shared memory): what the host sizes key splits by.
TTB_EXPORT int ttb_attention_mma_blocks_per_sm(int decode_shape, int head_dim) {
    if (head_dim == 64) return decode_shape ? 3 : 4;
    return decode_shape ? 2 : 2;
}

// Whether this kernel takes the geometry at all.
TTB_EXPORT int ttb_attention_mma_supports(int heads, int kv_heads, int head_dim) {
    if (head_dim != 64 && head_dim != 128) return 0;
    if (kv_heads < 1 || heads % kv_heads) return 0;
    return heads / kv_heads <= 16;
}

// decode_shape: 1 when every tile holds the heads of one token (16 rows), 0 for 64-row tiles.
// qtile_seg / qtile_tok0 may be null: tile i is then token 0 of segment i.
// With num_splits > 1, partial_o holds tokens * heads * num_splits * head_dim floats and partial_ml
// tokens * heads * num_splits * 2 floats of scratch memory.
// Pages are [num_pages, kv_heads, page_size, head_dim]; a block-table entry outside 0 .. num_pages-1 is not
// followed: the keys it stands for are left out and `status` (if not null) is set.
static int paged_attention_mma_impl(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                    const int* seg_pos0, const void* key_pages, const void* value_pages,
                                    const int* block_table, int table_width, int page_size, const int* qtile_seg,
                                    const int* qtile_tok0, int n_qtiles, int tokens, int heads, int kv_heads,
                                    int head_dim, float scale, int window, int decode_shape, int num_splits,
                                    float* partial_o, float* partial_ml, int num_pages, int* status,
                                    cudaStream_t stream, float softcap = 0.f, int chunk_size = 0, const float* sinks = nullptr,
                                    const float* dist_bias = nullptr, int far = 0) {
    if (n_qtiles == 0 || tokens == 0) return TTB_OK;
    if (softcap < 0.f || chunk_size < 0 || (dist_bias && (far < 0 || !(scale > 0.f)))) return TTB_ERR_ARGUMENT;
    if (!qkv || !out || !cu_seqlens || !seg_pos0 || !key_pages || !value_pages || !block_table) return TTB_ERR_ARGUMENT;
    if (!ttb_attention_mma_supports(heads, kv_heads, head_dim)) return TTB_ERR_UNSUPPORTED;
    if (num_splits < 1 || num_splits > 65535 || kv_heads > 65535) return TTB_ERR_UNSUPPORTED;
    if (num_splits > 1 && (!partial_o || !partial_ml)) return TTB_ERR_ARGUMENT;
    if ((q_row_stride & 7) || !aligned16(qkv) || !aligned16(key_pages) || !aligned16(value_pages) || !aligned16(out))
        return TTB_ERR_ARGUMENT;
    if (decode_shape && heads / kv_heads > 16) return TTB_ERR_UNSUPPORTED;
#define AM_ARGS qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table, table_width, page_size, \
                qtile_seg, qtile_tok0, n_qtiles, tokens, heads, kv_heads, scale, window, num_splits, partial_o, partial_ml, \
                num_pages, status, softcap, chunk_size, sinks, stream, dist_bias, far
    if (head_dim == 64) return decode_shape ? launch_attention<64, 1, 4, 4>(AM_ARGS) : launch_attention<64, 4, 1, 3>(AM_ARGS);
    return decode_shape ? launch_attention<128, 1, 4, 3>(AM_ARGS) : launch_attention<128, 4, 1, 2>(AM_ARGS);
#undef AM_ARGS
}

TTB_EXPORT int ttb_paged_attention_mma(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                       const int* seg_pos0, const void* key_pages, const void* value_pages,
                                       const int* block_table, int table_width, int page_size, const int* qtile_seg,
                                       const int* qtile_tok0, int n_qtiles, int tokens, int heads, int kv_heads,
                                       int head_dim, float scale, int window, int decode_shape, int num_splits,
                                       float* partial_o, float* partial_ml, cudaStream_t stream) {
    return paged_attention_mma_impl(qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table,
                                    table_width, page_size, qtile_seg, qtile_tok0, n_qtiles, tokens, heads, kv_heads,
                                    head_dim, scale, window, decode_shape, num_splits, partial_o, partial_ml,
                                    0x7fffffff, nullptr, stream);
}

// The same with the pool's size and a status word, as the engine calls it.
TTB_EXPORT int ttb_paged_attention_mma_checked(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                               const int* seg_pos0, const void* key_pages, const void* value_pages,
                                               const int* block_table, int table_width, int page_size,
                                               const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int tokens,
                                               int heads, int kv_heads, int head_dim, float scale, int window,
                                               int decode_shape, int num_splits, float* partial_o, float* partial_ml,
                                               int num_pages, int* status, cudaStream_t stream) {
    return paged_attention_mma_impl(qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table,
                                    table_width, page_size, qtile_seg, qtile_tok0, n_qtiles, tokens, heads, kv_heads,
                                    head_dim, scale, window, decode_shape, num_splits, partial_o, partial_ml,
                                    num_pages, status, stream);
}

// The same with a cap on the scores (0: none), chunks (0: none) and a sink per head (null: none); see the kernel.
TTB_EXPORT int ttb_paged_attention_mma_ext(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                           const int* seg_pos0, const void* key_pages, const void* value_pages,
                                           const int* block_table, int table_width, int page_size,
                                           const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int tokens,
                                           int heads, int kv_heads, int head_dim, float scale, int window,
                                           int decode_shape, int num_splits, float* partial_o, float* partial_ml,
                                           int num_pages, int* status, float softcap, int chunk_size, const float* sinks,
                                           cudaStream_t stream) {
    return paged_attention_mma_impl(qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table,
                                    table_width, page_size, qtile_seg, qtile_tok0, n_qtiles, tokens, heads, kv_heads,
                                    head_dim, scale, window, decode_shape, num_splits, partial_o, partial_ml,
                                    num_pages, status, stream, softcap, chunk_size, sinks);
}

// The same with a bias by distance, float32 [heads, far + 1] (null: none): dist_bias[h, min(p - key, far)] joins the capped score.
TTB_EXPORT int ttb_paged_attention_mma_bias(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                            const int* seg_pos0, const void* key_pages, const void* value_pages,
                                            const int* block_table, int table_width, int page_size,
                                            const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int tokens,
                                            int heads, int kv_heads, int head_dim, float scale, int window,
                                            int decode_shape, int num_splits, float* partial_o, float* partial_ml,
                                            int num_pages, int* status, float softcap, int chunk_size, const float* sinks,
                                            const float* dist_bias, int far, cudaStream_t stream) {
    return paged_attention_mma_impl(qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table,
                                    table_width, page_size, qtile_seg, qtile_tok0, n_qtiles, tokens, heads, kv_heads,
                                    head_dim, scale, window, decode_shape, num_splits, partial_o, partial_ml,
                                    num_pages, status, stream, softcap, chunk_size, sinks, dist_bias, far);
}

// ---------------------------------------------------------------------------------------------
// The same decode attention for callers that cannot allocate (see no_alloc.h). The partial
// results of the key splits go to this array in the library image instead of to memory that
// the caller or an allocator provides.
#include "no_alloc.h"

static __device__ __align__(256) unsigned char g_noalloc_scratch[TTB_NOALLOC_SCRATCH_BYTES];

#define TTB_NOALLOC_MAX_DEVICES 64
// In host code `g_noalloc_scratch` is only a handle for the symbol, not a device address; the
// address of each device's copy is looked up once, with that device current.
static float* g_noalloc_device_ptr[TTB_NOALLOC_MAX_DEVICES];

TTB_EXPORT unsigned int ttb_noalloc_scratch_bytes(void) { return TTB_NOALLOC_SCRATCH_BYTES; }

TTB_EXPORT int ttb_paged_attention_decode_noalloc(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                                  const int* seg_pos0, const void* key_pages, const void* value_pages,
                                                  const int* block_table, int table_width, int page_size, int segments,
                                                  int heads, int kv_heads, int head_dim, float scale, int window,
                                                  int num_splits, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (segments < 0 || num_splits < 1 || heads < 1 || head_dim < 1) return TTB_ERR_ARGUMENT;
    const size_t rows = (size_t)segments * heads * num_splits;
    const size_t need = rows * ((size_t)head_dim + 2) * sizeof(float);
    if (need > TTB_NOALLOC_SCRATCH_BYTES) return TTB_ERR_SCRATCH;
    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    if (device < 0 || device >= TTB_NOALLOC_MAX_DEVICES) return TTB_ERR_UNSUPPORTED;
    if (g_noalloc_device_ptr[device] == nullptr) {          // set-up, once per device
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        if (ptr == nullptr) return TTB_ERR_ARGUMENT;
        g_noalloc_device_ptr[device] = static_cast<float*>(ptr);
    }
    float* partial_o = g_noalloc_device_ptr[device];
    float* partial_ml = partial_o + rows * (size_t)head_dim;
    return ttb_paged_attention_mma(qkv, q_row_stride, out, cu_seqlens, seg_pos0, key_pages, value_pages, block_table,
                                   table_width, page_size, nullptr, nullptr, segments, segments, heads, kv_heads,
                                   head_dim, scale, window, /*decode_shape=*/1, num_splits, partial_o, partial_ml,
                                   stream);
}
