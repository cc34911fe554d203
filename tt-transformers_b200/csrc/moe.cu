// A routed feed-forward: router, grouping of (token, choice) pairs by expert, both products of the experts over
// those groups, and the weighted sum per token.
//
// route_top: z = W_r h in float32 (one block per token; every logit is summed in the same order whatever the batch
//   holds); the `top` largest logits are chosen, the lower index among equals; their weights are the softmax over
//   the chosen logits only. An optional extra row of W_r gives the shared expert's gate sigmoid(w . h).
// moe_align: counts the pairs of every expert and lays their indices out expert by expert (one block; no host read).
// moe_group_gemm: C = A W_e^T over the rows of each expert, with float32 accumulation on the CUDA cores. FIRST:
//   rows are gathered from the tokens, W_e = [gate rows; up rows], and the epilogue writes
//   g' * sigmoid(alpha g') * (u' + 1) with g' = min(g, L), u' = clamp(u, -L, L). Otherwise: rows are the pairs'
//   hidden vectors and the result goes to the pair's own row, float32. A pair's numbers do not depend on which other
//   pairs share its tile.
// moe_combine: out[t] = sum_j weight[t, j] * pair_out[t, j] (+ gate[t] * shared[t]) in float32, in the order of j.
// glu_clamped: the same activation on a dense [rows, 2 inter] product (the shared expert).
#include "common.cuh"

#define RT_THREADS 128
#define RT_MAX_EXPERTS 1024

// TPB tokens a block: a row of W_r is read once for all of them (with many tokens the reads of W_r from L2 are
// what the kernel waits for). A warp per logit row; then a warp per token selects.
template <typename T, int TPB>
__global__ void __launch_bounds__(TPB == 1 ? 1024 : 512, TPB == 1 ? 1 : 2)       // many tokens: two blocks an SM
route_top_kernel(const T* __restrict__ x, int ldx, const float* __restrict__ w_router, int width, int experts, int top,
                 int shared, int* __restrict__ choice, float* __restrict__ weight, float* __restrict__ shared_gate,
                 int tokens, int scores, const float* __restrict__ correction, float out_scale, float floor_) {
    extern __shared__ __align__(16) float rt_smem[];
    const int wpad = (width + 3) & ~3;
    float* h = rt_smem;                                   // [TPB, wpad]
    float* z = h + TPB * wpad;                            // [TPB, experts + 1]
    int* taken = reinterpret_cast<int*>(z + TPB * (experts + 1));    // [TPB, experts]
    if (TPB == 1) {      // a handful of tokens: the router's matrix on its way into L2 while the norm in front finishes
        const char* w = reinterpret_cast<const char*>(w_router);
        const size_t bytes = (size_t)(experts + (shared ? 1 : 0)) * width * sizeof(float);
        for (size_t off = (size_t)(blockIdx.x * blockDim.x + threadIdx.x) * 128; off < bytes; off += (size_t)gridDim.x * blockDim.x * 128)
            prefetch_l2(w + off);
    }
    pdl_wait();
    pdl_launch_dependents();
    const int t0 = blockIdx.x * TPB, nt = min(TPB, tokens - t0);
    if (TPB > 1 && (width & 3) == 0 && (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & (4 * sizeof(T) - 1)) == 0) {
        // four neighbouring values a load, every row's loads in flight together
        const int quads = width / 4;
        for (int q = threadIdx.x; q < TPB * quads; q += blockDim.x) {
            const int i = q / quads, c = (q - i * quads) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < nt) {
                const T* src = x + (size_t)(t0 + i) * ldx + c;
                if constexpr (sizeof(T) == 2) {
                    const uint2 raw = *reinterpret_cast<const uint2*>(src);
                    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
                    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
                    v = make_float4(lo.x, lo.y, hi.x, hi.y);
                } else {
                    v = *reinterpret_cast<const float4*>(src);
                }
            }
            *reinterpret_cast<float4*>(h + i * wpad + c) = v;
        }
    } else {
        for (int i = 0; i < TPB; ++i)
            for (int c = threadIdx.x; c < wpad; c += blockDim.x)
                h[i * wpad + c] = (i < nt && c < width) ? to_float(x[(size_t)(t0 + i) * ldx + c]) : 0.f;
    }
    for (int e = threadIdx.x; e < TPB * experts; e += blockDim.x) taken[e] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const bool vec = (width & 3) == 0;
    for (int e = warp; e < experts + (shared ? 1 : 0); e += nwarps) {
        const float* w = w_router + (size_t)e * width;
        float s[TPB];
#pragma unroll
        for (int i = 0; i < TPB; ++i) s[i] = 0.f;
        if (vec) {          // a lane's loads are independent of one another: they are in flight together
#pragma unroll 4
            for (int c = lane * 4; c < width; c += 128) {
                const float4 a = *reinterpret_cast<const float4*>(w + c);
#pragma unroll
                for (int i = 0; i < TPB; ++i) {
                    const float4 b = *reinterpret_cast<const float4*>(h + i * wpad + c);
                    s[i] = fmaf(a.x, b.x, s[i]); s[i] = fmaf(a.y, b.y, s[i]); s[i] = fmaf(a.z, b.z, s[i]); s[i] = fmaf(a.w, b.w, s[i]);
                }
            }
        } else {
            for (int c = lane; c < width; c += 32) {
                const float a = w[c];
#pragma unroll
                for (int i = 0; i < TPB; ++i) s[i] = fmaf(h[i * wpad + c], a, s[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < TPB; ++i) {
            const float r = warp_sum(s[i]);
            if (lane == 0) z[i * (experts + 1) + e] = r;
        }
    }
    __syncthreads();
    // a warp per token picks: in round j every lane looks at its share of the experts that are still free, the
    // lanes agree on the largest logit and, among equals, on the lowest index
    for (int i = warp; i < nt; i += nwarps) {
        const int t = t0 + i;
        const float* zt = z + i * (experts + 1);
        int* tk = taken + i * experts;
        float best_first = 0.f, denom = 0.f;
        for (int j = 0; j < top; ++j) {
            float best_z = -INFINITY;
            int best = 0x7fffffff;
            for (int e = lane; e < experts; e += 32) {
                // scores 2: the choice goes by the expert's own sigmoid score plus its correction
                const float v = tk[e] ? -INFINITY : (scores == 2 ? 1.f / (1.f + expf(-zt[e])) + correction[e] : zt[e]);
                if (!tk[e] && (best == 0x7fffffff || v > best_z)) { best = e; best_z = v; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float oz = __shfl_xor_sync(0xffffffffu, best_z, o);
                const int oe = __shfl_xor_sync(0xffffffffu, best, o);
                if (oe != 0x7fffffff && (best == 0x7fffffff || oz > best_z || (oz == best_z && oe < best))) { best = oe; best_z = oz; }
            }
            if (lane == 0) tk[best] = 1;
            __syncwarp();
            if (j == 0) best_first = best_z;
            const float p = scores == 2 ? 1.f / (1.f + expf(-zt[best]))
                                        : (scores == 1 ? 1.f / (1.f + expf(-best_z)) : expf(best_z - best_first));
            denom += p;
            if (lane == 0) {
                choice[(size_t)t * top + j] = best;
                weight[(size_t)t * top + j] = p;           // divided by the sum below
            }
        }
        __syncwarp();                                      // lane 0's weights are visible to the warp
        if (scores == 0)
            for (int j = lane; j < top; j += 32) weight[(size_t)t * top + j] /= denom;
        if (scores == 2)      // the chosen scores without their corrections, over their sum, times the router's scale
            for (int j = lane; j < top; j += 32) weight[(size_t)t * top + j] = weight[(size_t)t * top + j] / (denom + floor_) * out_scale;
        if (shared && lane == 0) shared_gate[t] = 1.f / (1.f + expf(-zt[experts]));
    }
}

template <typename T, int TPB>
static int route_top_launch(const void* x, int ldx, const float* w_router, int tokens, int width, int experts, int top,
                            int shared, int* choice, float* weight, float* shared_gate, int threads, int scores,
                            cudaStream_t stream, const float* correction = nullptr, float out_scale = 1.f, float floor_ = 0.f) {
    const size_t smem = ((size_t)TPB * (((width + 3) & ~3) + 2 * experts + 1)) * sizeof(float);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    static TtbOncePerDevice once;
    if (smem > 48 * 1024 && once.pending()) {
        cudaFuncSetAttribute(route_top_kernel<T, TPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        once.mark();
    }
    ttb_launch(route_top_kernel<T, TPB>, (tokens + TPB - 1) / TPB, threads, smem, stream, (const T*)x, ldx, w_router, width,
               experts, top, shared, choice, weight, shared_gate, tokens, scores, correction, out_scale, floor_);
    return ttb_launch_status();
}

// scores 0: the chosen experts' weights are the softmax over their logits; 1: each one's own sigmoid(logit), as it is;
// 2: chosen by sigmoid(logit) + correction[e], weighted by sigmoid(logit) / (sum over the chosen + floor) * out_scale.
TTB_EXPORT int ttb_route_top_corrected(const void* x, int dtype, int ldx, const float* w_router, int tokens, int width, int experts,
                                       int top, int shared, int* choice, float* weight, float* shared_gate, int scores,
                                       const float* correction, float out_scale, float floor_, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (scores < 0 || scores > 2) return TTB_ERR_UNSUPPORTED;
    if (!x || !w_router || !choice || !weight || (shared && !shared_gate) || (scores == 2 && !correction)) return TTB_ERR_ARGUMENT;
    if (experts < 1 || experts > RT_MAX_EXPERTS || top < 1 || top > experts) return TTB_ERR_UNSUPPORTED;
    if ((width & 3) == 0 && !aligned16(w_router)) return TTB_ERR_ARGUMENT;
    const int rows = experts + (shared ? 1 : 0);
    // a handful of tokens: a block per token and a warp per logit (latency); many: eight tokens a block and up to
    // sixteen warps (W_r is read once per block)
    const bool many = tokens > 64 && (size_t)8 * (width + 2 * experts + 4) * sizeof(float) <= 96 * 1024;
    const int most = many ? 16 : 32;
    const int threads = 32 * (rows < 4 ? 4 : (rows > most ? most : rows));
#define RT_LAUNCH(T)                                                                                                 \
    (many ? route_top_launch<T, 8>(x, ldx, w_router, tokens, width, experts, top, shared, choice, weight, shared_gate, threads, scores, stream, correction, out_scale, floor_) \
          : route_top_launch<T, 1>(x, ldx, w_router, tokens, width, experts, top, shared, choice, weight, shared_gate, threads, scores, stream, correction, out_scale, floor_))
    if (dtype == TTB_DTYPE_BF16) return RT_LAUNCH(__nv_bfloat16);
    if (dtype == TTB_DTYPE_F32) return RT_LAUNCH(float);
#undef RT_LAUNCH
    return TTB_ERR_UNSUPPORTED;
}

TTB_EXPORT int ttb_route_top_scored(const void* x, int dtype, int ldx, const float* w_router, int tokens, int width, int experts,
                                    int top, int shared, int* choice, float* weight, float* shared_gate, int scores,
                                    cudaStream_t stream) {
    if (scores != 0 && scores != 1) return TTB_ERR_UNSUPPORTED;
    return ttb_route_top_corrected(x, dtype, ldx, w_router, tokens, width, experts, top, shared, choice, weight, shared_gate, scores,
                                   nullptr, 1.f, 0.f, stream);
}

TTB_EXPORT int ttb_route_top(const void* x, int dtype, int ldx, const float* w_router, int tokens, int width, int experts,
                             int top, int shared, int* choice, float* weight, float* shared_gate, cudaStream_t stream) {
    return ttb_route_top_scored(x, dtype, ldx, w_router, tokens, width, experts, top, shared, choice, weight, shared_gate, 0,
                                stream);
}

// ---------------------------------------------------------------- grouping
// offsets[e] .. offsets[e + 1]: where expert e's pairs (token * top + choice rank) lie in `sorted`.
__global__ void __launch_bounds__(1024)
moe_align_kernel(const int* __restrict__ choice, int pairs, int experts, int top, int* __restrict__ offsets,
                 int* __restrict__ sorted, int* __restrict__ sorted_token, int* __restrict__ tile_info,
                 int* __restrict__ num_m_tiles, int tile_rows) {
    extern __shared__ int al_smem[];
    int* count = al_smem;                 // [experts + 1]
    pdl_wait();
    pdl_launch_dependents();
    for (int e = threadIdx.x; e <= experts; e += blockDim.x) count[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int e = choice[p];
        if ((unsigned)e < (unsigned)experts) atomicAdd(&count[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0, tiles = 0;
        for (int e = 0; e < experts; ++e) {
            const int c = count[e];
            count[e] = run;
            offsets[e] = run;
            if (tile_info != nullptr)             // row tiles of tile_rows rows, expert by expert: (expert, first row)
                for (int r = run; r < run + c; r += tile_rows) {
                    tile_info[2 * tiles] = e;
                    tile_info[2 * tiles + 1] = r;
                    ++tiles;
                }
            run += c;
        }
        offsets[experts] = run;
        if (tile_info != nullptr) *num_m_tiles = tiles;
    }
    __syncthreads();
    // every pair takes the next free place of its expert's range (a counter per expert in shared memory). Which
    // place a pair gets varies from run to run; no result depends on it, since every row of the products is
    // computed from that row alone.
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int e = choice[p];
        if ((unsigned)e >= (unsigned)experts) continue;
        const int slot = atomicAdd(&count[e], 1);
        sorted[slot] = p;
        if (sorted_token != nullptr) sorted_token[slot] = p / top;
    }
}

// sorted_token (the token of every grouped row), tile_info ((expert, first row) per row tile of tile_rows rows) and
// num_m_tiles (their count) may be null.
TTB_EXPORT int ttb_moe_align(const int* choice, int pairs, int experts, int top, int* offsets, int* sorted, int* sorted_token,
                             int* tile_info, int* num_m_tiles, int tile_rows, cudaStream_t stream) {
    if (pairs == 0) return TTB_OK;
    if (tile_info && (!num_m_tiles || tile_rows < 1)) return TTB_ERR_ARGUMENT;
    if (!choice || !offsets || !sorted || experts < 1 || experts > RT_MAX_EXPERTS) return TTB_ERR_ARGUMENT;
    ttb_launch(moe_align_kernel, 1, 1024, (size_t)(experts + 1) * sizeof(int), stream, choice, pairs, experts, top, offsets, sorted,
               sorted_token, tile_info, num_m_tiles, tile_rows);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the experts' products (CUDA cores, float32 sums)
#define MG_BM 32
#define MG_BN 64
#define MG_BK 16
#define MG_THREADS 128

// limit <= 0: no clamps and no unit offset, the plain gated unit g sigmoid(alpha g) u (alpha 1: silu(g) u).
__device__ __forceinline__ float glu_clamped(float g, float u, float limit, float alpha) {
    if (!(limit > 0.f)) return g / (1.f + expf(-alpha * g)) * u;
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
    return g / (1.f + expf(-alpha * g)) * (u + 1.f);
}

// Tile blockIdx.y of the pairs: walks the experts' groups in tiles of MG_BM rows. Returns false past the last tile.
__device__ __forceinline__ bool mg_find_tile(const int* offsets, int experts, int tile, int& expert, int& row0, int& row_end,
                                             int bm = MG_BM) {
    int seen = 0;
    for (int e = 0; e < experts; ++e) {
        const int begin = offsets[e], end = offsets[e + 1];
        const int tiles = (end - begin + bm - 1) / bm;
        if (tile < seen + tiles) {
            expert = e;
            row0 = begin + (tile - seen) * bm;
            row_end = end;
            return true;
        }
        seen += tiles;
    }
    return false;
}

template <typename TA, typename TC, bool FIRST>
__global__ void __launch_bounds__(MG_THREADS)
moe_group_gemm_kernel(const TA* __restrict__ A, int lda, const TA* __restrict__ W, long long w_expert_stride, int ldw,
                      TC* __restrict__ C, int ldc, const int* __restrict__ offsets, const int* __restrict__ sorted,
                      int experts, int top, int N, int K, float limit, float alpha) {
    __shared__ float As[MG_BK][MG_BM + 4];
    __shared__ float Ws[MG_BK][MG_BN + 4];
    __shared__ float Us[FIRST ? MG_BK : 1][MG_BN + 4];
    __shared__ int src_row[MG_BM];
    pdl_wait();
    pdl_launch_dependents();
    int expert, row0, row_end;
    if (!mg_find_tile(offsets, experts, blockIdx.y, expert, row0, row_end)) return;
    const int n0 = blockIdx.x * MG_BN;
    if (threadIdx.x < MG_BM) {
        const int r = row0 + threadIdx.x;
        // FIRST: the row of A is the pair's token; otherwise the pair's place in the grouped order
        src_row[threadIdx.x] = r < row_end ? (FIRST ? sorted[r] / top : r) : -1;
    }
    __syncthreads();
    const TA* We = W + (size_t)expert * w_expert_stride;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;      // 16 x 8 threads, each 4 rows x 4 columns
    float acc[4][4], acc_u[FIRST ? 4 : 1][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[i][j] = 0.f;
            if (FIRST) acc_u[i][j] = 0.f;
        }
    for (int k0 = 0; k0 < K; k0 += MG_BK) {
        for (int i = threadIdx.x; i < MG_BM * MG_BK; i += MG_THREADS) {
            const int r = i / MG_BK, k = i % MG_BK;
            const int src = src_row[r];
            As[k][r] = (src >= 0 && k0 + k < K) ? to_float(A[(size_t)src * lda + k0 + k]) : 0.f;
        }
        for (int i = threadIdx.x; i < MG_BN * MG_BK; i += MG_THREADS) {
            const int n = i / MG_BK, k = i % MG_BK;
            const bool in = n0 + n < N && k0 + k < K;
            Ws[k][n] = in ? to_float(We[(size_t)(n0 + n) * ldw + k0 + k]) : 0.f;
            if (FIRST) Us[k][n] = in ? to_float(We[(size_t)(N + n0 + n) * ldw + k0 + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < MG_BK; ++kk) {
            float a[4], w[4], u[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w[j] = Ws[kk][tx * 4 + j];
                if (FIRST) u[j] = Us[kk][tx * 4 + j];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
                    if (FIRST) acc_u[i][j] = fmaf(a[i], u[j], acc_u[i][j]);
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = row0 + ty * 4 + i;
        if (r >= row_end) continue;
        const size_t dst = FIRST ? (size_t)r : (size_t)sorted[r];     // hidden rows in grouped order; results by pair
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= N) continue;
            if (FIRST) C[dst * ldc + n] = from_float<TC>(glu_clamped(acc[i][j], acc_u[i][j], limit, alpha));
            else C[dst * ldc + n] = from_float<TC>(acc[i][j]);
        }
    }
}


// ---------------------------------------------------------------- the same products on the tensor cores (bfloat16)
// mma.sync m16n8k16, float32 accumulation: tiles of 64 pairs x 64 columns (FIRST: 64 gate and their 64 up rows
// of W_e), K in steps of 64 through shared memory; four warps of 16 rows each.
#define MM_BM 128
#define MM_BN 64
#define MM_BK 64
#define MM_LD (MM_BK + 8)
#define MM_THREADS 256
#define MM_STAGE_ELEMS(first) ((MM_BM + ((first) ? 2 : 1) * MM_BN) * MM_LD)

__device__ __forceinline__ void mm_ldsm_x4(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void mm_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16 bytes global -> shared past the registers; `bytes` 0 writes zeros and reads nothing
__device__ __forceinline__ void mm_cp16(void* dst, const void* src, int bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

// Tiles of 128 pairs x 64 columns (FIRST: 64 gate rows of W_e and their 64 up rows), eight warps of 16 rows, K in
// steps of 64 through two shared-memory stages: the next step's operands arrive (cp.async) under this step's products.
template <bool FIRST>
__global__ void __launch_bounds__(MM_THREADS)
moe_group_gemm_mma_kernel(const __nv_bfloat16* __restrict__ A, int lda, const __nv_bfloat16* __restrict__ W,
                          long long w_expert_stride, int ldw, void* __restrict__ C, int ldc,
                          const int* __restrict__ offsets, const int* __restrict__ sorted, int experts, int top, int N,
                          int K, float limit, float alpha) {
    extern __shared__ __align__(16) unsigned char mm_smem[];
    __nv_bfloat16* stage0 = reinterpret_cast<__nv_bfloat16*>(mm_smem);
    __shared__ int src_row[MM_BM];
    pdl_wait();
    pdl_launch_dependents();
    int expert, row0, row_end;
    if (!mg_find_tile(offsets, experts, blockIdx.y, expert, row0, row_end, MM_BM)) return;
    const int n0 = blockIdx.x * MM_BN;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
    if (tid < MM_BM) {
        const int r = row0 + tid;
        src_row[tid] = r < row_end ? (FIRST ? sorted[r] / top : r) : -1;
    }
    __syncthreads();
    const __nv_bfloat16* We = W + (size_t)expert * w_expert_stride;
    auto fetch = [&](int k0, __nv_bfloat16* st) {
        __nv_bfloat16* As = st;
        __nv_bfloat16* Ws = st + MM_BM * MM_LD;
        __nv_bfloat16* Us = Ws + MM_BN * MM_LD;
        for (int i = tid; i < MM_BM * (MM_BK / 8); i += MM_THREADS) {
            const int r = i / (MM_BK / 8), c = (i % (MM_BK / 8)) * 8;
            const int src = src_row[r];
            const bool in = src >= 0 && k0 + c < K;
            mm_cp16(As + r * MM_LD + c, in ? A + (size_t)src * lda + k0 + c : A, in ? 16 : 0);
        }
        for (int i = tid; i < MM_BN * (MM_BK / 8); i += MM_THREADS) {
            const int n = i / (MM_BK / 8), c = (i % (MM_BK / 8)) * 8;
            const bool in = n0 + n < N && k0 + c < K;
            mm_cp16(Ws + n * MM_LD + c, in ? We + (size_t)(n0 + n) * ldw + k0 + c : We, in ? 16 : 0);
            if (FIRST) mm_cp16(Us + n * MM_LD + c, in ? We + (size_t)(N + n0 + n) * ldw + k0 + c : We, in ? 16 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float acc[MM_BN / 8][4], acc_u[FIRST ? MM_BN / 8 : 1][4];
#pragma unroll
    for (int j = 0; j < MM_BN / 8; ++j) {
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        if (FIRST) acc_u[j][0] = acc_u[j][1] = acc_u[j][2] = acc_u[j][3] = 0.f;
    }
    const int steps = (K + MM_BK - 1) / MM_BK;
    fetch(0, stage0);
    for (int step = 0; step < steps; ++step) {
        const __nv_bfloat16* As = stage0 + (step & 1) * MM_STAGE_ELEMS(FIRST);
        const __nv_bfloat16* Ws = As + MM_BM * MM_LD;
        const __nv_bfloat16* Us = Ws + MM_BN * MM_LD;
        if (step + 1 < steps) {
            fetch((step + 1) * MM_BK, stage0 + ((step + 1) & 1) * MM_STAGE_ELEMS(FIRST));
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < MM_BK; kk += 16) {
            uint32_t a[4];
            mm_ldsm_x4(a, As + (warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * MM_LD + kk + (lane >> 4) * 8);
#pragma unroll
            for (int jp = 0; jp < MM_BN / 16; ++jp) {
                uint32_t b[4];
                mm_ldsm_x4(b, Ws + (jp * 16 + (lane & 7) + (lane >> 4) * 8) * MM_LD + kk + ((lane >> 3) & 1) * 8);
                mm_mma(acc[2 * jp], a, b[0], b[1]);
                mm_mma(acc[2 * jp + 1], a, b[2], b[3]);
                if (FIRST) {
                    mm_ldsm_x4(b, Us + (jp * 16 + (lane & 7) + (lane >> 4) * 8) * MM_LD + kk + ((lane >> 3) & 1) * 8);
                    mm_mma(acc_u[2 * jp], a, b[0], b[1]);
                    mm_mma(acc_u[2 * jp + 1], a, b[2], b[3]);
                }
            }
        }
        __syncthreads();              // this stage is read: the step after next may overwrite it
    }
#pragma unroll
    for (int half_row = 0; half_row < 2; ++half_row) {
        const int r = row0 + warp * 16 + g + 8 * half_row;
        if (r >= row_end) continue;
        const size_t dst = FIRST ? (size_t)r : (size_t)sorted[r];
#pragma unroll
        for (int j = 0; j < MM_BN / 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int n = n0 + 8 * j + 2 * t4 + e;
                if (n >= N) continue;
                const float v = acc[j][2 * half_row + e];
                if (FIRST)
                    reinterpret_cast<__nv_bfloat16*>(C)[dst * ldc + n] =
                        __float2bfloat16_rn(glu_clamped(v, acc_u[j][2 * half_row + e], limit, alpha));
                else
                    reinterpret_cast<float*>(C)[dst * ldc + n] = v;
            }
        }
    }
}

// first != 0: A = tokens [*, K], W = [experts, 2 N, K] (gate rows, then up rows), C = hidden [pairs, N] in the
// grouped order, type of A. first == 0: A = hidden [pairs, K], W = [experts, N, K], C = float32 [pairs, N] by pair.
TTB_EXPORT int ttb_moe_group_gemm(const void* A, int lda, const void* W, long long w_expert_stride, int ldw, void* C, int ldc,
                                  int dtype, int first, const int* offsets, const int* sorted, int pairs, int experts,
                                  int top, int N, int K, float limit, float alpha, cudaStream_t stream) {
    if (pairs == 0 || N == 0) return TTB_OK;
    if (!A || !W || !C || !offsets || !sorted || K < 1) return TTB_ERR_ARGUMENT;
    if (dtype == TTB_DTYPE_BF16 && (K & 7) == 0 && (lda & 7) == 0 && (ldw & 7) == 0 && (w_expert_stride & 7) == 0 &&
        aligned16(A) && aligned16(W)) {
        dim3 tc_grid((N + MM_BN - 1) / MM_BN, (pairs + MM_BM - 1) / MM_BM + experts);
        if (tc_grid.y > 65535) return TTB_ERR_UNSUPPORTED;
        static TtbOncePerDevice once;
        if (once.pending()) {
            cudaFuncSetAttribute(moe_group_gemm_mma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 2 * MM_STAGE_ELEMS(true) * 2);
            cudaFuncSetAttribute(moe_group_gemm_mma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 2 * MM_STAGE_ELEMS(false) * 2);
            once.mark();
        }
        if (first)
            ttb_launch(moe_group_gemm_mma_kernel<true>, tc_grid, MM_THREADS, 2 * MM_STAGE_ELEMS(true) * 2, stream, (const __nv_bfloat16*)A, lda,
                       (const __nv_bfloat16*)W, w_expert_stride, ldw, C, ldc, offsets, sorted, experts, top, N, K, limit, alpha);
        else
            ttb_launch(moe_group_gemm_mma_kernel<false>, tc_grid, MM_THREADS, 2 * MM_STAGE_ELEMS(false) * 2, stream, (const __nv_bfloat16*)A, lda,
                       (const __nv_bfloat16*)W, w_expert_stride, ldw, C, ldc, offsets, sorted, experts, top, N, K, limit, alpha);
        return ttb_launch_status();
    }
    dim3 grid((N + MG_BN - 1) / MG_BN, (pairs + MG_BM - 1) / MG_BM + experts);
    if (grid.y > 65535) return TTB_ERR_UNSUPPORTED;
#define MG_LAUNCH(TA, TC, FIRST)                                                                                     \
    ttb_launch(moe_group_gemm_kernel<TA, TC, FIRST>, grid, MG_THREADS, 0, stream, (const TA*)A, lda, (const TA*)W,   \
               w_expert_stride, ldw, (TC*)C, ldc, offsets, sorted, experts, top, N, K, limit, alpha)
    if (dtype == TTB_DTYPE_BF16) {
        if (first) MG_LAUNCH(__nv_bfloat16, __nv_bfloat16, true); else MG_LAUNCH(__nv_bfloat16, float, false);
    } else if (dtype == TTB_DTYPE_F32) {
        if (first) MG_LAUNCH(float, float, true); else MG_LAUNCH(float, float, false);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
#undef MG_LAUNCH
    return ttb_launch_status();
}


// ---------------------------------------------------------------- a handful of tokens: the experts as matrix-vector products
// Decode steps hold few (token, choice) pairs, most of them with an expert to themselves: every pair streams its
// expert's rows straight from memory, a warp per output row, no grouping. moe_gemv_first: hidden[p, :] =
// activation(W_gate,e x, W_up,e x) for pair p = token * top + j, e = choice[p]. moe_gemv_second: out[t, :] =
// sum_j weight[t, j] * W_down,e_j hidden[t * top + j] (+ gate[t] * shared[t]) in float32, j in order.
#define MV_THREADS 256
#define MV_ROWS_PER_WARP 4

// R dot products of one x (shared memory, float32) with R rows of W at once: the R loads of a step are independent
// and in flight together. Rows are given by pointer; all lanes get all R sums.
template <typename T, bool VEC, int R>
__device__ __forceinline__ void mv_dots(const T* const (&w)[R], const float* __restrict__ x, int K, int lane, float (&out)[R]) {
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = 0.f;
    if (VEC) {
#pragma unroll 2
        for (int k = lane * 8; k < K; k += 256) {
            float v[R][8];
#pragma unroll
            for (int r = 0; r < R; ++r) load8(w[r] + k, v[r]);
            const float4 xa = *reinterpret_cast<const float4*>(x + k), xb = *reinterpret_cast<const float4*>(x + k + 4);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float s = out[r];
                s = fmaf(v[r][0], xa.x, s); s = fmaf(v[r][1], xa.y, s); s = fmaf(v[r][2], xa.z, s); s = fmaf(v[r][3], xa.w, s);
                s = fmaf(v[r][4], xb.x, s); s = fmaf(v[r][5], xb.y, s); s = fmaf(v[r][6], xb.z, s); s = fmaf(v[r][7], xb.w, s);
                out[r] = s;
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) {
            const float xv = x[k];
#pragma unroll
            for (int r = 0; r < R; ++r) out[r] = fmaf(to_float(w[r][k]), xv, out[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = warp_sum(out[r]);
}

// GLU: W_e = [gate rows; up rows] and the clamped gated activation. Otherwise W_e = [rows] and hidden = relu(W_e x)^2.
template <typename T, bool VEC, bool GLU>
__global__ void __launch_bounds__(MV_THREADS)
moe_gemv_first_kernel(const T* __restrict__ x, int ldx, const T* __restrict__ W, long long w_expert_stride,
                      const int* __restrict__ choice, int experts, int top, T* __restrict__ hidden, int N, int K,
                      float limit, float alpha, int pairs, const T* __restrict__ shared_w, T* __restrict__ shared_hidden,
                      int shared_n, float shared_limit, const float* __restrict__ in_scale) {
    extern __shared__ __align__(16) float mv_x[];          // [K]
    pdl_wait();
    pdl_launch_dependents();
    int p = blockIdx.y, e = 0;
    const bool is_shared = p >= pairs;                      // rows past the pairs: the shared expert of token p - pairs
    if (is_shared) {
        W = shared_w;
        hidden = shared_hidden;
        N = shared_n;
        limit = shared_limit;
        p -= pairs;
    } else {
        e = choice[p];
    }
    const T* row = x + (size_t)(is_shared ? p : p / top) * ldx;
    if (in_scale != nullptr && !is_shared) {               // the pair's weight on its input, rounded like a stored row
        const float s = in_scale[p];
        for (int k = threadIdx.x; k < K; k += MV_THREADS) mv_x[k] = to_float(from_float<T>(to_float(row[k]) * s));
    } else {
        for (int k = threadIdx.x; k < K; k += MV_THREADS) mv_x[k] = to_float(row[k]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_begin = (blockIdx.x * (MV_THREADS / 32) + warp) * MV_ROWS_PER_WARP;
    if (n_begin >= N) return;
    const bool valid = is_shared || (unsigned)e < (unsigned)experts;
    const T* We = W + (size_t)(valid ? e : 0) * w_expert_stride;
    if (!GLU) {
        const T* rows[MV_ROWS_PER_WARP];
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i) rows[i] = We + (size_t)min(n_begin + i, N - 1) * K;
        float d[MV_ROWS_PER_WARP];
        mv_dots<T, VEC, MV_ROWS_PER_WARP>(rows, mv_x, K, lane, d);
        if (lane < MV_ROWS_PER_WARP && n_begin + lane < N) {
            float z = 0.f;
#pragma unroll
            for (int i = 0; i < MV_ROWS_PER_WARP; ++i)
                if (lane == i) z = d[i];
            z = fmaxf(z, 0.f);
            hidden[(size_t)p * N + n_begin + lane] = from_float<T>(valid ? z * z : 0.f);
        }
    } else {
        const T* rows[2 * MV_ROWS_PER_WARP];
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i) {
            const int n = min(n_begin + i, N - 1);             // rows past the end repeat the last one and are not stored
            rows[2 * i] = We + (size_t)n * K;
            rows[2 * i + 1] = We + (size_t)(N + n) * K;
        }
        float d[2 * MV_ROWS_PER_WARP];
        mv_dots<T, VEC, 2 * MV_ROWS_PER_WARP>(rows, mv_x, K, lane, d);
        if (lane < MV_ROWS_PER_WARP && n_begin + lane < N) {
            float g = 0.f, u = 0.f;
#pragma unroll
            for (int i = 0; i < MV_ROWS_PER_WARP; ++i)
                if (lane == i) { g = d[2 * i]; u = d[2 * i + 1]; }
            hidden[(size_t)p * N + n_begin + lane] = from_float<T>(valid ? glu_clamped(g, u, limit, alpha) : 0.f);
        }
    }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(MV_THREADS)
moe_gemv_second_kernel(const T* __restrict__ hidden, const T* __restrict__ W, long long w_expert_stride,
                       const int* __restrict__ choice, const float* __restrict__ weight, int experts, int top,
                       const T* __restrict__ shared_out, const float* __restrict__ shared_gate, float* __restrict__ out,
                       int N, int K, const T* __restrict__ shared_w, const T* __restrict__ shared_hidden, int shared_k) {
    extern __shared__ __align__(16) float mv_h[];          // [top, K] then [shared_k]
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.y;
    for (int i = threadIdx.x; i < top * K; i += MV_THREADS) mv_h[i] = to_float(hidden[(size_t)t * top * K + i]);
    if (shared_w != nullptr)
        for (int i = threadIdx.x; i < shared_k; i += MV_THREADS) mv_h[top * K + i] = to_float(shared_hidden[(size_t)t * shared_k + i]);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_begin = (blockIdx.x * (MV_THREADS / 32) + warp) * MV_ROWS_PER_WARP;
    if (n_begin >= N) return;
    float acc[MV_ROWS_PER_WARP];
#pragma unroll
    for (int i = 0; i < MV_ROWS_PER_WARP; ++i) acc[i] = 0.f;
    for (int j = 0; j < top; ++j) {
        const int e = choice[(size_t)t * top + j];
        if ((unsigned)e >= (unsigned)experts) continue;
        const T* rows[MV_ROWS_PER_WARP];
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i)
            rows[i] = W + (size_t)e * w_expert_stride + (size_t)min(n_begin + i, N - 1) * K;
        float d[MV_ROWS_PER_WARP];
        mv_dots<T, VEC, MV_ROWS_PER_WARP>(rows, mv_h + (size_t)j * K, K, lane, d);
        const float wj = weight != nullptr ? weight[(size_t)t * top + j] : 1.f;
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i) acc[i] = fmaf(wj, d[i], acc[i]);
    }
    if (shared_w != nullptr) {                  // the shared expert's down product, times the token's gate
        const T* rows[MV_ROWS_PER_WARP];
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i) rows[i] = shared_w + (size_t)min(n_begin + i, N - 1) * shared_k;
        float d[MV_ROWS_PER_WARP];
        mv_dots<T, VEC, MV_ROWS_PER_WARP>(rows, mv_h + (size_t)top * K, shared_k, lane, d);
        const float sg = shared_gate[t];
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i) acc[i] = fmaf(sg, d[i], acc[i]);
    }
    if (lane < MV_ROWS_PER_WARP && n_begin + lane < N) {
        float v = 0.f;
#pragma unroll
        for (int i = 0; i < MV_ROWS_PER_WARP; ++i)
            if (lane == i) v = acc[i];
        const int n = n_begin + lane;
        if (shared_out != nullptr) v = fmaf(shared_gate[t], to_float(shared_out[(size_t)t * N + n]), v);
        out[(size_t)t * N + n] = v;
    }
}

// x [tokens, width]; w_gate_up [experts, 2 inter, width]; w_down [experts, width, inter]; hidden: scratch
// [tokens * top, inter] of the compute type; out float32 [tokens, width]. The shared expert either comes as its
// finished output (shared_out, compute type) or as its weights (shared_gate_up [2 shared_inter, width], shared_down
// [width, shared_inter], scratch shared_hidden [tokens, shared_inter]) and then runs inside the two kernels; or not at all.
// ttb_moe_gemv_plain: experts without a gate, y = W_down relu(W_up x)^2, w_up [experts, inter, width]; no shared expert.
static int moe_gemv_launch(const void* x, int ldx, const void* w_gate_up, const void* w_down, const int* choice,
                           const float* weight, void* hidden, const void* shared_out, const float* shared_gate, float* out,
                           int dtype, int tokens, int experts, int top, int inter, int width, float limit, float alpha,
                           const void* shared_gate_up, const void* shared_down, void* shared_hidden, int shared_inter,
                           float shared_limit, bool glu, cudaStream_t stream, const float* in_scale);

TTB_EXPORT int ttb_moe_gemv_plain(const void* x, int ldx, const void* w_up, const void* w_down, const int* choice,
                                  const float* weight, void* hidden, float* out, int dtype, int tokens, int experts, int top,
                                  int inter, int width, cudaStream_t stream) {
    return moe_gemv_launch(x, ldx, w_up, w_down, choice, weight, hidden, nullptr, nullptr, out, dtype, tokens, experts, top, inter,
                           width, 0.f, 0.f, nullptr, nullptr, nullptr, 0, 0.f, false, stream, nullptr);
}

TTB_EXPORT int ttb_moe_gemv(const void* x, int ldx, const void* w_gate_up, const void* w_down, const int* choice,
                            const float* weight, void* hidden, const void* shared_out, const float* shared_gate, float* out,
                            int dtype, int tokens, int experts, int top, int inter, int width, float limit, float alpha,
                            const void* shared_gate_up, const void* shared_down, void* shared_hidden, int shared_inter,
                            float shared_limit, cudaStream_t stream) {
    return moe_gemv_launch(x, ldx, w_gate_up, w_down, choice, weight, hidden, shared_out, shared_gate, out, dtype, tokens, experts,
                           top, inter, width, limit, alpha, shared_gate_up, shared_down, shared_hidden, shared_inter, shared_limit,
                           true, stream, nullptr);
}

// Gated experts whose weight multiplies their INPUT: hidden = act(W_gate,e (s x), W_up,e (s x)) with s = in_scale[pair]
// (s x rounded to the compute type), out[t] = sum_j W_down,e_j hidden[t * top + j]. limit <= 0: silu(g) u for alpha 1.
TTB_EXPORT int ttb_moe_gemv_scaled(const void* x, int ldx, const void* w_gate_up, const void* w_down, const int* choice,
                                   const float* in_scale, void* hidden, float* out, int dtype, int tokens, int experts, int top,
                                   int inter, int width, float limit, float alpha, cudaStream_t stream) {
    if (!in_scale) return TTB_ERR_ARGUMENT;
    return moe_gemv_launch(x, ldx, w_gate_up, w_down, choice, nullptr, hidden, nullptr, nullptr, out, dtype, tokens, experts,
                           top, inter, width, limit, alpha, nullptr, nullptr, nullptr, 0, 0.f, true, stream, in_scale);
}

static int moe_gemv_launch(const void* x, int ldx, const void* w_gate_up, const void* w_down, const int* choice,
                           const float* weight, void* hidden, const void* shared_out, const float* shared_gate, float* out,
                           int dtype, int tokens, int experts, int top, int inter, int width, float limit, float alpha,
                           const void* shared_gate_up, const void* shared_down, void* shared_hidden, int shared_inter,
                           float shared_limit, bool glu, cudaStream_t stream, const float* in_scale) {
    if (tokens == 0) return TTB_OK;
    if (!x || !w_gate_up || !w_down || !choice || !(weight || in_scale) || !hidden || !out) return TTB_ERR_ARGUMENT;
    if ((shared_out || shared_gate_up) && !shared_gate) return TTB_ERR_ARGUMENT;
    if (shared_gate_up && (!shared_down || !shared_hidden || shared_inter < 1 || shared_out)) return TTB_ERR_ARGUMENT;
    const int pairs = tokens * top;
    const int sk = shared_gate_up ? shared_inter : 0;
    if (pairs + tokens > 65535) return TTB_ERR_UNSUPPORTED;
    const size_t smem1 = (size_t)width * sizeof(float), smem2 = ((size_t)top * inter + sk) * sizeof(float);
    if (smem1 > 48 * 1024 || smem2 > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    const int per_block = (MV_THREADS / 32) * MV_ROWS_PER_WARP;
    const int widest = inter > sk ? inter : sk;
    dim3 g1((widest + per_block - 1) / per_block, pairs + (shared_gate_up ? tokens : 0)), g2((width + per_block - 1) / per_block, tokens);
    const long long s1 = (glu ? 2LL : 1LL) * inter * width, s2 = (long long)width * inter;
#define MV_LAUNCH(T, VEC)                                                                                            \
    do {                                                                                                             \
        if (glu)                                                                                                     \
            ttb_launch(moe_gemv_first_kernel<T, VEC, true>, g1, MV_THREADS, smem1, stream, (const T*)x, ldx, (const T*)w_gate_up, s1, \
                       choice, experts, top, (T*)hidden, inter, width, limit, alpha, pairs, (const T*)shared_gate_up, \
                       (T*)shared_hidden, sk, shared_limit, in_scale);                                               \
        else                                                                                                         \
            ttb_launch(moe_gemv_first_kernel<T, VEC, false>, g1, MV_THREADS, smem1, stream, (const T*)x, ldx, (const T*)w_gate_up, s1, \
                       choice, experts, top, (T*)hidden, inter, width, limit, alpha, pairs, (const T*)shared_gate_up, \
                       (T*)shared_hidden, sk, shared_limit, in_scale);                                               \
        ttb_launch(moe_gemv_second_kernel<T, VEC>, g2, MV_THREADS, smem2, stream, (const T*)hidden, (const T*)w_down, s2,  \
                   choice, weight, experts, top, (const T*)shared_out, shared_gate, out, width, inter,               \
                   (const T*)(shared_gate_up ? shared_down : nullptr), (const T*)shared_hidden, sk);                 \
    } while (0)
    const bool vec = (width & 7) == 0 && (inter & 7) == 0 && (sk & 7) == 0 && aligned32(w_gate_up) && aligned32(w_down) &&
                     (!shared_gate_up || (aligned32(shared_gate_up) && aligned32(shared_down)));
    if (dtype == TTB_DTYPE_BF16) { if (vec) MV_LAUNCH(__nv_bfloat16, true); else MV_LAUNCH(__nv_bfloat16, false); }
    else if (dtype == TTB_DTYPE_F32) { if (vec) MV_LAUNCH(float, true); else MV_LAUNCH(float, false); }
    else return TTB_ERR_UNSUPPORTED;
#undef MV_LAUNCH
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the weighted sum per token
template <typename TS>
__global__ void moe_combine_kernel(const float* __restrict__ pair_out, const float* __restrict__ weight, int top,
                                   const TS* __restrict__ shared_out, const float* __restrict__ shared_gate,
                                   float* __restrict__ out, int width) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const float sg = shared_out != nullptr ? shared_gate[t] : 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        float s = 0.f;
        for (int j = 0; j < top; ++j)
            s = fmaf(weight != nullptr ? weight[(size_t)t * top + j] : 1.f, pair_out[((size_t)t * top + j) * width + c], s);
        if (shared_out != nullptr) s = fmaf(sg, to_float(shared_out[(size_t)t * width + c]), s);
        out[(size_t)t * width + c] = s;
    }
}

TTB_EXPORT int ttb_moe_combine(const float* pair_out, const float* weight, int top, const void* shared_out, int shared_dtype,
                               const float* shared_gate, float* out, int tokens, int width, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!pair_out || !out || (shared_out && !shared_gate)) return TTB_ERR_ARGUMENT;       // weight null: every weight is 1
    if (shared_out && shared_dtype == TTB_DTYPE_BF16)
        ttb_launch(moe_combine_kernel<__nv_bfloat16>, tokens, 256, 0, stream, pair_out, weight, top,
                   (const __nv_bfloat16*)shared_out, shared_gate, out, width);
    else
        ttb_launch(moe_combine_kernel<float>, tokens, 256, 0, stream, pair_out, weight, top, (const float*)shared_out,
                   shared_gate, out, width);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the activation on a dense product
template <typename T>
__global__ void glu_clamped_kernel(const T* __restrict__ gate_up, T* __restrict__ out, int rows, int inter, float limit,
                                   float alpha) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)rows * inter;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / inter, c = i % inter;
        out[i] = from_float<T>(glu_clamped(to_float(gate_up[r * 2 * inter + c]), to_float(gate_up[r * 2 * inter + inter + c]),
                                           limit, alpha));
    }
}

TTB_EXPORT int ttb_glu_clamped(const void* gate_up, void* out, int dtype, int rows, int inter, float limit, float alpha,
                               cudaStream_t stream) {
    if (rows == 0 || inter == 0) return TTB_OK;
    if (!gate_up || !out) return TTB_ERR_ARGUMENT;
    const size_t total = (size_t)rows * inter;
    const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(glu_clamped_kernel<__nv_bfloat16>, blocks, 256, 0, stream, (const __nv_bfloat16*)gate_up, (__nv_bfloat16*)out,
                   rows, inter, limit, alpha);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(glu_clamped_kernel<float>, blocks, 256, 0, stream, (const float*)gate_up, (float*)out, rows, inter, limit, alpha);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// ---------------------------------------------------------------- rows gathered with a weight on each
// out[i, :] = scale[pair_of[i]] * x[token_of[i], :], rounded to the rows' type: the inputs of experts whose weight stands
// before their activation, laid out in the grouped order.
template <typename T>
__global__ void gather_rows_scaled_kernel(const T* __restrict__ x, int ldx, const int* __restrict__ token_of,
                                          const int* __restrict__ pair_of, const float* __restrict__ scale, T* __restrict__ out,
                                          int width) {
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x;
    const T* src = x + (size_t)token_of[i] * ldx;
    const float s = scale[pair_of[i]];
    for (int c = threadIdx.x; c < width; c += blockDim.x) out[(size_t)i * width + c] = from_float<T>(to_float(src[c]) * s);
}

TTB_EXPORT int ttb_gather_rows_scaled(const void* x, int dtype, int ldx, const int* token_of, const int* pair_of,
                                      const float* scale, void* out, int rows, int width, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!x || !token_of || !pair_of || !scale || !out) return TTB_ERR_ARGUMENT;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(gather_rows_scaled_kernel<__nv_bfloat16>, rows, 128, 0, stream, (const __nv_bfloat16*)x, ldx, token_of, pair_of,
                   scale, (__nv_bfloat16*)out, width);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(gather_rows_scaled_kernel<float>, rows, 128, 0, stream, (const float*)x, ldx, token_of, pair_of, scale,
                   (float*)out, width);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
