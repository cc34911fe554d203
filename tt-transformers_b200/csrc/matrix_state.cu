// Mixers with a float32 matrix state per head and request, walked token by token:
//
//   shifted_state:  o_t = (S + diag(u) k_t v_t^T)^T r_t;  S <- diag(w_t) S + k_t v_t^T            (S: dim x dim)
//                   then per head o / rms(o), times a weight per element, times silu(gate)
//   delta_rule:     S <- diag(g_t) S;  d = beta_t (v_t - S^T k_t);  S <- S + k_t d^T;  o_t = S^T q_t   (S: dim x vdim)
//                   q, k made unit vectors per head (q also times dim^-1/2) on the way in; then per head o / rms(o),
//                   times a weight per value channel, times sigmoid(gate)
//
// and what stands before them: token_shift (the five mixes of a token with the token before), lowrank_expand (the second
// half of a low-rank map in float32 with the decays' nonlinearities), add_row_vector.
//
// The walk: a block per (segment, head). Thread (c, g) keeps rows g*DR .. g*DR+DR-1 of column c of the state in
// registers; sums over the rows of a column go through shared memory (one barrier per sum, buffers in turn). Tokens come
// in tiles of MS_TILE through shared memory; a tile's outputs are normed and written by the whole block. Every state
// element is updated by one thread in the order of the tokens, so a request's result does not depend on how it was cut
// into steps or what else the batch holds. Decays arrive as logarithms (float32, never positive) and are exponentiated here.
//
// Long segments run as parts of `part_len` tokens side by side, in three launches. Both recurrences are linear in the
// state, S_end = M S_start + E, column by column: (1) every part walks from a zero state to its E, and, for the delta
// rule, D more columns that start as the identity and are fed zeros as values, which end as M (the token-shift state's M
// is diagonal: the product of the part's decays, kept as the sum of their logarithms); (2) a block per head folds the
// parts in order, S_(p+1) = M_p S_p + E_p, from the request's state, leaves every part's start state and the
// request's new state; (3) every part walks again from its start state and writes its outputs. Parts start at multiples
// of part_len from the first token that a step brings for a request.
#include "common.cuh"

#define MS_TILE 16
#define MS_MAX_THREADS 1024

__device__ __forceinline__ float ms_load(const void* p, int dtype, size_t i) {
    return dtype == TTB_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                                   : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void ms_store(void* p, int dtype, size_t i, float v) {
    if (dtype == TTB_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}
__device__ __forceinline__ float ms_sigmoid(float v) { return 1.f / (1.f + expf(-v)); }
// Four neighbouring values of a row vector in shared memory, rows from `row` on; beyond `rows` zeros (a state row that
// does not exist is multiplied by zeros and stays zero). vec: the vector is 16-byte aligned at every multiple of four.
__device__ __forceinline__ float4 ms_row4(const float* v, int row, int rows, bool vec) {
    if (vec) return row < rows ? *reinterpret_cast<const float4*>(v + row) : make_float4(0.f, 0.f, 0.f, 0.f);
    return make_float4(row < rows ? v[row] : 0.f, row + 1 < rows ? v[row + 1] : 0.f, row + 2 < rows ? v[row + 2] : 0.f,
                       row + 3 < rows ? v[row + 3] : 0.f);
}

// ---------------------------------------------------------------- token shift
// out[t, s, c] = x[t, c] + (before[t, c] - x[t, c]) * mu[s, c]; before = the segment's token in front, or the request's
// kept input for the segment's first token. The kept input is replaced later, by the walk.
__global__ void __launch_bounds__(256)
token_shift_kernel(const void* __restrict__ x, int dtype, int ldx, const float* __restrict__ mu, int mixes,
                   const int* __restrict__ seg_of_token, const int* __restrict__ cu_seqlens, const int* __restrict__ slots,
                   const void* __restrict__ kept, void* __restrict__ out, int tokens, int width) {
    pdl_wait();
    pdl_launch_dependents();
    // blockIdx.y: which run of 256 columns (a handful of tokens still fill the device with blocks)
    for (int t = blockIdx.x; t < tokens; t += gridDim.x) {
        const int seg = seg_of_token[t];
        const bool first = t == cu_seqlens[seg];
        const size_t kept_row = (size_t)slots[seg] * width;
        for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < width; c += gridDim.y * blockDim.x) {
            const float cur = ms_load(x, dtype, (size_t)t * ldx + c);
            const float before = first ? ms_load(kept, dtype, kept_row + c) : ms_load(x, dtype, (size_t)(t - 1) * ldx + c);
            const float diff = before - cur;
            for (int s = 0; s < mixes; ++s)
                ms_store(out, dtype, ((size_t)t * mixes + s) * width + c, fmaf(diff, mu[(size_t)s * width + c], cur));
        }
    }
}

TTB_EXPORT int ttb_token_shift(const void* x, int dtype, int ldx, const float* mu, int mixes, const int* seg_of_token,
                               const int* cu_seqlens, const int* slots, const void* kept, void* out, int tokens, int width,
                               cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!x || !mu || !seg_of_token || !cu_seqlens || !slots || !kept || !out || mixes < 1 || width < 1) return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    const int runs = tokens >= 148 * 4 ? 1 : (width + 255) / 256 < 64 ? (width + 255) / 256 : 64;
    ttb_launch(token_shift_kernel, dim3(tokens < 148 * 8 ? tokens : 148 * 8, runs), 256, 0, stream, x, dtype, ldx, mu, mixes,
               seg_of_token, cu_seqlens, slots, kept, out, tokens, width);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the second half of a low-rank map
// out[t, n] = f(sum_r act(in[t, r]) W[n, r] + bias[n]), float32 arithmetic; in float32 [tokens, ld_in]; W [N, rank] of
// the compute type. act: 0 none, 1 tanh. f: 0 z; 1 -exp(z); 2 -rate[n / (N / heads)] * softplus(z).
#define LR_TOKENS 32        // tokens a block
#define LR_RANK 64          // the rank in tiles of this many
#define LR_LD (LR_RANK + 4) // a row in shared memory: 16-byte aligned, and the eight threads of a vector load in different banks
// A block of 256 threads takes LR_TOKENS tokens and 32 CPT columns: thread (cn, tg) the columns cn + 32 k (k < CPT) and the
// tokens 4 tg .. 4 tg + 3, 4 CPT sums in registers; inputs (behind their activation) and weights pass shared memory in
// tiles of LR_RANK and are read four values a load. CPT 4 for prompt portions, 1 for a handful of tokens (more blocks,
// fewer loads in a row before the first product).
template <int CPT>
__global__ void __launch_bounds__(256)
lowrank_expand_kernel(const float* __restrict__ in, int ld_in, const void* __restrict__ w, int w_dtype,
                      const float* __restrict__ bias, const float* __restrict__ rate, int per_head, int act, int f,
                      float* __restrict__ out, int tokens, int N, int rank) {
    constexpr int COLS = 32 * CPT;
    __shared__ __align__(16) float xs[LR_TOKENS][LR_LD];
    __shared__ __align__(16) float ws[COLS][LR_LD];
    pdl_wait();
    pdl_launch_dependents();
    const int t0 = blockIdx.x * LR_TOKENS, n0 = blockIdx.y * COLS;
    const int cn = threadIdx.x & 31, tg = threadIdx.x >> 5;
    float acc[CPT][4];
#pragma unroll
    for (int k = 0; k < CPT; ++k)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[k][q] = 0.f;
    for (int r0 = 0; r0 < rank; r0 += LR_RANK) {
        const int nr = min(LR_RANK, rank - r0);
        __syncthreads();
        // tiles are filled to LR_RANK with zeros, so that the products need no bound
#pragma unroll 4
        for (int i = threadIdx.x; i < LR_TOKENS * LR_RANK; i += 256) {
            const int tt = i / LR_RANK, r = i - tt * LR_RANK;
            const float v = (t0 + tt < tokens && r < nr) ? in[(size_t)(t0 + tt) * ld_in + r0 + r] : 0.f;
            xs[tt][r] = act == 1 ? tanhf(v) : v;
        }
#pragma unroll 8
        for (int i = threadIdx.x; i < COLS * LR_RANK; i += 256) {
            const int c = i / LR_RANK, r = i - c * LR_RANK;
            ws[c][r] = (n0 + c < N && r < nr) ? ms_load(w, w_dtype, (size_t)(n0 + c) * rank + r0 + r) : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int r = 0; r < LR_RANK; r += 4) {
            float4 xv[4], wv[CPT];
#pragma unroll
            for (int q = 0; q < 4; ++q) xv[q] = *reinterpret_cast<const float4*>(&xs[tg * 4 + q][r]);
#pragma unroll
            for (int k = 0; k < CPT; ++k) wv[k] = *reinterpret_cast<const float4*>(&ws[cn + 32 * k][r]);
#pragma unroll
            for (int k = 0; k < CPT; ++k)
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    acc[k][q] = fmaf(xv[q].w, wv[k].w, fmaf(xv[q].z, wv[k].z, fmaf(xv[q].y, wv[k].y, fmaf(xv[q].x, wv[k].x, acc[k][q]))));
        }
    }
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
        const int n = n0 + cn + 32 * k;
        if (n >= N) continue;
        const float b = bias != nullptr ? bias[n] : 0.f;
        const float rt = f == 2 ? rate[n / per_head] : 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int t = t0 + tg * 4 + q;
            if (t >= tokens) continue;
            float z = acc[k][q] + b;
            if (f == 1) z = -expf(z);
            else if (f == 2) z = -rt * (z > 20.f ? z : log1pf(expf(z)));
            out[(size_t)t * N + n] = z;
        }
    }
}

TTB_EXPORT int ttb_lowrank_expand(const float* in, int ld_in, const void* w, int w_dtype, const float* bias, const float* rate,
                                  int heads, int act, int f, float* out, int tokens, int N, int rank, cudaStream_t stream) {
    if (tokens == 0 || N == 0) return TTB_OK;
    if (!in || !w || !out || rank < 1 || (f == 2 && (!rate || heads < 1 || N % heads))) return TTB_ERR_ARGUMENT;
    if (w_dtype != TTB_DTYPE_BF16 && w_dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    if (act < 0 || act > 1 || f < 0 || f > 2) return TTB_ERR_UNSUPPORTED;
    const int cpt = tokens <= 2 * LR_TOKENS ? 1 : 4;
    const int by = (N + 32 * cpt - 1) / (32 * cpt);
    if (by > 65535) return TTB_ERR_UNSUPPORTED;
    dim3 grid((tokens + LR_TOKENS - 1) / LR_TOKENS, by);
    if (cpt == 1)
        ttb_launch(lowrank_expand_kernel<1>, grid, 256, 0, stream, in, ld_in, w, w_dtype, bias, rate, f == 2 ? N / heads : 1, act, f,
                   out, tokens, N, rank);
    else
        ttb_launch(lowrank_expand_kernel<4>, grid, 256, 0, stream, in, ld_in, w, w_dtype, bias, rate, f == 2 ? N / heads : 1, act, f,
                   out, tokens, N, rank);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- x += vector, row by row
__global__ void add_row_vector_kernel(void* __restrict__ x, int dtype, int ld, const float* __restrict__ vec, int rows, int width) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)rows * width;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / width, c = i - r * width;
        ms_store(x, dtype, r * ld + c, ms_load(x, dtype, r * ld + c) + vec[c]);
    }
}

TTB_EXPORT int ttb_add_row_vector(void* x, int dtype, int ld, const float* vec, int rows, int width, cudaStream_t stream) {
    if (rows == 0 || width == 0) return TTB_OK;
    if (!x || !vec) return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    const size_t total = (size_t)rows * width;
    const int blocks = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
    ttb_launch(add_row_vector_kernel, blocks, 256, 0, stream, x, dtype, ld, vec, rows, width);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the walks
struct MsArgs {
    // shifted_state: a = r, b = k, c = v, gate = silu gate (all [T, heads * dim] of the compute type, row strides below)
    // delta_rule:    a = q, b = k (heads of kv_heads, [T, .] columns of `conv`), c = v; gate float32 [T, heads * vdim]
    const void* a; const void* b; const void* c; const void* gate;
    long long ld_a, ld_b, ld_c, ld_gate;
    int dtype;                   // of a, b, c, out, kept
    int gate_dtype;
    const float* log_decay;      // [T, heads * dim]
    const float* bonus;          // shifted_state: [heads, dim]
    const float* beta; int ld_beta;   // delta_rule: logits [T, heads] with a row stride
    const float* norm_w;         // shifted_state: [heads * dim]; delta_rule: [vdim]
    float eps;
    const int* cu_seqlens; const int* slots;
    float* state;                // [slots, heads, D, V]
    void* kept;                  // shifted_state: [slots, width]; delta_rule: [slots, taps - 1, channels]
    const void* raw; long long ld_raw;   // what the kept inputs are refreshed from: x [T, width], or the convolutions' inputs [T, channels]
    int width;                   // shifted_state: the model width; delta_rule: channels
    int taps;
    void* out;                   // [T, heads * V]
    int heads, kv_heads, D, V, R, write;
    int mode;                    // 0: the whole segment; 1: a part from zero to its end state (and transition); 2: a part from its start state
    int parts, part_len;
    float* part_end;             // [segments, heads, parts, D, V (+ D for the delta rule)]
    float* part_start;           // [segments, heads, parts, D, V]
    float* part_log;             // shifted_state: [segments, heads, parts, D], the sums of the parts' log decays
};

template <bool DELTA> static int ms_launch_mode(MsArgs& p, int segments, cudaStream_t stream);

template <int DR, bool DELTA, int CAP>
__global__ void __launch_bounds__(CAP, DR == 8 ? 2 : 1)
matrix_state_walk_kernel(const MsArgs p) {
    extern __shared__ __align__(16) float ms_smem[];
    const int D = p.D, V = p.V, R = p.R;
    float* sa = ms_smem;                       // [TILE, D]  r or q
    float* sb = sa + MS_TILE * D;              // [TILE, D]  k
    float* sw = sb + MS_TILE * D;              // [TILE, D]  decay
    float* sbonus = sw + MS_TILE * D;          // [D]
    float* sc = sbonus + D;                    // [TILE, V]  v
    float* so = sc + MS_TILE * V;              // [TILE, V]  outputs
    float* part_sums = so + MS_TILE * V;       // [2, R, V (+ D)]
    float* sbeta = part_sums + 2 * R * (V + (DELTA ? D : 0));   // [TILE]
    float* sscale = sbeta + MS_TILE;           // [TILE, 2]: unit-norm factors of q and k (delta), then the outputs' norm
    pdl_wait();
    pdl_launch_dependents();
    const int seg = blockIdx.x, head = blockIdx.y, part = blockIdx.z;
    const int kvh = DELTA ? head / (p.heads / p.kv_heads) : head;
    const int tid = threadIdx.x, nthreads = blockDim.x;
    const int VA = (DELTA && p.mode == 1) ? V + D : V;         // columns walked: the transition's ride along in mode 1
    const int col = tid % VA, grp = tid / VA;
    const bool active = grp < R;
    const int row0 = grp * DR;
    const int start = p.cu_seqlens[seg], len = p.cu_seqlens[seg + 1] - start;
    const int t_begin = p.mode == 0 ? 0 : part * p.part_len;
    const int t_end = p.mode == 0 ? len : min(len, t_begin + p.part_len);
    if (p.mode != 0 && t_begin >= t_end) return;
    const int slot = p.slots[seg];
    const size_t part_index = ((size_t)seg * p.heads + head) * p.parts + part;
    float* state = p.state + ((size_t)slot * p.heads + head) * D * V;
    float S[DR];
#pragma unroll
    for (int i = 0; i < DR; ++i) {
        S[i] = 0.f;
        if (active && row0 + i < D) {
            if (p.mode == 0) S[i] = state[(size_t)(row0 + i) * V + col];
            else if (p.mode == 2) S[i] = p.part_start[part_index * D * V + (size_t)(row0 + i) * V + col];
            else if (col >= V) S[i] = (row0 + i == col - V) ? 1.f : 0.f;
        }
    }
    if (!DELTA)
        for (int d = tid; d < D; d += nthreads) sbonus[d] = p.bonus[(size_t)head * D + d];
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
    const bool vec = (D & 3) == 0;                 // row vectors in shared memory start on 16-byte boundaries
    int turn = 0;
    for (int t0 = t_begin; t0 < t_end; t0 += MS_TILE) {
        const int nt = min(MS_TILE, t_end - t0);
        __syncthreads();                       // the tile before is written out
        for (int i = tid; i < nt * D; i += nthreads) {
            const int tt = i / D, d = i - tt * D;
            const size_t t = (size_t)(start + t0 + tt);
            sa[i] = ms_load(p.a, p.dtype, t * p.ld_a + (size_t)kvh * D + d);
            sb[i] = ms_load(p.b, p.dtype, t * p.ld_b + (size_t)kvh * D + d);
            sw[i] = expf(p.log_decay[t * ((size_t)p.heads * D) + (size_t)head * D + d]);
        }
        for (int i = tid; i < nt * V; i += nthreads) {
            const int tt = i / V, c = i - tt * V;
            sc[i] = ms_load(p.c, p.dtype, (size_t)(start + t0 + tt) * p.ld_c + (size_t)head * V + c);
        }
        if (DELTA) {
            for (int tt = tid; tt < nt; tt += nthreads) sbeta[tt] = ms_sigmoid(p.beta[(size_t)(start + t0 + tt) * p.ld_beta + head]);
            __syncthreads();
            for (int i = warp; i < 2 * nt; i += nwarps) {          // unit vectors: a warp per (token, q or k)
                const float* src = (i & 1 ? sb : sa) + (i >> 1) * D;
                float s = 0.f;
                for (int d = lane; d < D; d += 32) s = fmaf(src[d], src[d], s);
                s = warp_sum(s);
                if (lane == 0) sscale[i] = (1.f / sqrtf(s + 1e-6f)) * (i & 1 ? 1.f : 1.f / sqrtf((float)D));
            }
            __syncthreads();
            for (int i = tid; i < nt * D; i += nthreads) {
                const int tt = i / D;
                sa[i] *= sscale[2 * tt];
                sb[i] *= sscale[2 * tt + 1];
            }
        }
        __syncthreads();
        for (int tt = 0; tt < nt; ++tt) {
            const float* a = sa + tt * D;
            const float* b = sb + tt * D;
            const float* w = sw + tt * D;
            // the sum of a column over its row groups: through shared memory (buffers in turn, one barrier), or, where a
            // thread holds the whole column (R == 1), the thread's own number and no barrier at all
#define MS_COLUMN_SUM(result, mine_value, everybody)                                             \
            do {                                                                                 \
                if (R == 1) {                                                                    \
                    result = (mine_value);                                                       \
                } else {                                                                         \
                    float* slot_ = part_sums + (size_t)turn * R * VA;                            \
                    if (active) slot_[grp * VA + col] = (mine_value);                            \
                    __syncthreads();                                                             \
                    float total_ = 0.f;                                                          \
                    if ((everybody) || grp == 0) {      /* up to eight groups without a loop */  \
                        _Pragma("unroll")                                                        \
                        for (int g = 0; g < 8; ++g)                                              \
                            if (g < R) total_ += slot_[g * VA + col];                            \
                        for (int g = 8; g < R; ++g) total_ += slot_[g * VA + col];               \
                    }                                                                            \
                    result = total_;                                                             \
                    turn ^= 1;                                                                   \
                }                                                                                \
            } while (0)
            if (DELTA) {
                float s4[4] = {0.f, 0.f, 0.f, 0.f};              // four chains side by side instead of one of DR links
                if (active) {
#pragma unroll
                    for (int i = 0; i < DR; i += 4) {
                        const float4 wv = ms_row4(w, row0 + i, D, vec), bv = ms_row4(b, row0 + i, D, vec);
                        S[i] *= wv.x; S[i + 1] *= wv.y; S[i + 2] *= wv.z; S[i + 3] *= wv.w;
                        s4[0] = fmaf(S[i], bv.x, s4[0]); s4[1] = fmaf(S[i + 1], bv.y, s4[1]);
                        s4[2] = fmaf(S[i + 2], bv.z, s4[2]); s4[3] = fmaf(S[i + 3], bv.w, s4[3]);
                    }
                }
                float got;
                MS_COLUMN_SUM(got, (s4[0] + s4[1]) + (s4[2] + s4[3]), true);
                const float d = sbeta[tt] * ((col < V ? sc[tt * V + col] : 0.f) - got);
                if (p.mode == 1) {                  // end states only: nobody reads this token's output
                    if (active) {
#pragma unroll
                        for (int i = 0; i < DR; i += 4) {
                            const float4 bv = ms_row4(b, row0 + i, D, vec);
                            S[i] = fmaf(bv.x, d, S[i]); S[i + 1] = fmaf(bv.y, d, S[i + 1]);
                            S[i + 2] = fmaf(bv.z, d, S[i + 2]); S[i + 3] = fmaf(bv.w, d, S[i + 3]);
                        }
                    }
                } else {
                    s4[0] = s4[1] = s4[2] = s4[3] = 0.f;
                    if (active) {
#pragma unroll
                        for (int i = 0; i < DR; i += 4) {
                            const float4 bv = ms_row4(b, row0 + i, D, vec), av = ms_row4(a, row0 + i, D, vec);
                            S[i] = fmaf(bv.x, d, S[i]); S[i + 1] = fmaf(bv.y, d, S[i + 1]);
                            S[i + 2] = fmaf(bv.z, d, S[i + 2]); S[i + 3] = fmaf(bv.w, d, S[i + 3]);
                            s4[0] = fmaf(S[i], av.x, s4[0]); s4[1] = fmaf(S[i + 1], av.y, s4[1]);
                            s4[2] = fmaf(S[i + 2], av.z, s4[2]); s4[3] = fmaf(S[i + 3], av.w, s4[3]);
                        }
                    }
                    float o;
                    MS_COLUMN_SUM(o, (s4[0] + s4[1]) + (s4[2] + s4[3]), false);
                    if (grp == 0) so[tt * V + col] = o;
                }
            } else {
                const float vc = sc[tt * V + col];
                if (p.mode == 1) {                  // end states only
                    if (active) {
#pragma unroll
                        for (int i = 0; i < DR; i += 4) {
                            const float4 wv = ms_row4(w, row0 + i, D, vec), bv = ms_row4(b, row0 + i, D, vec);
                            S[i] = fmaf(wv.x, S[i], bv.x * vc); S[i + 1] = fmaf(wv.y, S[i + 1], bv.y * vc);
                            S[i + 2] = fmaf(wv.z, S[i + 2], bv.z * vc); S[i + 3] = fmaf(wv.w, S[i + 3], bv.w * vc);
                        }
                    }
                    continue;
                }
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
                if (active) {
#pragma unroll
                    for (int i = 0; i < DR; i += 4) {
                        const float4 wv = ms_row4(w, row0 + i, D, vec), bv = ms_row4(b, row0 + i, D, vec);
                        const float4 av = ms_row4(a, row0 + i, D, vec), uv = ms_row4(sbonus, row0 + i, D, vec);
                        const float k0 = bv.x * vc, k1 = bv.y * vc, k2 = bv.z * vc, k3 = bv.w * vc;
                        s4[0] = fmaf(av.x, fmaf(uv.x, k0, S[i]), s4[0]); s4[1] = fmaf(av.y, fmaf(uv.y, k1, S[i + 1]), s4[1]);
                        s4[2] = fmaf(av.z, fmaf(uv.z, k2, S[i + 2]), s4[2]); s4[3] = fmaf(av.w, fmaf(uv.w, k3, S[i + 3]), s4[3]);
                        S[i] = fmaf(wv.x, S[i], k0); S[i + 1] = fmaf(wv.y, S[i + 1], k1);
                        S[i + 2] = fmaf(wv.z, S[i + 2], k2); S[i + 3] = fmaf(wv.w, S[i + 3], k3);
                    }
                }
                float o;
                MS_COLUMN_SUM(o, (s4[0] + s4[1]) + (s4[2] + s4[3]), false);
                if (grp == 0) so[tt * V + col] = o;
            }
#undef MS_COLUMN_SUM
        }
        if (p.mode == 1) continue;
        __syncthreads();
        // the tile's outputs: per head o / rms(o), a weight, the gate
        for (int tt = warp; tt < nt; tt += nwarps) {
            float s = 0.f;
            for (int c = lane; c < V; c += 32) s = fmaf(so[tt * V + c], so[tt * V + c], s);
            s = warp_sum(s);
            if (lane == 0) sscale[tt] = rsqrtf(s / (float)V + p.eps);
        }
        __syncthreads();
        for (int i = tid; i < nt * V; i += nthreads) {
            const int tt = i / V, c = i - tt * V;
            const size_t t = (size_t)(start + t0 + tt);
            const float g = ms_load(p.gate, p.gate_dtype, t * p.ld_gate + (size_t)head * V + c);
            const float weight = DELTA ? p.norm_w[c] : p.norm_w[(size_t)head * V + c];
            const float gated = DELTA ? ms_sigmoid(g) : g * ms_sigmoid(g);
            ms_store(p.out, p.dtype, t * ((size_t)p.heads * V) + (size_t)head * V + c, so[i] * sscale[tt] * weight * gated);
        }
    }
    if (p.mode == 1) {                              // the part's end state from zero, the transition beside it
#pragma unroll
        for (int i = 0; i < DR; ++i)
            if (active && row0 + i < D) p.part_end[part_index * D * VA + (size_t)(row0 + i) * VA + col] = S[i];
        if (!DELTA)
            for (int d = tid; d < D; d += nthreads) {
                float sum = 0.f;
                for (int t = t_begin; t < t_end; ++t) sum += p.log_decay[(size_t)(start + t) * ((size_t)p.heads * D) + (size_t)head * D + d];
                p.part_log[part_index * D + d] = sum;
            }
        return;
    }
    if (!p.write || len == 0) return;
    if (p.mode == 2 && part != (len - 1) / p.part_len) return;      // the last part refreshes the kept inputs
    if (p.mode == 0) {
#pragma unroll
        for (int i = 0; i < DR; ++i)
            if (active && row0 + i < D) state[(size_t)(row0 + i) * V + col] = S[i];
    }
    if (!DELTA) {
        // the kept input becomes the segment's last token; the heads share the columns between them
        const int c0 = (int)((long long)p.width * head / p.heads), c1 = (int)((long long)p.width * (head + 1) / p.heads);
        for (int c = c0 + tid; c < c1; c += nthreads)
            ms_store(p.kept, p.dtype, (size_t)slot * p.width + c, ms_load(p.raw, p.dtype, (size_t)(start + len - 1) * p.ld_raw + c));
        return;
    }
    // the convolutions' kept inputs for the channels this head owns: its values, and q and k of its key head if it is
    // that head's first. A thread per channel walks the kept rows oldest first, so a short segment shifts the old rows
    // down before it overwrites them.
    const int keep = p.taps - 1;
    if (keep <= 0) return;
    const int qk = p.kv_heads * D;
    const bool owns_qk = head % (p.heads / p.kv_heads) == 0;
    const int count = V + (owns_qk ? 2 * D : 0);
    for (int i = tid; i < count; i += nthreads) {
        int ch;
        if (i < V) ch = 2 * qk + head * V + i;
        else if (i < V + D) ch = kvh * D + (i - V);
        else ch = qk + kvh * D + (i - V - D);
        for (int j = 0; j < keep; ++j) {
            const int local = len - keep + j;
            float v;
            if (local >= 0) v = ms_load(p.raw, p.dtype, (size_t)(start + local) * p.ld_raw + ch);
            else v = ms_load(p.kept, p.dtype, ((size_t)slot * keep + (keep + local)) * p.width + ch);
            ms_store(p.kept, p.dtype, ((size_t)slot * keep + j) * p.width + ch, v);
        }
    }
}

// The parts folded in order: S_0 = the request's state; S_(p+1) = M_p S_p + E_p. Columns of the state do not mix, and with
// a diagonal M nothing does: the token-shift state folds element by element (a thread per element, blocks of 256), the
// delta rule in tiles of FOLD_COLS columns per block with M_p staged in shared memory. Leaves every part's start state in
// part_start and, with `write`, the state behind the last part in the request's slot.
#define FOLD_COLS 16
__global__ void __launch_bounds__(256)
matrix_state_fold_diagonal_kernel(const MsArgs p) {
    pdl_wait();
    pdl_launch_dependents();
    const int D = p.D, V = p.V, n = D * V;
    const int seg = blockIdx.x, head = blockIdx.y, i = blockIdx.z * 256 + threadIdx.x;
    const int len = p.cu_seqlens[seg + 1] - p.cu_seqlens[seg];
    if (len == 0 || i >= n) return;
    const int nparts = (len + p.part_len - 1) / p.part_len;
    float* state = p.state + ((size_t)p.slots[seg] * p.heads + head) * n;
    float cur = state[i];
    const size_t first = ((size_t)seg * p.heads + head) * p.parts;
    for (int part = 0; part < nparts; ++part) {
        p.part_start[(first + part) * n + i] = cur;
        cur = fmaf(expf(p.part_log[(first + part) * D + i / V]), cur, p.part_end[(first + part) * n + i]);
    }
    if (p.write) state[i] = cur;
}

// `buffers` 2: M of the next part is on its way (asynchronous copies) while this part is multiplied; 1: one at a time.
__global__ void __launch_bounds__(256)
matrix_state_fold_kernel(const MsArgs p, int buffers) {
    extern __shared__ __align__(16) float fold_smem[];
    const int D = p.D, V = p.V, n = D * V, VA = V + D, m_size = D * (D + 1);
    float* M = fold_smem;                          // [buffers][D, D + 1]
    float* cur = M + (size_t)buffers * m_size;     // [D, FOLD_COLS]
    float* next = cur + D * FOLD_COLS;
    pdl_wait();
    pdl_launch_dependents();
    const int seg = blockIdx.x, head = blockIdx.y, tid = threadIdx.x;
    const int c0 = blockIdx.z * FOLD_COLS, ncols = min(FOLD_COLS, V - c0);
    const int len = p.cu_seqlens[seg + 1] - p.cu_seqlens[seg];
    if (len == 0) return;
    const int nparts = (len + p.part_len - 1) / p.part_len;
    const size_t first = ((size_t)seg * p.heads + head) * p.parts;
    float* state = p.state + ((size_t)p.slots[seg] * p.heads + head) * n;
    auto fetch = [&](int part) {                   // M_part into its buffer, four bytes a copy (rows are padded by one)
        const float* end = p.part_end + (first + part) * D * VA;
        float* dst = M + (size_t)(buffers == 2 ? (part & 1) : 0) * m_size;
        for (int i = tid; i < D * D; i += blockDim.x) {
            const int r = i / D, j = i - r * D;
            const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst + r * (D + 1) + j);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(end + (size_t)r * VA + V + j) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(0);
    for (int e = tid; e < D * FOLD_COLS; e += blockDim.x) {          // columns beyond the state's are zeros and stay zeros
        const int r = e / FOLD_COLS, c = e - r * FOLD_COLS;
        cur[e] = c < ncols ? state[(size_t)r * V + c0 + c] : 0.f;
        next[e] = 0.f;
    }
    for (int part = 0; part < nparts; ++part) {
        if (buffers == 2 && part + 1 < nparts) {
            fetch(part + 1);                       // the buffer of part - 1: everybody is past its products (the barrier below)
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();                           // M_part and the state before the part are in place
        const float* Mp = M + (size_t)(buffers == 2 ? (part & 1) : 0) * m_size;
        const float* end = p.part_end + (first + part) * D * VA;     // row r: [E (V) | M (D)]
        float* begin = p.part_start + (first + part) * n;
        // a thread takes four neighbouring columns of one row: a number of M serves four products
        for (int e = tid; e < D * (FOLD_COLS / 4); e += blockDim.x) {
            const int r = e / (FOLD_COLS / 4), c = (e - r * (FOLD_COLS / 4)) * 4;
            if (c >= ncols) continue;
            const float4 before = *reinterpret_cast<const float4*>(cur + r * FOLD_COLS + c);
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const float* row = Mp + r * (D + 1);
            for (int j = 0; j < D; ++j) {
                const float m = row[j];
                const float4 sv = *reinterpret_cast<const float4*>(cur + j * FOLD_COLS + c);
                acc[0] = fmaf(m, sv.x, acc[0]); acc[1] = fmaf(m, sv.y, acc[1]);
                acc[2] = fmaf(m, sv.z, acc[2]); acc[3] = fmaf(m, sv.w, acc[3]);
            }
            const float was[4] = {before.x, before.y, before.z, before.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float v = 0.f;
                if (c + q < ncols) {
                    begin[(size_t)r * V + c0 + c + q] = was[q];
                    v = end[(size_t)r * VA + c0 + c + q] + acc[q];
                }
                next[r * FOLD_COLS + c + q] = v;
            }
        }
        __syncthreads();
        float* t = cur; cur = next; next = t;
        if (buffers == 1 && part + 1 < nparts) fetch(part + 1);
    }
    if (p.write)
        for (int e = tid; e < D * ncols; e += blockDim.x) {
            const int r = e / ncols, c = e - r * ncols;
            state[(size_t)r * V + c0 + c] = cur[r * FOLD_COLS + c];
        }
}

template <bool DELTA>
static int ms_launch(MsArgs& p, int segments, cudaStream_t stream) {
    const int D = p.D, V = p.V;
    if (D < 1 || V < 1 || V > MS_MAX_THREADS || p.heads < 1 || p.heads > 65535) return TTB_ERR_UNSUPPORTED;
    if (p.parts > 1) {
        if (!p.part_end || !p.part_start || (!DELTA && !p.part_log) || p.part_len < 1 || p.parts > 65535) return TTB_ERR_ARGUMENT;
        const size_t one_m = (size_t)D * (D + 1) * sizeof(float), states = 2 * (size_t)D * FOLD_COLS * sizeof(float);
        const int fold_buffers = 2 * one_m + states <= 200 * 1024 ? 2 : 1;
        const size_t fold_smem = DELTA ? fold_buffers * one_m + states : 0;
        if (fold_smem > 200 * 1024 || (DELTA && V + D > MS_MAX_THREADS)) {      // too large a transition: the walk as a whole
            p.mode = 0;
            p.parts = 1;
            return ms_launch_mode<DELTA>(p, segments, stream);
        }
        MsArgs ends = p;
        ends.mode = 1;
        int rc = ms_launch_mode<DELTA>(ends, segments, stream);
        if (rc != TTB_OK) return rc;
        if (DELTA) {
            static TtbOncePerDevice once;
            if (fold_smem > 48 * 1024 && once.pending()) {
                cudaFuncSetAttribute(matrix_state_fold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
                once.mark();
            }
            ttb_launch(matrix_state_fold_kernel, dim3(segments, p.heads, (V + FOLD_COLS - 1) / FOLD_COLS), 256, fold_smem, stream, p,
                       fold_buffers);
        } else {
            ttb_launch(matrix_state_fold_diagonal_kernel, dim3(segments, p.heads, (D * V + 255) / 256), 256, 0, stream, p);
        }
        rc = ttb_launch_status();
        if (rc != TTB_OK) return rc;
        p.mode = 2;
        return ms_launch_mode<DELTA>(p, segments, stream);
    }
    p.mode = 0;
    p.parts = 1;
    return ms_launch_mode<DELTA>(p, segments, stream);
}

template <bool DELTA>
static int ms_launch_mode(MsArgs& p, int segments, cudaStream_t stream) {
    const int D = p.D, V = p.V;
    const int VA = (DELTA && p.mode == 1) ? V + D : V;
    if (VA > MS_MAX_THREADS) return TTB_ERR_UNSUPPORTED;
    // the fewest rows a thread that still lets a column's row groups fit one block, and at most 512 threads where that works
    // (a thread that holds a whole column needs no barrier, but its sums are chains as long as the column: measured at
    // 64 x 64 and 128 x 128, 871 against 635 us and 2,105 against 2,011 us a call of 2,048 tokens)
    int DR = 8;
    while (DR < 64 && VA * ((D + DR - 1) / DR) > 512) DR *= 2;
    const int R = (D + DR - 1) / DR;
    if (VA * R > MS_MAX_THREADS) return TTB_ERR_UNSUPPORTED;
    p.R = R;
    int threads = (VA * R + 31) / 32 * 32;
    if (threads < 64) threads = 64;
    const size_t smem = ((size_t)MS_TILE * (3 * D + 2 * V) + 2 * (size_t)R * (V + (DELTA ? D : 0)) + MS_TILE + D + 2 * MS_TILE) * sizeof(float);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    dim3 grid(segments, p.heads, p.mode == 0 ? 1 : p.parts);
#define MS_GO(DRV, CAPV)                                                                                             \
    do {                                                                                                             \
        static TtbOncePerDevice once;                                                                                \
        if (smem > 48 * 1024 && once.pending()) {                                                                    \
            cudaFuncSetAttribute(matrix_state_walk_kernel<DRV, DELTA, CAPV>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
            once.mark();                                                                                             \
        }                                                                                                            \
        ttb_launch(matrix_state_walk_kernel<DRV, DELTA, CAPV>, grid, threads, smem, stream, p);                      \
    } while (0)
    // sixty-four rows a thread want registers: the fewer threads a block has, the more of them a thread may use
    if (DR == 8) MS_GO(8, 512); else if (DR == 16) MS_GO(16, 512); else if (DR == 32) MS_GO(32, 512);
    else if (threads <= 256) MS_GO(64, 256); else if (threads <= 512) MS_GO(64, 512); else MS_GO(64, 1024);
#undef MS_GO
    return ttb_launch_status();
}

// r, k, v and the gate (before its silu): [T, heads * dim] each, of the compute type, with a common row stride `ld`.
// log_decay float32 [T, heads * dim]; bonus float32 [heads, dim]; norm_w float32 [heads * dim].
// state float32 [slots, heads, dim, dim]; kept [slots, width]: the request's last input, refreshed from x [T, ldx].
TTB_EXPORT int ttb_shifted_state(const void* r, const void* k, const void* v, const void* g, int dtype, long long ld, const float* log_decay,
                                 const float* bonus, const float* norm_w, float eps, const void* x, long long ldx, int width,
                                 const int* cu_seqlens, const int* slots, float* state, void* kept, void* out, int segments,
                                 int heads, int dim, int write, int parts, int part_len, float* part_end, float* part_start,
                                 float* part_log, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!r || !k || !v || !g || !log_decay || !bonus || !norm_w || !x || !cu_seqlens || !slots || !state || !kept || !out) return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    MsArgs p = {};
    p.a = r; p.b = k; p.c = v; p.gate = g;
    p.ld_a = p.ld_b = p.ld_c = p.ld_gate = ld;
    p.dtype = p.gate_dtype = dtype;
    p.log_decay = log_decay; p.bonus = bonus; p.norm_w = norm_w; p.eps = eps;
    p.cu_seqlens = cu_seqlens; p.slots = slots; p.state = state; p.kept = kept; p.raw = x; p.ld_raw = ldx; p.width = width;
    p.taps = 2; p.out = out; p.heads = heads; p.kv_heads = heads; p.D = dim; p.V = dim; p.write = write;
    p.parts = parts; p.part_len = part_len; p.part_end = part_end; p.part_start = part_start; p.part_log = part_log;
    return ms_launch<false>(p, segments, stream);
}

// conv [T, q | k | v] after the convolutions and their silu (q, k: kv_heads * dim; v: heads * vdim), row stride ld_conv;
// raw: the convolutions' inputs in the same layout; beta float32 logits [T, heads] (row stride ld_beta); log_decay float32
// [T, heads * dim]; gate float32 logits [T, heads * vdim]; norm_w float32 [vdim]. state float32 [slots, heads, dim, vdim];
// kept [slots, taps - 1, channels]. parts > 1: part_end [segments, heads, parts, dim, vdim + dim] and part_start [segments, heads,
// parts, dim, vdim] are scratch memory (the token-shift state: part_end [.., dim, dim] and part_log [segments, heads, parts, dim]).
TTB_EXPORT int ttb_delta_rule(const void* conv, int dtype, long long ld_conv, const void* raw, long long ld_raw,
                              const float* beta, int ld_beta, const float* log_decay, const float* gate, const float* norm_w,
                              float eps, const int* cu_seqlens, const int* slots, float* state, void* kept, void* out,
                              int segments, int heads, int kv_heads, int dim, int vdim, int taps, int write, int parts, int part_len,
                              float* part_end, float* part_start, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!conv || !raw || !beta || !log_decay || !gate || !norm_w || !cu_seqlens || !slots || !state || !out || (taps > 1 && !kept))
        return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    if (kv_heads < 1 || heads % kv_heads) return TTB_ERR_UNSUPPORTED;
    const size_t el = dtype == TTB_DTYPE_BF16 ? 2 : 4;
    const long long qk = (long long)kv_heads * dim;
    MsArgs p = {};
    p.a = conv; p.b = (const char*)conv + qk * el; p.c = (const char*)conv + 2 * qk * el; p.gate = gate;
    p.ld_a = p.ld_b = p.ld_c = ld_conv; p.ld_gate = (long long)heads * vdim;
    p.dtype = dtype; p.gate_dtype = TTB_DTYPE_F32;
    p.log_decay = log_decay; p.beta = beta; p.ld_beta = ld_beta; p.norm_w = norm_w; p.eps = eps;
    p.cu_seqlens = cu_seqlens; p.slots = slots; p.state = state; p.kept = kept; p.raw = raw; p.ld_raw = ld_raw;
    p.width = (int)(2 * qk + (long long)heads * vdim); p.taps = taps; p.out = out;
    p.heads = heads; p.kv_heads = kv_heads; p.D = dim; p.V = vdim; p.write = write;
    p.parts = parts; p.part_len = part_len; p.part_end = part_end; p.part_start = part_start; p.part_log = nullptr;
    return ms_launch<true>(p, segments, stream);
}
