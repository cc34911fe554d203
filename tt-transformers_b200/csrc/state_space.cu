// A state-space mixer with a matrix state per head: short causal convolution, the recurrence, gate and grouped norm.
//
//   u = silu(conv(x B C) + b)                       ss_conv_silu: a thread per (token, channel), the request's kept inputs
//                                                   before the step's first token
//   dt = softplus(dt_raw + dt_bias); a = exp(-rate dt)
//   S_t = a S_(t-1) + dt B_t x_t^T;  y_t = S_t^T C_t + D x_t      ss_scan: a block per (head, segment, part of the segment)
//   out = rms_groups(y * silu(z)) * w               ss_gate_norm: a block per (token, norm group)
//
// ss_scan keeps the head's state S [N, P] in registers: thread (col, ng) owns PC neighbouring columns and the rows
// ng, ng + NG, ... (R of them). Tokens come in tiles of SS_TILE through shared memory (x, dt B, C, a per token); a thread
// leaves its share of y for every token of the tile in shared memory and the tile's y is summed over the row groups
// afterwards, in a fixed order, so the walk itself has no barrier per token. Everything is float32.
// Long segments run as parts side by side: every part but the last first walks from a zero state and leaves its end
// state E_k and the logarithm of its decays' product L_k (ENDS_ONLY); ss_prefix turns these into the parts' start
// states, start_(k+1) = exp(L_k) start_k + E_k; then every part walks from its start state and writes y. The last part
// stores the state and the convolution's new kept inputs.
#include "common.cuh"

#define SS_TILE 8

__device__ __forceinline__ float ss_load(const void* p, int dtype, size_t i) {
    return dtype == TTB_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                                   : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void ss_store(void* p, int dtype, size_t i, float v) {
    if (dtype == TTB_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}
// four neighbouring values; i a multiple of 4 and p on a 16-byte boundary
__device__ __forceinline__ float4 ss_load4(const void* p, int dtype, size_t i) {
    if (dtype == TTB_DTYPE_BF16) {
        const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p) + i);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
}
__device__ __forceinline__ void ss_store4(void* p, int dtype, size_t i, float4 v) {
    if (dtype == TTB_DTYPE_BF16) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 raw;
        raw.x = *reinterpret_cast<const unsigned*>(&lo);
        raw.y = *reinterpret_cast<const unsigned*>(&hi);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = raw;
    } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = v;
    }
}
__device__ __forceinline__ float ss_silu(float v) { return v / (1.f + expf(-v)); }
__device__ __forceinline__ float ss_softplus(float v) { return v > 20.f ? v : log1pf(expf(v)); }

// ---------------------------------------------------------------- convolution and silu
__global__ void __launch_bounds__(256)
ss_conv_silu_kernel(const void* __restrict__ in, int dtype, int ld, const float* __restrict__ conv_w,
                    const float* __restrict__ conv_b, const int* __restrict__ seg_of_token, const int* __restrict__ cu_seqlens,
                    const int* __restrict__ slots, const void* __restrict__ tail, void* __restrict__ out, int tokens,
                    int channels, int taps) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)tokens * channels;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / channels), c = (int)(i % channels);
        const int seg = seg_of_token[t];
        const int local = t - cu_seqlens[seg];
        float acc = conv_b[c];
        for (int j = 0; j < taps; ++j) {
            const int back = taps - 1 - j;                       // tap j looks `back` tokens back
            float v;
            if (local - back >= 0) v = ss_load(in, dtype, (size_t)(t - back) * ld + c);
            else v = ss_load(tail, dtype, ((size_t)slots[seg] * (taps - 1) + (taps - 1 + local - back)) * channels + c);
            acc = fmaf(conv_w[(size_t)c * taps + j], v, acc);
        }
        ss_store(out, dtype, i, ss_silu(acc));
    }
}


// the same with four neighbouring channels a thread (channels, ld and the column offset multiples of 4)
__global__ void __launch_bounds__(256)
ss_conv_silu4_kernel(const void* __restrict__ in, int dtype, int ld, const float* __restrict__ conv_w,
                     const float* __restrict__ conv_b, const int* __restrict__ seg_of_token, const int* __restrict__ cu_seqlens,
                     const int* __restrict__ slots, const void* __restrict__ tail, void* __restrict__ out, int tokens,
                     int channels, int taps) {
    pdl_wait();
    pdl_launch_dependents();
    // a block walks tokens, its threads the token's groups of four channels: no division per element
    const int quads = channels / 4;
    for (int t = blockIdx.x; t < tokens; t += gridDim.x) {
        const int seg = seg_of_token[t];
        const int local = t - cu_seqlens[seg];
        const size_t kept = (size_t)slots[seg] * (taps - 1);
        for (int q = threadIdx.x; q < quads; q += blockDim.x) {
            const int c = q * 4;
            float4 acc = *reinterpret_cast<const float4*>(conv_b + c);
            for (int j = 0; j < taps; ++j) {
                const int back = taps - 1 - j;
                float4 v;
                if (local - back >= 0) v = ss_load4(in, dtype, (size_t)(t - back) * ld + c);
                else v = ss_load4(tail, dtype, (kept + (taps - 1 + local - back)) * channels + c);
                acc.x = fmaf(conv_w[(size_t)c * taps + j], v.x, acc.x);
                acc.y = fmaf(conv_w[(size_t)(c + 1) * taps + j], v.y, acc.y);
                acc.z = fmaf(conv_w[(size_t)(c + 2) * taps + j], v.z, acc.z);
                acc.w = fmaf(conv_w[(size_t)(c + 3) * taps + j], v.w, acc.w);
            }
            ss_store4(out, dtype, (size_t)t * channels + c,
                      make_float4(ss_silu(acc.x), ss_silu(acc.y), ss_silu(acc.z), ss_silu(acc.w)));
        }
    }
}

// Prompt portions: a thread takes four neighbouring channels over SS_CONV_RUN tokens in a row and keeps the last
// taps - 1 inputs and its taps' weights in registers, so a token costs one load of its own input. The window is read
// anew at the run's first token and wherever another segment begins. The same sums in the same order as above.
#define SS_CONV_RUN 8
template <int TAPS>
__global__ void __launch_bounds__(128)
ss_conv_silu_run_kernel(const void* __restrict__ in, int dtype, int ld, const float* __restrict__ conv_w,
                        const float* __restrict__ conv_b, const int* __restrict__ seg_of_token, const int* __restrict__ cu_seqlens,
                        const int* __restrict__ slots, const void* __restrict__ tail, void* __restrict__ out, int tokens,
                        int channels) {
    pdl_wait();
    pdl_launch_dependents();
    const int q = blockIdx.y * blockDim.x + threadIdx.x;
    if (q >= channels / 4) return;
    const int c = q * 4;
    const int t_first = blockIdx.x * SS_CONV_RUN, t_last = min(tokens, t_first + SS_CONV_RUN);
    float w[4][TAPS];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < TAPS; ++j) w[i][j] = conv_w[(size_t)(c + i) * TAPS + j];
    const float4 bias = *reinterpret_cast<const float4*>(conv_b + c);
    float4 win[TAPS];                                            // win[j]: the input TAPS - 1 - j tokens back
    int seg = -1, seg_begin = 0;
    size_t kept = 0;
    for (int t = t_first; t < t_last; ++t) {
        const int s = seg_of_token[t];
        const bool fresh = t == t_first || s != seg;
        if (s != seg) {
            seg = s;
            seg_begin = cu_seqlens[s];
            kept = (size_t)slots[s] * (TAPS - 1);
        }
        const int local = t - seg_begin;
        if (fresh) {
#pragma unroll
            for (int j = 0; j < TAPS - 1; ++j) {
                const int back = TAPS - 1 - j;
                if (local - back >= 0) win[j] = ss_load4(in, dtype, (size_t)(t - back) * ld + c);
                else win[j] = ss_load4(tail, dtype, (kept + (TAPS - 1 + local - back)) * channels + c);
            }
        } else {
#pragma unroll
            for (int j = 0; j < TAPS - 1; ++j) win[j] = win[j + 1];
        }
        win[TAPS - 1] = ss_load4(in, dtype, (size_t)t * ld + c);
        float4 acc = bias;
#pragma unroll
        for (int j = 0; j < TAPS; ++j) {
            acc.x = fmaf(w[0][j], win[j].x, acc.x);
            acc.y = fmaf(w[1][j], win[j].y, acc.y);
            acc.z = fmaf(w[2][j], win[j].z, acc.z);
            acc.w = fmaf(w[3][j], win[j].w, acc.w);
        }
        ss_store4(out, dtype, (size_t)t * channels + c, make_float4(ss_silu(acc.x), ss_silu(acc.y), ss_silu(acc.z), ss_silu(acc.w)));
    }
}

// ---------------------------------------------------------------- the recurrence
struct SsScanArgs {
    const void* u;            // [T, channels] after convolution and silu: x | B | C
    const void* proj;         // [T, ld]: the input projection (step sizes, and the convolution's raw inputs for the kept ones)
    int dtype, ld, conv_off, dt_off;
    const float *dt_bias, *rate, *skip;
    const int *cu_seqlens, *slots;
    float* state;             // [slots, heads, N, P]
    void* tail;               // [slots, taps - 1, channels]
    float* y;                 // [T, heads * P]
    float* part_state;        // [segments, heads, parts, N * P]: E_k, then start_(k+1)
    float* part_log;          // [segments, heads, parts]
    int heads, P, N, groups, channels, taps, write_state, parts, part_len, NG;
};

// The convolution's new kept inputs, for the channels one head owns: its x columns, and B and C of its group if it is
// the group's first head. A thread per channel walks the kept rows oldest first, so a short segment shifts the old rows
// down before it overwrites them.
__device__ __forceinline__ void ss_keep_inputs(const SsScanArgs& a, int head, int group, int seg_start, int seg_len, int slot,
                                               int tid) {
    const int keep = a.taps - 1;
    if (keep <= 0) return;
    const int P = a.P, N = a.N, inner = a.heads * P;
    const bool owns_group = head % (a.heads / a.groups) == 0;
    const int mine = P + (owns_group ? 2 * N : 0);
    for (int i = tid; i < mine; i += blockDim.x) {
        int ch;
        if (i < P) ch = head * P + i;
        else if (i < P + N) ch = inner + group * N + (i - P);
        else ch = inner + a.groups * N + group * N + (i - P - N);
        for (int j = 0; j < keep; ++j) {
            const int local = seg_len - keep + j;
            float v;
            if (local >= 0) v = ss_load(a.proj, a.dtype, (size_t)(seg_start + local) * a.ld + a.conv_off + ch);
            else v = ss_load(a.tail, a.dtype, ((size_t)slot * keep + (keep + local)) * a.channels + ch);
            ss_store(a.tail, a.dtype, ((size_t)slot * keep + j) * a.channels + ch, v);
        }
    }
}

template <int PC, int R, bool ENDS_ONLY>
__global__ void __launch_bounds__(PC == 1 && R == 32 ? 1024 : 256)
ss_scan_kernel(const SsScanArgs a) {
    extern __shared__ __align__(16) float ss_smem[];
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y, part = blockIdx.z;
    const int P = a.P, N = a.N, NG = a.NG;
    const int seg_start = a.cu_seqlens[seg], seg_len = a.cu_seqlens[seg + 1] - seg_start;
    const int parts_here = a.parts > 1 ? max(1, (seg_len + a.part_len - 1) / a.part_len) : 1;
    if (part >= parts_here || seg_len <= 0) return;
    const bool last_part = part == parts_here - 1;
    if (ENDS_ONLY && last_part) return;                              // nobody starts from the last part's end
    const int t_begin = seg_start + (a.parts > 1 ? part * a.part_len : 0);
    const int t_end = last_part ? seg_start + seg_len : t_begin + a.part_len;
    const int cols = P / PC, threads = cols * NG;
    const int tid = threadIdx.x, col = tid % cols, ng = tid / cols;
    const bool active = tid < threads;
    const int inner = a.heads * P, group = head / (a.heads / a.groups);
    float* xs = ss_smem;                                             // [TILE, P]
    float* bs = xs + SS_TILE * P;                                    // [TILE, N]   dt * B
    float* cs = bs + SS_TILE * N;                                    // [TILE, N]
    float* decay = cs + SS_TILE * N;                                 // [TILE] then dt [TILE]
    float* ypart = decay + 2 * SS_TILE;                              // [TILE, NG, P]
    const int slot = a.slots[seg];
    float S[R][PC];
    const float* start = nullptr;
    if (!ENDS_ONLY) {
        start = part == 0 ? a.state + ((size_t)slot * a.heads + head) * N * P
                          : a.part_state + (((size_t)seg * a.heads + head) * a.parts + (part - 1)) * N * P;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int n = ng + r * NG;
#pragma unroll
        for (int c = 0; c < PC; ++c) S[r][c] = (start != nullptr && active && n < N) ? start[(size_t)n * P + col * PC + c] : 0.f;
    }
    const float rate = a.rate[head], bias = a.dt_bias[head], skip = a.skip[head];
    float log_sum = 0.f;
    for (int t0 = t_begin; t0 < t_end; t0 += SS_TILE) {
        const int nt = min(SS_TILE, t_end - t0);
        __syncthreads();                                             // the tile before is summed and stored
        if (tid < nt) {
            const float dt = ss_softplus(ss_load(a.proj, a.dtype, (size_t)(t0 + tid) * a.ld + a.dt_off + head) + bias);
            decay[tid] = expf(-rate * dt);
            decay[SS_TILE + tid] = dt;
        }
        __syncthreads();
        for (int i = tid; i < nt * P; i += blockDim.x) {
            const int k = i / P, p = i % P;
            xs[k * P + p] = ss_load(a.u, a.dtype, (size_t)(t0 + k) * a.channels + head * P + p);
        }
        for (int i = tid; i < nt * N; i += blockDim.x) {
            const int k = i / N, n = i % N;
            const size_t row = (size_t)(t0 + k) * a.channels + inner + group * N + n;
            bs[k * N + n] = decay[SS_TILE + k] * ss_load(a.u, a.dtype, row);
            if (!ENDS_ONLY) cs[k * N + n] = ss_load(a.u, a.dtype, row + (size_t)a.groups * N);
        }
        if (ENDS_ONLY && tid == 0)
            for (int k = 0; k < nt; ++k) log_sum -= rate * decay[SS_TILE + k];
        __syncthreads();
        if (active) {
            for (int k = 0; k < nt; ++k) {
                const float ak = decay[k];
                float xv[PC], acc[PC];
#pragma unroll
                for (int c = 0; c < PC; ++c) { xv[c] = xs[k * P + col * PC + c]; acc[c] = 0.f; }
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int n = ng + r * NG;
                    if (n < N) {
                        const float b = bs[k * N + n];
                        const float cn = ENDS_ONLY ? 0.f : cs[k * N + n];
#pragma unroll
                        for (int c = 0; c < PC; ++c) {
                            S[r][c] = fmaf(ak, S[r][c], b * xv[c]);
                            if (!ENDS_ONLY) acc[c] = fmaf(S[r][c], cn, acc[c]);
                        }
                    }
                }
                if (!ENDS_ONLY) {
#pragma unroll
                    for (int c = 0; c < PC; ++c) ypart[((size_t)k * NG + ng) * P + col * PC + c] = acc[c];
                }
            }
        }
        if (!ENDS_ONLY) {
            __syncthreads();
            for (int i = tid; i < nt * P; i += blockDim.x) {
                const int k = i / P, p = i % P;
                float s = 0.f;
                for (int g = 0; g < NG; ++g) s += ypart[((size_t)k * NG + g) * P + p];
                a.y[(size_t)(t0 + k) * inner + head * P + p] = fmaf(skip, xs[k * P + p], s);
            }
        }
    }
    if (ENDS_ONLY) {
        float* dst = a.part_state + (((size_t)seg * a.heads + head) * a.parts + part) * N * P;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int n = ng + r * NG;
            if (active && n < N)
#pragma unroll
                for (int c = 0; c < PC; ++c) dst[(size_t)n * P + col * PC + c] = S[r][c];
        }
        if (tid == 0) a.part_log[((size_t)seg * a.heads + head) * a.parts + part] = log_sum;
        return;
    }
    if (!last_part || !a.write_state) return;
    float* dst = a.state + ((size_t)slot * a.heads + head) * N * P;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int n = ng + r * NG;
        if (active && n < N)
#pragma unroll
            for (int c = 0; c < PC; ++c) dst[(size_t)n * P + col * PC + c] = S[r][c];
    }
    ss_keep_inputs(a, head, group, seg_start, seg_len, slot, tid);
}

// ---------------------------------------------------------------- the recurrence, packed
// The same walk for heads whose sizes divide evenly (P and N multiples of 4, R a multiple of 4 that divides N), issued
// as two-wide float32 operations. Thread (col, ng) owns columns 4 col .. 4 col + 3 and the R neighbouring rows from
// ng R on; a register pair holds two neighbouring rows of one column. Inside a tile the state is kept relative to the
// decays so far, T_k = S_k / A_k with A_k = a_0 .. a_k, which leaves one multiply-add per element for the update and
// one for the output:
//   T_k = T_(k-1) + (dt_k B_k / A_k) x_k^T,   y_k = A_k (T_k^T C_k) + D x_k,   S = A_last T at the tile's end.
// A tile whose decays' product is below SS_RELATIVE_FLOOR (1 / A_k would leave the float32 range) takes the direct form
// S_k = a_k S_(k-1) + dt_k B_k x_k^T instead; every thread of the block takes the same branch.
#define SS_RELATIVE_FLOOR 1e-20f
#define SS_PTILE 16                  // tokens of a tile of the packed walk; at most a warp, whose lanes sum the step sizes

template <bool V> struct SsForm { static constexpr bool value = V; };

template <int R, bool ENDS_ONLY>
__global__ void __launch_bounds__(256, R <= 8 ? 3 : (R == 16 ? 2 : 1))
ss_scan_packed_kernel(const SsScanArgs a) {
    extern __shared__ __align__(16) float ss_smem[];
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y, part = blockIdx.z;
    const int P = a.P, N = a.N, NG = a.NG;
    const int seg_start = a.cu_seqlens[seg], seg_len = a.cu_seqlens[seg + 1] - seg_start;
    const int parts_here = a.parts > 1 ? max(1, (seg_len + a.part_len - 1) / a.part_len) : 1;
    if (part >= parts_here || seg_len <= 0) return;
    const bool last_part = part == parts_here - 1;
    if (ENDS_ONLY && last_part) return;
    const int t_begin = seg_start + (a.parts > 1 ? part * a.part_len : 0);
    const int t_end = last_part ? seg_start + seg_len : t_begin + a.part_len;
    const int cols = P / 4, threads = cols * NG;
    const int tid = threadIdx.x, col = tid % cols, ng = tid / cols;
    const int warp = tid / 32, lane = tid % 32, warps = blockDim.x / 32;
    const bool active = tid < threads;
    const int inner = a.heads * P, group = head / (a.heads / a.groups);
    float* xs = ss_smem;                                             // [TILE, P, 2]  every x twice: a pair for two rows
    float* bs = xs + 2 * SS_PTILE * P;                                // [TILE, N]     dt B / A (or dt B, direct form)
    float* cs = bs + SS_PTILE * N;                                    // [TILE, N]
    float* meta = cs + SS_PTILE * N;                                  // [4, TILE]     a_k, A_k, dt_k, the tile's log
    float* ypart = meta + 4 * SS_PTILE;                               // [TILE, NG, P]
    const int slot = a.slots[seg];
    float2 S[R / 2][4];
    const int n0 = ng * R;
    const float* start = nullptr;
    if (!ENDS_ONLY) {
        start = part == 0 ? a.state + ((size_t)slot * a.heads + head) * N * P
                          : a.part_state + (((size_t)seg * a.heads + head) * a.parts + (part - 1)) * N * P;
    }
#pragma unroll
    for (int r = 0; r < R / 2; ++r) {
        float4 even = make_float4(0.f, 0.f, 0.f, 0.f), odd = even;
        if (start != nullptr && active) {
            even = *reinterpret_cast<const float4*>(start + (size_t)(n0 + 2 * r) * P + col * 4);
            odd = *reinterpret_cast<const float4*>(start + (size_t)(n0 + 2 * r + 1) * P + col * 4);
        }
        S[r][0] = make_float2(even.x, odd.x); S[r][1] = make_float2(even.y, odd.y);
        S[r][2] = make_float2(even.z, odd.z); S[r][3] = make_float2(even.w, odd.w);
    }
    const float rate = a.rate[head], bias = a.dt_bias[head], skip = a.skip[head];
    float log_sum = 0.f;
    for (int t0 = t_begin; t0 < t_end; t0 += SS_PTILE) {
        const int nt = min(SS_PTILE, t_end - t0);
        __syncthreads();                                             // the tile before is walked, summed and stored
        if (tid < 32) {
            // a lane per token: its step size, then the running sum of the tile's step sizes by shuffles
            float dt = 0.f;
            if (tid < nt) dt = ss_softplus(ss_load(a.proj, a.dtype, (size_t)(t0 + tid) * a.ld + a.dt_off + head) + bias);
            float sum = dt;
#pragma unroll
            for (int off = 1; off < SS_PTILE; off *= 2) {
                const float below = __shfl_up_sync(0xffffffffu, sum, off);
                if (tid >= off) sum += below;
            }
            if (tid < nt) {
                meta[tid] = expf(-rate * dt);
                meta[SS_PTILE + tid] = expf(-rate * sum);
                meta[2 * SS_PTILE + tid] = dt;
                if (ENDS_ONLY && tid == nt - 1) meta[3 * SS_PTILE] = -rate * sum;
            }
        }
        __syncthreads();
        const bool relative = meta[SS_PTILE + nt - 1] >= SS_RELATIVE_FLOOR;
        if (ENDS_ONLY && tid == 0) log_sum += meta[3 * SS_PTILE];
        for (int k = warp; k < nt; k += warps) {
            const size_t row = (size_t)(t0 + k) * a.channels;
            for (int p = lane * 4; p < P; p += 128) {
                const float4 v = ss_load4(a.u, a.dtype, row + head * P + p);
                *reinterpret_cast<float4*>(xs + 2 * (k * P + p)) = make_float4(v.x, v.x, v.y, v.y);
                *reinterpret_cast<float4*>(xs + 2 * (k * P + p) + 4) = make_float4(v.z, v.z, v.w, v.w);
            }
            const float scale = relative ? meta[2 * SS_PTILE + k] / meta[SS_PTILE + k] : meta[2 * SS_PTILE + k];
            for (int n = lane * 4; n < N; n += 128) {
                float4 v = ss_load4(a.u, a.dtype, row + inner + group * N + n);
                v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
                *reinterpret_cast<float4*>(bs + k * N + n) = v;
                if (!ENDS_ONLY)
                    *reinterpret_cast<float4*>(cs + k * N + n) = ss_load4(a.u, a.dtype, row + inner + (a.groups + group) * N + n);
            }
        }
        __syncthreads();
        if (active) {
            // the branch is taken outside the walk: one copy of the loop for each form
            auto walk = [&](auto form) {
                constexpr bool RELATIVE = decltype(form)::value;
                for (int k = 0; k < nt; ++k) {
                    const float4 xa = *reinterpret_cast<const float4*>(xs + 2 * (k * P + col * 4));
                    const float4 xb = *reinterpret_cast<const float4*>(xs + 2 * (k * P + col * 4) + 4);
                    const float2 xv[4] = {make_float2(xa.x, xa.y), make_float2(xa.z, xa.w), make_float2(xb.x, xb.y),
                                          make_float2(xb.z, xb.w)};
                    float2 acc[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[c] = make_float2(0.f, 0.f);
                    const float ak = RELATIVE ? 1.f : meta[k];
                    const float2 aa = make_float2(ak, ak);
#pragma unroll
                    for (int q = 0; q < R / 4; ++q) {
                        const float4 b4 = *reinterpret_cast<const float4*>(bs + k * N + n0 + 4 * q);
                        float4 c4 = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (!ENDS_ONLY) c4 = *reinterpret_cast<const float4*>(cs + k * N + n0 + 4 * q);
                        const float2 bp[2] = {make_float2(b4.x, b4.y), make_float2(b4.z, b4.w)};
                        const float2 cp[2] = {make_float2(c4.x, c4.y), make_float2(c4.z, c4.w)};
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                float2& s = S[2 * q + h][c];
                                if (RELATIVE) s = __ffma2_rn(bp[h], xv[c], s);
                                else s = __ffma2_rn(aa, s, __fmul2_rn(bp[h], xv[c]));
                                if (!ENDS_ONLY) acc[c] = __ffma2_rn(s, cp[h], acc[c]);
                            }
                        }
                    }
                    if (!ENDS_ONLY) {
                        const float post = RELATIVE ? meta[SS_PTILE + k] : 1.f;
                        *reinterpret_cast<float4*>(ypart + ((size_t)k * NG + ng) * P + col * 4) =
                            make_float4(post * (acc[0].x + acc[0].y), post * (acc[1].x + acc[1].y),
                                        post * (acc[2].x + acc[2].y), post * (acc[3].x + acc[3].y));
                    }
                }
            };
            if (relative) walk(SsForm<true>());
            else walk(SsForm<false>());
            if (relative) {
                const float last = meta[SS_PTILE + nt - 1];
                const float2 ll = make_float2(last, last);
#pragma unroll
                for (int r = 0; r < R / 2; ++r)
#pragma unroll
                    for (int c = 0; c < 4; ++c) S[r][c] = __fmul2_rn(S[r][c], ll);
            }
        }
        if (!ENDS_ONLY) {
            __syncthreads();
            for (int i = tid * 4; i < nt * P; i += blockDim.x * 4) {     // P is a multiple of 4: four columns of one token
                const int k = i / P, p = i - k * P;
                float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int g = 0; g < NG; ++g) {
                    const float4 v = *reinterpret_cast<const float4*>(ypart + ((size_t)k * NG + g) * P + p);
                    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
                }
                const float* x = xs + 2 * (k * P + p);
                *reinterpret_cast<float4*>(a.y + (size_t)(t0 + k) * inner + head * P + p) =
                    make_float4(fmaf(skip, x[0], s.x), fmaf(skip, x[2], s.y), fmaf(skip, x[4], s.z), fmaf(skip, x[6], s.w));
            }
        }
    }
    float* dst = nullptr;
    if (ENDS_ONLY) dst = a.part_state + (((size_t)seg * a.heads + head) * a.parts + part) * N * P;
    else if (last_part && a.write_state) dst = a.state + ((size_t)slot * a.heads + head) * N * P;
    if (dst != nullptr && active) {
#pragma unroll
        for (int r = 0; r < R / 2; ++r) {
            *reinterpret_cast<float4*>(dst + (size_t)(n0 + 2 * r) * P + col * 4) =
                make_float4(S[r][0].x, S[r][1].x, S[r][2].x, S[r][3].x);
            *reinterpret_cast<float4*>(dst + (size_t)(n0 + 2 * r + 1) * P + col * 4) =
                make_float4(S[r][0].y, S[r][1].y, S[r][2].y, S[r][3].y);
        }
    }
    if (ENDS_ONLY) {
        if (tid == 0) a.part_log[((size_t)seg * a.heads + head) * a.parts + part] = log_sum;
        return;
    }
    if (last_part && a.write_state) ss_keep_inputs(a, head, group, seg_start, seg_len, slot, tid);
}

// ---------------------------------------------------------------- long segments on the tensor cores
// A part of SSM_PART tokens that starts from the state S0, with l_i the sum of the logarithms of the decays up to and
// including token i (l_i <= 0, float32):
//   y_i   = exp(l_i) S0^T C_i + sum_(j<=i) (C_i . B_j) exp(l_i - l_j) dt_j x_j + D x_i
//   S_end = exp(l_last) S0 + sum_j exp(l_last - l_j) dt_j B_j x_j^T
// Only differences l_i - l_j <= 0 are exponentiated, so nothing overflows however fast a head forgets. x, B and C are
// the bfloat16 numbers that left the convolution and enter their products as they are; what carries a step size, a
// decay or the state is float32 and enters its product as a sum of two bfloat16 numbers (v = hi + lo, hi = bf16(v),
// lo = bf16(v - hi): sixteen bits of mantissa), each half with a product of its own, sums in float32. Three launches:
// every part's end state from zero (B'^T X); the parts' start states (stored as their two halves) and the segment's
// last state, element by element; then every part's outputs (G = C B^T, Y1 = C S0, M = G * decays, Y2 = M X). A block
// per (head, segment, part); rows past the segment's end are zero. Rows in shared memory are padded by 16 bytes so
// that a fragment's rows fall into different banks; buffers whose contents are dead take the next phase's results.
#include <mma.h>
using namespace nvcuda;
#define SSM_PART 64
#define SSM_THREADS 256

struct SsmLayout {
    int ldn, ldp, ldm, ldg, ldy;                       // elements: bfloat16 rows of N, P and SSM_PART; float32 rows of G and Y
    size_t c, b, x, s_hi, s_lo, g, meta, total, ends_total;
};
static __host__ __device__ inline size_t ssm_max(size_t a, size_t b) { return a > b ? a : b; }
static __host__ __device__ inline SsmLayout ssm_layout(int P, int N) {
    SsmLayout L;
    L.ldn = N + 8; L.ldp = P + 8; L.ldm = SSM_PART + 8; L.ldg = SSM_PART + 4; L.ldy = P + 4;
    size_t o = 0;
    L.c = o; o += (size_t)SSM_PART * L.ldn * 2;                                   // C (outputs); low halves of B' (end states)
    L.b = o; o += ssm_max((size_t)SSM_PART * L.ldn * 2, (size_t)SSM_PART * L.ldy * 4);   // B, then Y1; high halves of B'
    L.x = o; o += (size_t)SSM_PART * L.ldp * 2;
    L.meta = o; o += 4 * SSM_PART * sizeof(float);                                // dt, l, a warp's total
    L.ends_total = o;
    const size_t half = ssm_max((size_t)N * L.ldp * 2, (size_t)SSM_PART * L.ldm * 2);
    L.s_hi = o; o += half;                                                        // S0's halves, then M's
    L.s_lo = o; o += half;
    L.g = o; o += ssm_max((size_t)SSM_PART * L.ldg * 4, (size_t)SSM_PART * L.ldy * 4);   // G, then Y2
    L.total = o;
    return L;
}

__device__ __forceinline__ void ssm_split(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}
__device__ __forceinline__ void ssm_copy16(void* dst_shared, const void* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst_shared);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void ssm_copies_done() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// dts[k] = softplus(dt_k + bias) and logs[k] = -rate (dt_0 + .. + dt_k) for the part's tokens; zero steps past its end
__device__ __forceinline__ void ssm_steps(const SsScanArgs& a, int head, int t0, int nt, float* dts, float* logs, float* total) {
    const int tid = threadIdx.x;
    const float rate = a.rate[head], bias = a.dt_bias[head];
    if (tid < SSM_PART) {                                                // two whole warps
        float dt = 0.f;
        if (tid < nt) dt = ss_softplus(ss_load(a.proj, a.dtype, (size_t)(t0 + tid) * a.ld + a.dt_off + head) + bias);
        float sum = dt;
#pragma unroll
        for (int off = 1; off < 32; off *= 2) {
            const float below = __shfl_up_sync(0xffffffffu, sum, off);
            if ((tid & 31) >= off) sum += below;
        }
        if (tid == 31) total[0] = sum;
        dts[tid] = dt;
        logs[tid] = sum;
    }
    __syncthreads();
    if (tid < SSM_PART) logs[tid] = -rate * (tid >= 32 ? logs[tid] + total[0] : logs[tid]);
    __syncthreads();
}

// rows [SSM_PART, cols] of bfloat16 from u (row stride a.channels) into shared memory rows of ld elements, sixteen
// bytes a copy, all in flight at once; rows past nt are zeroed
__device__ __forceinline__ void ssm_copy_rows(const SsScanArgs& a, int t0, int nt, int col0, int cols, __nv_bfloat16* dst, int ld) {
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(a.u);
    const int chunks = cols / 8;
    for (int i = threadIdx.x; i < SSM_PART * chunks; i += blockDim.x) {
        const int k = i / chunks, c = (i - k * chunks) * 8;
        if (k < nt) ssm_copy16(dst + (size_t)k * ld + c, u + (size_t)(t0 + k) * a.channels + col0 + c);
        else *reinterpret_cast<uint4*>(dst + (size_t)k * ld + c) = make_uint4(0u, 0u, 0u, 0u);
    }
}

__global__ void __launch_bounds__(SSM_THREADS)
ss_part_ends_mma_kernel(const SsScanArgs a) {
    extern __shared__ __align__(128) unsigned char ssm_smem[];
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y, part = blockIdx.z;
    const int P = a.P, N = a.N;
    const int seg_start = a.cu_seqlens[seg], seg_len = a.cu_seqlens[seg + 1] - seg_start;
    const int parts_here = max(1, (seg_len + SSM_PART - 1) / SSM_PART);
    if (part >= parts_here || seg_len <= 0) return;
    const int t0 = seg_start + part * SSM_PART, nt = min(SSM_PART, seg_start + seg_len - t0);
    const SsmLayout L = ssm_layout(P, N);
    __nv_bfloat16* Bl = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.c);
    __nv_bfloat16* Bh = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.b);
    __nv_bfloat16* Xs = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.x);
    float* dts = reinterpret_cast<float*>(ssm_smem + L.meta);
    float* logs = dts + SSM_PART;
    const int tid = threadIdx.x, warp = tid / 32, warps = blockDim.x / 32;
    const int inner = a.heads * P, group = head / (a.heads / a.groups);
    ssm_copy_rows(a, t0, nt, head * P, P, Xs, L.ldp);
    ssm_copy_rows(a, t0, nt, inner + group * N, N, Bh, L.ldn);           // B as it is; scaled in place below
    ssm_steps(a, head, t0, nt, dts, logs, logs + SSM_PART);              // while the copies fly
    ssm_copies_done();
    __syncthreads();
    const float l_last = logs[nt - 1];
    for (int i = tid; i < SSM_PART * (N / 2); i += blockDim.x) {         // B'_j = exp(l_last - l_j) dt_j B_j in two halves
        const int k = i / (N / 2), n = (i - k * (N / 2)) * 2;
        const float w = k < nt ? expf(l_last - logs[k]) * dts[k] : 0.f;
        __nv_bfloat162* hi = reinterpret_cast<__nv_bfloat162*>(Bh + (size_t)k * L.ldn + n);
        const float2 v = __bfloat1622float2(*hi);
        __nv_bfloat16 h0, l0, h1, l1;
        ssm_split(v.x * w, h0, l0);
        ssm_split(v.y * w, h1, l1);
        *hi = __halves2bfloat162(h0, h1);
        *reinterpret_cast<__nv_bfloat162*>(Bl + (size_t)k * L.ldn + n) = __halves2bfloat162(l0, l1);
    }
    __syncthreads();
    float* dst = a.part_state + (((size_t)seg * a.heads + head) * a.parts + part) * N * P;
    const int tiles_p = P / 16, tiles = (N / 16) * tiles_p;
    for (int tile = warp; tile < tiles; tile += warps) {
        const int ti = tile / tiles_p, tj = tile - ti * tiles_p;
        wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
        wmma::fill_fragment(acc, 0.f);
#pragma unroll
        for (int kk = 0; kk < SSM_PART / 16; ++kk) {
            wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::col_major> fa;    // B'^T: element (n, j) = B'[j][n]
            wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> fb;
            wmma::load_matrix_sync(fb, Xs + (size_t)kk * 16 * L.ldp + tj * 16, L.ldp);
            wmma::load_matrix_sync(fa, Bh + (size_t)kk * 16 * L.ldn + ti * 16, L.ldn);
            wmma::mma_sync(acc, fa, fb, acc);
            wmma::load_matrix_sync(fa, Bl + (size_t)kk * 16 * L.ldn + ti * 16, L.ldn);
            wmma::mma_sync(acc, fa, fb, acc);
        }
        wmma::store_matrix_sync(dst + (size_t)ti * 16 * P + tj * 16, acc, P, wmma::mem_row_major);
    }
    if (tid == 0) a.part_log[((size_t)seg * a.heads + head) * a.parts + part] = l_last;
}

// Element by element over a segment's parts: start_0 = the request's state, start_(k+1) = exp(l_k) start_k + E_k. The
// start states go to `starts` as their two bfloat16 halves ([.., part, half, N P]); the state after the last part goes
// to the request's slot.
__global__ void __launch_bounds__(256)
ss_prefix_all_kernel(float* __restrict__ state, const int* __restrict__ cu_seqlens, const int* __restrict__ slots,
                     const float* __restrict__ part_state, __nv_bfloat16* __restrict__ starts, const float* __restrict__ part_log,
                     int heads, int elems, int parts, int write_state) {
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y;
    const int seg_len = cu_seqlens[seg + 1] - cu_seqlens[seg];
    if (seg_len <= 0) return;
    const int parts_here = (seg_len + SSM_PART - 1) / SSM_PART;
    float* s0 = state + ((size_t)slots[seg] * heads + head) * elems;
    const float* ps = part_state + ((size_t)seg * heads + head) * parts * elems;
    __nv_bfloat16* st = starts + ((size_t)seg * heads + head) * parts * elems * 2;
    const float* pl = part_log + ((size_t)seg * heads + head) * parts;
    for (int i = 2 * (blockIdx.z * blockDim.x + threadIdx.x); i < elems; i += 2 * gridDim.z * blockDim.x) {   // elems is even
        float2 s = *reinterpret_cast<const float2*>(s0 + i);
        for (int k0 = 0; k0 < parts_here; k0 += 8) {                     // eight parts' loads in flight ahead of the chain
            float2 e[8];
            float d[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool have = k0 + j < parts_here;
                e[j] = have ? *reinterpret_cast<const float2*>(ps + (size_t)(k0 + j) * elems + i) : make_float2(0.f, 0.f);
                d[j] = have ? expf(pl[k0 + j]) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j < parts_here) {
                    __nv_bfloat16 hx, lx, hy, ly;
                    ssm_split(s.x, hx, lx);
                    ssm_split(s.y, hy, ly);
                    *reinterpret_cast<__nv_bfloat162*>(st + (size_t)(k0 + j) * 2 * elems + i) = __halves2bfloat162(hx, hy);
                    *reinterpret_cast<__nv_bfloat162*>(st + (size_t)(k0 + j) * 2 * elems + elems + i) = __halves2bfloat162(lx, ly);
                    s.x = fmaf(d[j], s.x, e[j].x);
                    s.y = fmaf(d[j], s.y, e[j].y);
                }
            }
        }
        if (write_state) *reinterpret_cast<float2*>(s0 + i) = s;
    }
}

__global__ void __launch_bounds__(SSM_THREADS, 2)
ss_part_out_mma_kernel(const SsScanArgs a, const __nv_bfloat16* __restrict__ starts) {
    extern __shared__ __align__(128) unsigned char ssm_smem[];
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y, part = blockIdx.z;
    const int P = a.P, N = a.N;
    const int seg_start = a.cu_seqlens[seg], seg_len = a.cu_seqlens[seg + 1] - seg_start;
    const int parts_here = max(1, (seg_len + SSM_PART - 1) / SSM_PART);
    if (part >= parts_here || seg_len <= 0) return;
    const int t0 = seg_start + part * SSM_PART, nt = min(SSM_PART, seg_start + seg_len - t0);
    const SsmLayout L = ssm_layout(P, N);
    __nv_bfloat16* Cs = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.c);
    __nv_bfloat16* Bs = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.b);
    float* Y1 = reinterpret_cast<float*>(ssm_smem + L.b);                 // once G is done
    __nv_bfloat16* Xs = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.x);
    __nv_bfloat16* Sh = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.s_hi);
    __nv_bfloat16* Sl = reinterpret_cast<__nv_bfloat16*>(ssm_smem + L.s_lo);
    __nv_bfloat16* Mh = Sh;                                              // once Y1 is done
    __nv_bfloat16* Ml = Sl;
    float* G = reinterpret_cast<float*>(ssm_smem + L.g);
    float* Y2 = G;                                                       // once M is done
    float* dts = reinterpret_cast<float*>(ssm_smem + L.meta);
    float* logs = dts + SSM_PART;
    const int tid = threadIdx.x, warp = tid / 32, warps = blockDim.x / 32;
    const int inner = a.heads * P, group = head / (a.heads / a.groups);
    ssm_copy_rows(a, t0, nt, inner + group * N, N, Bs, L.ldn);
    ssm_copy_rows(a, t0, nt, inner + (a.groups + group) * N, N, Cs, L.ldn);
    ssm_copy_rows(a, t0, nt, head * P, P, Xs, L.ldp);
    {   // the part's start state, stored as its two halves
        const __nv_bfloat16* src = starts + (((size_t)seg * a.heads + head) * a.parts + part) * 2 * N * P;
        const int chunks = P / 8;
        for (int i = tid; i < N * chunks; i += blockDim.x) {
            const int n = i / chunks, c = (i - n * chunks) * 8;
            ssm_copy16(Sh + (size_t)n * L.ldp + c, src + (size_t)n * P + c);
            ssm_copy16(Sl + (size_t)n * L.ldp + c, src + (size_t)(N + n) * P + c);
        }
    }
    ssm_steps(a, head, t0, nt, dts, logs, logs + SSM_PART);              // while the copies fly
    ssm_copies_done();
    __syncthreads();
    const int tiles_p = P / 16, rows = SSM_PART / 16;
    for (int tile = warp; tile < rows * (rows + 1) / 2; tile += warps) { // G = C B^T, on and below its diagonal
        int ti = 0, first = 0;
        while (first + ti + 1 <= tile) { first += ti + 1; ++ti; }
        const int tj = tile - first;
        wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
        wmma::fill_fragment(acc, 0.f);
        for (int kk = 0; kk < N / 16; ++kk) {
            wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> fa;
            wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::col_major> fb;    // B^T: element (n, j) = B[j][n]
            wmma::load_matrix_sync(fa, Cs + (size_t)ti * 16 * L.ldn + kk * 16, L.ldn);
            wmma::load_matrix_sync(fb, Bs + (size_t)tj * 16 * L.ldn + kk * 16, L.ldn);
            wmma::mma_sync(acc, fa, fb, acc);
        }
        wmma::store_matrix_sync(G + ti * 16 * L.ldg + tj * 16, acc, L.ldg, wmma::mem_row_major);
    }
    __syncthreads();                                                     // B is read; its place takes Y1
    for (int tile = warp; tile < rows * tiles_p; tile += warps) {        // Y1 = C S0
        const int ti = tile / tiles_p, tj = tile - ti * tiles_p;
        wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
        wmma::fill_fragment(acc, 0.f);
        for (int kk = 0; kk < N / 16; ++kk) {
            wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> fa;
            wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> fb;
            wmma::load_matrix_sync(fa, Cs + (size_t)ti * 16 * L.ldn + kk * 16, L.ldn);
            wmma::load_matrix_sync(fb, Sh + (size_t)kk * 16 * L.ldp + tj * 16, L.ldp);
            wmma::mma_sync(acc, fa, fb, acc);
            wmma::load_matrix_sync(fb, Sl + (size_t)kk * 16 * L.ldp + tj * 16, L.ldp);
            wmma::mma_sync(acc, fa, fb, acc);
        }
        wmma::store_matrix_sync(Y1 + (size_t)ti * 16 * L.ldy + tj * 16, acc, L.ldy, wmma::mem_row_major);
    }
    __syncthreads();                                                     // S0 is read; its place takes M
    // M_ij = G_ij exp(l_i - l_j) dt_j for j <= i inside the part, zero elsewhere; in two halves
    for (int idx = tid; idx < SSM_PART * SSM_PART; idx += blockDim.x) {
        const int i = idx / SSM_PART, j = idx - i * SSM_PART;
        float v = 0.f;
        if (j <= i && i < nt) v = G[i * L.ldg + j] * expf(logs[i] - logs[j]) * dts[j];
        ssm_split(v, Mh[i * L.ldm + j], Ml[i * L.ldm + j]);
    }
    __syncthreads();                                                     // G is read; its place takes Y2
    for (int tile = warp; tile < rows * tiles_p; tile += warps) {        // Y2 = M X
        const int ti = tile / tiles_p, tj = tile - ti * tiles_p;
        wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
        wmma::fill_fragment(acc, 0.f);
        for (int kk = 0; kk <= ti; ++kk) {                               // M is zero right of its diagonal
            wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> fa;
            wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> fb;
            wmma::load_matrix_sync(fb, Xs + (size_t)kk * 16 * L.ldp + tj * 16, L.ldp);
            wmma::load_matrix_sync(fa, Mh + ti * 16 * L.ldm + kk * 16, L.ldm);
            wmma::mma_sync(acc, fa, fb, acc);
            wmma::load_matrix_sync(fa, Ml + ti * 16 * L.ldm + kk * 16, L.ldm);
            wmma::mma_sync(acc, fa, fb, acc);
        }
        wmma::store_matrix_sync(Y2 + (size_t)ti * 16 * L.ldy + tj * 16, acc, L.ldy, wmma::mem_row_major);
    }
    __syncthreads();
    const float skip = a.skip[head];
    const int quads = P / 4;
    for (int idx = tid; idx < nt * quads; idx += blockDim.x) {
        const int i = idx / quads, p = (idx - i * quads) * 4;
        const float decayed = expf(logs[i]);
        const float4 y1 = *reinterpret_cast<const float4*>(Y1 + (size_t)i * L.ldy + p);
        const float4 y2 = *reinterpret_cast<const float4*>(Y2 + (size_t)i * L.ldy + p);
        const __nv_bfloat16* x = Xs + (size_t)i * L.ldp + p;
        *reinterpret_cast<float4*>(a.y + (size_t)(t0 + i) * inner + head * P + p) =
            make_float4(fmaf(decayed, y1.x, y2.x) + skip * __bfloat162float(x[0]),
                        fmaf(decayed, y1.y, y2.y) + skip * __bfloat162float(x[1]),
                        fmaf(decayed, y1.z, y2.z) + skip * __bfloat162float(x[2]),
                        fmaf(decayed, y1.w, y2.w) + skip * __bfloat162float(x[3]));
    }
    if (part == parts_here - 1 && a.write_state) ss_keep_inputs(a, head, group, seg_start, seg_len, a.slots[seg], tid);
}

// Sizes and buffers the tensor-core form takes: bfloat16 activations, parts of SSM_PART tokens, head sizes in whole
// fragments, rows on 16-byte boundaries. part_state then holds twice segments * heads * parts * N * P floats: the
// parts' end states and, behind them, their start states in halves.
static int ssm_supported(const SsScanArgs& a, int dtype) {
    if (dtype != TTB_DTYPE_BF16 || a.parts < 2 || a.part_len != SSM_PART) return 0;
    if (a.P % 16 || a.N % 16 || a.channels % 8) return 0;
    if (ssm_layout(a.P, a.N).total > 200 * 1024) return 0;
    return (uintptr_t)a.u % 16 == 0 && (uintptr_t)a.y % 16 == 0 && (uintptr_t)a.part_state % 32 == 0 && (uintptr_t)a.state % 16 == 0;
}

static void ssm_launch(const SsScanArgs& a, int segments, cudaStream_t stream) {
    const SsmLayout L = ssm_layout(a.P, a.N);
    static TtbOncePerDevice once;
    if (once.pending()) {
        cudaFuncSetAttribute(ss_part_ends_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(ss_part_out_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        once.mark();
    }
    const dim3 grid(a.heads, segments, a.parts);
    const int elems = a.N * a.P;
    __nv_bfloat16* starts = reinterpret_cast<__nv_bfloat16*>(a.part_state + (size_t)segments * a.heads * a.parts * elems);
    ttb_launch(ss_part_ends_mma_kernel, grid, SSM_THREADS, L.ends_total, stream, a);
    ttb_launch(ss_prefix_all_kernel, dim3(a.heads, segments, (elems / 2 + 255) / 256), 256, 0, stream, a.state, a.cu_seqlens, a.slots,
               (const float*)a.part_state, starts, (const float*)a.part_log, a.heads, elems, a.parts, a.write_state);
    ttb_launch(ss_part_out_mma_kernel, grid, SSM_THREADS, L.total, stream, a, (const __nv_bfloat16*)starts);
}

// start_(k+1) = exp(L_k) start_k + E_k over the parts of a segment, element by element; E_k's place takes start_(k+1)
__global__ void __launch_bounds__(256)
ss_prefix_kernel(const float* __restrict__ state, const int* __restrict__ cu_seqlens, const int* __restrict__ slots,
                 float* __restrict__ part_state, const float* __restrict__ part_log, int heads, int elems, int parts, int part_len) {
    pdl_wait();
    pdl_launch_dependents();
    const int head = blockIdx.x, seg = blockIdx.y;
    const int seg_len = cu_seqlens[seg + 1] - cu_seqlens[seg];
    const int parts_here = (seg_len + part_len - 1) / part_len;
    if (parts_here < 2) return;
    const float* s0 = state + ((size_t)slots[seg] * heads + head) * elems;
    float* ps = part_state + ((size_t)seg * heads + head) * parts * elems;
    const float* pl = part_log + ((size_t)seg * heads + head) * parts;
    for (int i = blockIdx.z * blockDim.x + threadIdx.x; i < elems; i += gridDim.z * blockDim.x) {
        float s = s0[i];
        for (int k0 = 0; k0 + 1 < parts_here; k0 += 8) {                 // eight parts' loads in flight ahead of the chain
            float e[8], d[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool have = k0 + j + 1 < parts_here;
                e[j] = have ? ps[(size_t)(k0 + j) * elems + i] : 0.f;
                d[j] = have ? expf(pl[k0 + j]) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j + 1 < parts_here) {
                    s = fmaf(d[j], s, e[j]);
                    ps[(size_t)(k0 + j) * elems + i] = s;
                }
            }
        }
    }
}

template <int PC, int R>
static void ss_scan_launch(const SsScanArgs& a, int segments, int threads, size_t smem, bool ends_only, cudaStream_t stream) {
    dim3 grid(a.heads, segments, a.parts);
    static TtbOncePerDevice once;
    if (once.pending()) {
        cudaFuncSetAttribute(ss_scan_kernel<PC, R, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(ss_scan_kernel<PC, R, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        once.mark();
    }
    if (ends_only) ttb_launch(ss_scan_kernel<PC, R, true>, grid, threads, smem, stream, a);
    else ttb_launch(ss_scan_kernel<PC, R, false>, grid, threads, smem, stream, a);
}

template <int R>
static void ss_scan_packed_launch(const SsScanArgs& a, int segments, int threads, size_t smem, bool ends_only, cudaStream_t stream) {
    dim3 grid(a.heads, segments, a.parts);
    static TtbOncePerDevice once;
    if (once.pending()) {
        cudaFuncSetAttribute(ss_scan_packed_kernel<R, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(ss_scan_packed_kernel<R, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        once.mark();
    }
    // the parts' end states need no outputs: without their buffer more blocks fit an SM
    const size_t ends_smem = (size_t)SS_PTILE * (2 * a.P + 2 * a.N + 4) * sizeof(float);
    if (ends_only) ttb_launch(ss_scan_packed_kernel<R, true>, grid, threads, ends_smem, stream, a);
    else ttb_launch(ss_scan_packed_kernel<R, false>, grid, threads, smem, stream, a);
}

// How the state of one head is dealt out: rows per thread (R, a power of two up to 32) and row groups (NG).
static bool ss_plan(int P, int N, int& pc, int& r, int& ng) {
    pc = (P % 4 == 0) ? 4 : 1;
    const int cols = P / pc;
    for (r = 1; r <= 32; r *= 2) {
        ng = (N + r - 1) / r;
        const int threads = cols * ng;
        if (threads <= (pc == 4 && r < 16 ? 128 : 256) || (r == 32 && pc == 1 && threads <= 1024)) return true;
    }
    return false;
}

TTB_EXPORT int ttb_state_space_supports(int P, int N) {
    int pc, r, ng;
    if (P < 1 || N < 1 || !ss_plan(P, N, pc, r, ng)) return 0;
    const size_t smem = ((size_t)SS_TILE * (P + 2 * N + 2) + (size_t)SS_TILE * ng * P) * sizeof(float);
    return smem <= 200 * 1024;
}

TTB_EXPORT int ttb_conv_silu(const void* in, int dtype, int ld, const float* conv_w, const float* conv_b, const int* seg_of_token,
                             const int* cu_seqlens, const int* slots, const void* tail, void* out, int tokens, int channels,
                             int taps, cudaStream_t stream) {
    if (tokens == 0 || channels == 0) return TTB_OK;
    if (!in || !conv_w || !conv_b || !seg_of_token || !cu_seqlens || !slots || !out || taps < 1 || (taps > 1 && !tail))
        return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    const size_t unit = dtype == TTB_DTYPE_BF16 ? 8 : 16;               // bytes of four values
    const bool quads = channels % 4 == 0 && ld % 4 == 0 && (uintptr_t)in % unit == 0 && (uintptr_t)out % unit == 0 &&
                       (uintptr_t)conv_b % 16 == 0 && (taps == 1 || (uintptr_t)tail % unit == 0);
    const size_t total = (size_t)tokens * channels;
    const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    if (quads && tokens >= 64 * SS_CONV_RUN && taps >= 2 && taps <= 4) {
        const dim3 grid((tokens + SS_CONV_RUN - 1) / SS_CONV_RUN, (channels / 4 + 127) / 128);
        if (taps == 2)
            ttb_launch(ss_conv_silu_run_kernel<2>, grid, 128, 0, stream, in, dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens,
                       slots, tail, out, tokens, channels);
        else if (taps == 3)
            ttb_launch(ss_conv_silu_run_kernel<3>, grid, 128, 0, stream, in, dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens,
                       slots, tail, out, tokens, channels);
        else
            ttb_launch(ss_conv_silu_run_kernel<4>, grid, 128, 0, stream, in, dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens,
                       slots, tail, out, tokens, channels);
    } else if (quads)
        ttb_launch(ss_conv_silu4_kernel, tokens < 148 * 16 ? tokens : 148 * 16, channels / 4 >= 256 ? 256 : 128, 0, stream, in,
                   dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens, slots, tail, out, tokens, channels, taps);
    else
        ttb_launch(ss_conv_silu_kernel, blocks, 256, 0, stream, in, dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens, slots,
                   tail, out, tokens, channels, taps);
    return ttb_launch_status();
}

// u [T, heads P + 2 groups N] after the convolution; proj [T, ld] with the raw convolution inputs at column conv_off and the
// raw step sizes at dt_off. parts > 1: part_state [segments, heads, parts, N P] and part_log [segments, heads, parts] are
// scratch, and three launches run (ends, prefix, walk); parts == 1: one launch.
TTB_EXPORT int ttb_state_space_scan(const void* u, const void* proj, int dtype, int ld, int conv_off, int dt_off,
                                    const float* dt_bias, const float* rate, const float* skip, const int* cu_seqlens,
                                    const int* slots, float* state, void* tail, float* y, int segments, int heads, int P, int N,
                                    int groups, int taps, int write_state, float* part_state, float* part_log, int parts,
                                    int part_len, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!u || !proj || !dt_bias || !rate || !skip || !cu_seqlens || !slots || !state || !y || (taps > 1 && !tail))
        return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    if (heads < 1 || groups < 1 || heads % groups || heads > 65535 || segments > 65535 || parts < 1 || parts > 65535)
        return TTB_ERR_UNSUPPORTED;
    if (parts > 1 && (!part_state || !part_log || part_len < 1)) return TTB_ERR_ARGUMENT;
    int pc, r, ng;
    if (!ttb_state_space_supports(P, N) || !ss_plan(P, N, pc, r, ng)) return TTB_ERR_UNSUPPORTED;
    SsScanArgs a;
    a.u = u; a.proj = proj; a.dtype = dtype; a.ld = ld; a.conv_off = conv_off; a.dt_off = dt_off;
    a.dt_bias = dt_bias; a.rate = rate; a.skip = skip; a.cu_seqlens = cu_seqlens; a.slots = slots;
    a.state = state; a.tail = tail; a.y = y; a.part_state = part_state; a.part_log = part_log;
    a.heads = heads; a.P = P; a.N = N; a.groups = groups; a.channels = heads * P + 2 * groups * N; a.taps = taps;
    a.write_state = write_state; a.parts = parts; a.part_len = part_len; a.NG = ng;
    int threads = (P / pc) * ng;
    threads = (threads + 31) / 32 * 32;
    if (threads < 64) threads = 64;
    const size_t smem = ((size_t)SS_TILE * (P + 2 * N + 2) + (size_t)SS_TILE * ng * P) * sizeof(float);
#define SS_RUN(PC, R, ENDS) ss_scan_launch<PC, R>(a, segments, threads, smem, ENDS, stream)
#define SS_PICK(ENDS)                                                                          \
    do {                                                                                       \
        if (pc == 4) {                                                                         \
            switch (r) {                                                                       \
                case 1: SS_RUN(4, 1, ENDS); break;   case 2: SS_RUN(4, 2, ENDS); break;        \
                case 4: SS_RUN(4, 4, ENDS); break;   case 8: SS_RUN(4, 8, ENDS); break;        \
                case 16: SS_RUN(4, 16, ENDS); break; default: SS_RUN(4, 32, ENDS); break;      \
            }                                                                                  \
        } else {                                                                               \
            switch (r) {                                                                       \
                case 1: SS_RUN(1, 1, ENDS); break;   case 2: SS_RUN(1, 2, ENDS); break;        \
                case 4: SS_RUN(1, 4, ENDS); break;   case 8: SS_RUN(1, 8, ENDS); break;        \
                case 16: SS_RUN(1, 16, ENDS); break; default: SS_RUN(1, 32, ENDS); break;      \
            }                                                                                  \
        }                                                                                      \
    } while (0)
    // the packed walk: whole groups of four columns and of four rows, float32 stores of the state on 16-byte boundaries
    const size_t packed_smem = ((size_t)SS_PTILE * (2 * P + 2 * N + 4) + (size_t)SS_PTILE * ng * P) * sizeof(float);
    const bool packed = pc == 4 && r >= 4 && N % r == 0 && N % 4 == 0 && threads <= 256 && packed_smem <= 200 * 1024 &&
                        (dtype == TTB_DTYPE_BF16 ? ((uintptr_t)u % 8 == 0) : ((uintptr_t)u % 16 == 0)) &&
                        (uintptr_t)state % 16 == 0 && (uintptr_t)y % 16 == 0 && (parts == 1 || (uintptr_t)part_state % 16 == 0);
#define SS_PACKED(ENDS)                                                                                        \
    do {                                                                                                       \
        switch (r) {                                                                                           \
            case 4: ss_scan_packed_launch<4>(a, segments, threads, packed_smem, ENDS, stream); break;          \
            case 8: ss_scan_packed_launch<8>(a, segments, threads, packed_smem, ENDS, stream); break;          \
            case 16: ss_scan_packed_launch<16>(a, segments, threads, packed_smem, ENDS, stream); break;        \
            default: ss_scan_packed_launch<32>(a, segments, threads, packed_smem, ENDS, stream); break;        \
        }                                                                                                      \
    } while (0)
    if (ssm_supported(a, dtype)) {
        ssm_launch(a, segments, stream);
        return ttb_launch_status();
    }
    if (parts > 1) {
        if (packed) SS_PACKED(true);
        else SS_PICK(true);
        const int elems = N * P;
        dim3 grid(heads, segments, (elems + 255) / 256);
        ttb_launch(ss_prefix_kernel, grid, 256, 0, stream, (const float*)state, cu_seqlens, slots, part_state,
                   (const float*)part_log, heads, elems, parts, part_len);
    }
    if (packed) SS_PACKED(false);
    else SS_PICK(false);
#undef SS_PACKED
#undef SS_PICK
#undef SS_RUN
    return ttb_launch_status();
}

// ---------------------------------------------------------------- gate, then the RMS norm in equal parts
// out[t, c] = v / sqrt(mean_part(v^2) + eps) * w[c], v = y[t, c] * silu(z[t, c]); a block per (token, part).
#define SS_GATE_KEEP 8
__global__ void __launch_bounds__(128)
ss_gate_norm_kernel(const float* __restrict__ y, const void* __restrict__ z, int z_dtype, int z_stride,
                    const float* __restrict__ weight, float eps, void* __restrict__ out, int out_dtype, int inner, int part) {
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, c0 = blockIdx.y * part;
    // a thread's first SS_GATE_KEEP values stay in registers between the sum and the scaling; wider parts read the rest twice
    float kept[SS_GATE_KEEP];
    float sumsq = 0.f;
#pragma unroll
    for (int j = 0; j < SS_GATE_KEEP; ++j) {
        const int c = threadIdx.x + j * blockDim.x;
        kept[j] = 0.f;
        if (c < part) kept[j] = y[(size_t)t * inner + c0 + c] * ss_silu(ss_load(z, z_dtype, (size_t)t * z_stride + c0 + c));
        sumsq += kept[j] * kept[j];
    }
    for (int c = threadIdx.x + SS_GATE_KEEP * blockDim.x; c < part; c += blockDim.x) {
        const float v = y[(size_t)t * inner + c0 + c] * ss_silu(ss_load(z, z_dtype, (size_t)t * z_stride + c0 + c));
        sumsq += v * v;
    }
    sumsq = block_sum(sumsq, scratch);
    const float scale = 1.f / sqrtf(sumsq / (float)part + eps);
#pragma unroll
    for (int j = 0; j < SS_GATE_KEEP; ++j) {
        const int c = threadIdx.x + j * blockDim.x;
        if (c < part) ss_store(out, out_dtype, (size_t)t * inner + c0 + c, kept[j] * scale * weight[c0 + c]);
    }
    for (int c = threadIdx.x + SS_GATE_KEEP * blockDim.x; c < part; c += blockDim.x) {
        const float v = y[(size_t)t * inner + c0 + c] * ss_silu(ss_load(z, z_dtype, (size_t)t * z_stride + c0 + c));
        ss_store(out, out_dtype, (size_t)t * inner + c0 + c, v * scale * weight[c0 + c]);
    }
}

TTB_EXPORT int ttb_gate_group_norm(const float* y, const void* z, int z_dtype, int z_stride, const float* weight, float eps,
                                   void* out, int out_dtype, int tokens, int inner, int parts, cudaStream_t stream) {
    if (tokens == 0 || inner == 0) return TTB_OK;
    if (!y || !z || !weight || !out || parts < 1 || inner % parts || parts > 65535) return TTB_ERR_ARGUMENT;
    ttb_launch(ss_gate_norm_kernel, dim3(tokens, parts), 128, 0, stream, y, z, z_dtype, z_stride, weight, eps, out, out_dtype,
               inner, inner / parts);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- decode steps: one token a segment
// The walk of one token, the gate and the group norm in one launch. A block per (head, segment): the head's state is read,
// decayed, updated and written once (four columns a thread, row groups side by side, their partial outputs summed in a
// fixed order), v = (S^T C + D x) silu(z) goes to `gated` in float32 and the head's sum of v^2 to `partial`. The block that
// is the last of its norm group to finish (a counter per segment and norm group; it leaves the counter at zero for the
// next step) sums the group's partial sums in head order and writes the normed values. Nobody waits for anybody.
// A norm group holds whole heads: heads is a multiple of norm_groups.
struct SsTokenArgs {
    SsScanArgs s;             // u, proj, offsets, per-head vectors, segments' slots, the state, kept inputs; y = `gated`
    const float* norm_w;      // [heads * P]
    void* out;                // [segments, heads * P], the compute dtype
    float* partial;           // [segments, heads]
    int* counter;             // [segments, norm_groups], zero between launches
    float eps;
    int norm_groups;
};

__global__ void __launch_bounds__(256)
ss_token_kernel(const SsTokenArgs g) {
    extern __shared__ __align__(16) float sst_smem[];
    __shared__ float scratch[32];
    __shared__ int is_last;
    pdl_wait();
    pdl_launch_dependents();
    const SsScanArgs& a = g.s;
    const int head = blockIdx.x, seg = blockIdx.y;
    const int P = a.P, N = a.N;
    const int t = a.cu_seqlens[seg];
    if (a.cu_seqlens[seg + 1] - t != 1) return;
    const int tid = threadIdx.x;
    const int inner = a.heads * P, group = head / (a.heads / a.groups);
    const int cols = P / 4, row_groups = min(blockDim.x / cols, N);
    float* xs = sst_smem;                                    // [P]
    float* bs = xs + P;                                      // [N]  dt B
    float* cs = bs + N;                                      // [N]
    float* ypart = sst_smem + ((P + 2 * N + 3) & ~3);        // [row_groups, P], on a 16-byte boundary
    const int slot = a.slots[seg];
    const float dt = ss_softplus(ss_load(a.proj, a.dtype, (size_t)t * a.ld + a.dt_off + head) + a.dt_bias[head]);
    const float decay = expf(-a.rate[head] * dt);
    const size_t row = (size_t)t * a.channels;
    for (int p = tid; p < P; p += blockDim.x) xs[p] = ss_load(a.u, a.dtype, row + head * P + p);
    for (int n = tid; n < N; n += blockDim.x) {
        bs[n] = dt * ss_load(a.u, a.dtype, row + inner + group * N + n);
        cs[n] = ss_load(a.u, a.dtype, row + inner + (a.groups + group) * N + n);
    }
    __syncthreads();
    const int col = tid % cols, rg = tid / cols;
    if (rg < row_groups) {
        float* S = a.state + ((size_t)slot * a.heads + head) * N * P + col * 4;
        const float4 x = *reinterpret_cast<const float4*>(xs + col * 4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int n0 = rg; n0 < N; n0 += 4 * row_groups) {                // four rows' loads in flight
            float4 s[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + j * row_groups;
                if (n < N) s[j] = *reinterpret_cast<const float4*>(S + (size_t)n * P);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + j * row_groups;
                if (n < N) {
                    const float b = bs[n], c = cs[n];
                    s[j].x = fmaf(decay, s[j].x, b * x.x); s[j].y = fmaf(decay, s[j].y, b * x.y);
                    s[j].z = fmaf(decay, s[j].z, b * x.z); s[j].w = fmaf(decay, s[j].w, b * x.w);
                    acc.x = fmaf(s[j].x, c, acc.x); acc.y = fmaf(s[j].y, c, acc.y);
                    acc.z = fmaf(s[j].z, c, acc.z); acc.w = fmaf(s[j].w, c, acc.w);
                    if (a.write_state) *reinterpret_cast<float4*>(S + (size_t)n * P) = s[j];
                }
            }
        }
        *reinterpret_cast<float4*>(ypart + (size_t)rg * P + col * 4) = acc;
    }
    __syncthreads();
    const float skip = a.skip[head];
    float sumsq = 0.f;
    for (int p = tid; p < P; p += blockDim.x) {
        float y = 0.f;
        for (int r = 0; r < row_groups; ++r) y += ypart[(size_t)r * P + p];
        y = fmaf(skip, xs[p], y);
        const float v = y * ss_silu(ss_load(a.proj, a.dtype, (size_t)t * a.ld + head * P + p));
        a.y[(size_t)t * inner + head * P + p] = v;
        sumsq += v * v;
    }
    sumsq = block_sum(sumsq, scratch);
    const int heads_per = a.heads / g.norm_groups, ng = head / heads_per;
    if (tid == 0) g.partial[(size_t)seg * a.heads + head] = sumsq;
    __threadfence();                                                     // this block's values and sum before its count
    __syncthreads();
    if (tid == 0) {
        const int before = atomicAdd(g.counter + (size_t)seg * g.norm_groups + ng, 1);
        is_last = before == heads_per - 1;
    }
    __syncthreads();
    if (a.write_state) ss_keep_inputs(a, head, group, t, 1, slot, tid);
    if (!is_last) return;
    __threadfence();
    float total = 0.f;
    for (int h = 0; h < heads_per; ++h) total += __ldcg(g.partial + (size_t)seg * a.heads + ng * heads_per + h);
    const int part = heads_per * P;
    const float scale = 1.f / sqrtf(total / (float)part + g.eps);
    for (int c = tid; c < part; c += blockDim.x) {
        const size_t i = (size_t)t * inner + (size_t)ng * part + c;
        ss_store(g.out, a.dtype, i, __ldcg(a.y + i) * scale * g.norm_w[(size_t)ng * part + c]);
    }
    if (tid == 0) g.counter[(size_t)seg * g.norm_groups + ng] = 0;
}

// One decoded token per segment: u [segments, channels] after the convolution, proj [segments, z | x B C | dt] with row
// stride ld, gated float32 [segments, heads P] (scratch), partial float32 [segments, heads], counter int32
// [segments, norm_groups] holding zeros (and left so), out [segments, heads P] of the compute dtype.
TTB_EXPORT int ttb_state_space_token(const void* u, const void* proj, int dtype, int ld, int conv_off, int dt_off,
                                     const float* dt_bias, const float* rate, const float* skip, const int* cu_seqlens,
                                     const int* slots, float* state, void* tail, float* gated, const float* norm_w, float eps,
                                     void* out, float* partial, int* counter, int segments, int heads, int P, int N, int groups,
                                     int norm_groups, int taps, int write_state, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!u || !proj || !dt_bias || !rate || !skip || !cu_seqlens || !slots || !state || !gated || !norm_w || !out || !partial ||
        !counter || (taps > 1 && !tail))
        return TTB_ERR_ARGUMENT;
    if (dtype != TTB_DTYPE_BF16 && dtype != TTB_DTYPE_F32) return TTB_ERR_UNSUPPORTED;
    if (heads < 1 || groups < 1 || norm_groups < 1 || heads % groups || heads % norm_groups || P % 4 || P / 4 > 256 || N < 1 ||
        (uintptr_t)state % 16)
        return TTB_ERR_UNSUPPORTED;
    const int row_groups = 256 / (P / 4) < N ? 256 / (P / 4) : N;
    const size_t smem = ((size_t)((P + 2 * N + 3) & ~3) + (size_t)row_groups * P) * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    SsTokenArgs g;
    SsScanArgs& a = g.s;
    a.u = u; a.proj = proj; a.dtype = dtype; a.ld = ld; a.conv_off = conv_off; a.dt_off = dt_off;
    a.dt_bias = dt_bias; a.rate = rate; a.skip = skip; a.cu_seqlens = cu_seqlens; a.slots = slots;
    a.state = state; a.tail = tail; a.y = gated; a.part_state = nullptr; a.part_log = nullptr;
    a.heads = heads; a.P = P; a.N = N; a.groups = groups; a.channels = heads * P + 2 * groups * N; a.taps = taps;
    a.write_state = write_state; a.parts = 1; a.part_len = 1; a.NG = 1;
    g.norm_w = norm_w; g.out = out; g.partial = partial; g.counter = counter; g.eps = eps; g.norm_groups = norm_groups;
    ttb_launch(ss_token_kernel, dim3(heads, segments), 256, smem, stream, g);
    return ttb_launch_status();
}
