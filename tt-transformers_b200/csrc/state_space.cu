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
    if (quads)
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
__global__ void __launch_bounds__(128)
ss_gate_norm_kernel(const float* __restrict__ y, const void* __restrict__ z, int z_dtype, int z_stride,
                    const float* __restrict__ weight, float eps, void* __restrict__ out, int out_dtype, int inner, int part) {
    __shared__ float scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, c0 = blockIdx.y * part;
    float sumsq = 0.f;
    for (int c = threadIdx.x; c < part; c += blockDim.x) {
        const float v = y[(size_t)t * inner + c0 + c] * ss_silu(ss_load(z, z_dtype, (size_t)t * z_stride + c0 + c));
        sumsq += v * v;
    }
    sumsq = block_sum(sumsq, scratch);
    const float scale = 1.f / sqrtf(sumsq / (float)part + eps);
    for (int c = threadIdx.x; c < part; c += blockDim.x) {
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
