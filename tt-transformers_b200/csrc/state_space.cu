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
    // the convolution's new kept inputs, for the channels this head owns: its x columns, and B and C of its group if it
    // is the group's first head. A thread per channel walks the kept rows oldest first, so a short segment shifts the old
    // rows down before it overwrites them.
    const int keep = a.taps - 1;
    if (keep <= 0) return;
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
        for (int k = 0; k + 1 < parts_here; ++k) {
            s = fmaf(expf(pl[k]), s, ps[(size_t)k * elems + i]);
            ps[(size_t)k * elems + i] = s;
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

// How the state of one head is dealt out: rows per thread (R, a power of two up to 32) and row groups (NG).
static bool ss_plan(int P, int N, int& pc, int& r, int& ng) {
    pc = (P % 4 == 0) ? 4 : 1;
    const int cols = P / pc;
    for (r = 1; r <= 32; r *= 2) {
        ng = (N + r - 1) / r;
        const int threads = cols * ng;
        if (threads <= 256 || (r == 32 && pc == 1 && threads <= 1024)) return true;
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
    const size_t total = (size_t)tokens * channels;
    const int blocks = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    ttb_launch(ss_conv_silu_kernel, blocks, 256, 0, stream, in, dtype, ld, conv_w, conv_b, seg_of_token, cu_seqlens, slots, tail,
               out, tokens, channels, taps);
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
    if (parts > 1) {
        SS_PICK(true);
        const int elems = N * P;
        dim3 grid(heads, segments, (elems + 1023) / 1024);
        ttb_launch(ss_prefix_kernel, grid, 256, 0, stream, (const float*)state, cu_seqlens, slots, part_state,
                   (const float*)part_log, heads, elems, parts, part_len);
    }
    SS_PICK(false);
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
