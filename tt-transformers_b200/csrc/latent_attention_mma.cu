// Attention over paged latents on the tensor cores (mma.sync m16n8k16, bfloat16 in, float32 sums and softmax).
//
// All heads of a token read the same cache rows [latent | extra], so a tile's 64 query rows are (token, head)
// pairs: the heads of 64 / heads tokens, or, with more than 64 heads, a group of 64 heads of one token. A block
// walks the keys of its segment in tiles of 64 that start at multiples of 64 from position 0 (the order of summation
// for a query does not depend on how its request was cut into steps): S = Q K^T over latent + extra elements,
// online softmax in float32 (base 2, the scale folded in), O += P C, where the values C are the latent part of
// the very rows that served as keys, read from the same shared-memory tile with transposing loads. The rotated
// query part is rotated by its token's position while the tile is loaded. A sink starts the running maximum and
// sum of a row at (sink, 1): one more term of the denominator without a value. Output columns are handled in
// chunks of LM_CHUNK per block; key tiles may be split over blocks (decode, few tiles), which then leave float32
// partial sums with their maxima for latent_attention_merge.
//
// Rows of the cache beyond the last visible key are never read (zeros take their place), so pages that were never
// written cannot reach a result. Tiles are derived on the device from the segment bounds: blockIdx.x counts
// (segment, tile in segment) up to the longest segment, blocks past their segment's end return at once.
#include "common.cuh"

#define LM_ROWS 64
#define LM_KEYS 64
#define LM_THREADS 128
#define LM_CHUNK_SMALL 128     // output columns per block: one chunk holds latents up to 128 columns,
#define LM_CHUNK_LARGE 256     // or up to 256 (more registers, fewer blocks an SM); wider latents take several chunks

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_u32(uint32_t (&r)[4], uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans_u32(uint32_t (&r)[4], uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 2^x in one instruction (exp2f adds range handling around it); 2^-inf = 0
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 16 bytes global -> shared without passing registers; `bytes` 0 writes zeros instead (the source is not read)
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct LatentMmaArgs {
    const __nv_bfloat16* q_lat; long long ql_stride_t, ql_stride_h;
    const __nv_bfloat16* q_rot; long long qr_stride_t, qr_stride_h;
    __nv_bfloat16* out;
    const int* cu_seqlens; const int* seg_pos0;
    const __nv_bfloat16* rows; const int* block_table; int table_width, page_size, num_pages;
    int heads, heads_per_group, tokens_per_tile, tiles_per_seg, chunks, segments;
    int latent, extra, rotary_dim;
    float scale_log2; const float* sinks; const float* inv_freq;
    int splits; float* partial_o; float* partial_ml; int* status;
    int window;      // 0: every earlier key; w: a query at position p sees the keys above p - w
    float amplitude; // what the rotation's cosines and sines are multiplied by
    int paired;      // a block takes two query tiles (one from each end of the segment) or one
    int stages;      // key tiles in shared memory at a time: 2 (the next one is fetched under the products) or 1
};

// One query tile of one segment against its share of the key tiles.
template <int LM_CHUNK>
__device__ __forceinline__ void latent_attention_tile(const LatentMmaArgs& a, int seg, int tile_in_seg) {
    extern __shared__ __align__(16) unsigned char lm_smem[];
    const int dk = a.latent + a.extra, ldq = dk + 8, vecs = dk / 8;
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(lm_smem);      // [LM_ROWS][ldq]
    __nv_bfloat16* Ks = Qs + LM_ROWS * ldq;                              // [LM_KEYS][ldq]
    const int seg_begin = a.cu_seqlens[seg], seg_len = a.cu_seqlens[seg + 1] - seg_begin;
    const int tok_off0 = tile_in_seg * a.tokens_per_tile;
    if (tok_off0 >= seg_len) return;
    const int ntok = min(a.tokens_per_tile, seg_len - tok_off0);
    const int pos0 = a.seg_pos0[seg] + tok_off0;            // position of the tile's first token
    const int hgroup = blockIdx.y / a.chunks, chunk = blockIdx.y % a.chunks;
    const int h0 = hgroup * a.heads_per_group, nh = min(a.heads_per_group, a.heads - h0);
    const int col0 = chunk * LM_CHUNK, ncols = min(LM_CHUNK, a.latent - col0);
    const int valid_rows = ntok * nh;                        // row r: token r / nh of the tile, head h0 + r % nh
    const int split = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
    const int* table = a.block_table + (size_t)seg * a.table_width;

    // ---- the query tile: latent part as it is, rotated part rotated by the token's position
    const int lat_vecs = a.latent / 8;
    for (int r = warp; r < LM_ROWS; r += LM_THREADS / 32) {
        const bool row_valid = r < valid_rows;
        const size_t tok = seg_begin + tok_off0 + (row_valid ? r / nh : 0);
        const int h = h0 + (row_valid ? r % nh : 0);
        const __nv_bfloat16* src = a.q_lat + tok * a.ql_stride_t + (size_t)h * a.ql_stride_h;
        for (int c = lane; c < lat_vecs; c += 32)
            *reinterpret_cast<uint4*>(Qs + r * ldq + c * 8) = row_valid ? *reinterpret_cast<const uint4*>(src + c * 8) : make_uint4(0, 0, 0, 0);
        if (a.extra > 0) {
            const int half = a.rotary_dim / 2;
            const __nv_bfloat16* rsrc = a.q_rot + tok * a.qr_stride_t + (size_t)h * a.qr_stride_h;
            for (int d = lane; d < a.extra; d += 32) {
                float v = 0.f;
                if (row_valid) {
                    v = __bfloat162float(rsrc[d]);
                    if (d < a.rotary_dim) {          // rotated by the token's position: pairs (i, i + rotary_dim / 2)
                        const int f = d < half ? d : d - half;
                        float sn, cs;
                        sincosf((float)(pos0 + r / nh) * a.inv_freq[f], &sn, &cs);
                        const float other = __bfloat162float(rsrc[d < half ? d + half : d - half]);
                        v = (d < half ? v * cs - other * sn : v * cs + other * sn) * a.amplitude;
                    }
                }
                Qs[r * ldq + a.latent + d] = __float2bfloat16_rn(v);
            }
        }
    }

    // ---- which key tiles are this block's
    const int last_key = pos0 + ntok - 1;
    const int first_key = (a.window > 0 && pos0 - a.window + 1 > 0) ? pos0 - a.window + 1 : 0;   // what the tile's first token sees
    const int kt_first = first_key / LM_KEYS, nk = last_key / LM_KEYS + 1 - kt_first;
    const int per = (nk + a.splits - 1) / a.splits;
    const int kt_begin = kt_first + split * per, kt_end = min(kt_first + nk, kt_begin + per);

    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const int row_pos0 = r0 < valid_rows ? pos0 + r0 / nh : -1;      // -1: no key is visible, the row is idle
    const int row_pos1 = r1 < valid_rows ? pos0 + r1 / nh : -1;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    if (a.sinks != nullptr && split == 0) {            // the sink: a term of the denominator without a value
        const float log2e = 1.4426950408889634f;
        if (r0 < valid_rows) { m0 = a.sinks[h0 + r0 % nh] * log2e; l0 = t4 == 0 ? 1.f : 0.f; }
        if (r1 < valid_rows) { m1 = a.sinks[h0 + r1 % nh] * log2e; l1 = t4 == 0 ? 1.f : 0.f; }
    }
    float o[LM_CHUNK / 8][4];
#pragma unroll
    for (int j = 0; j < LM_CHUNK / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    // one key tile into shared memory: two threads per row, each copies its half of the row in 16-byte pieces that
    // bypass the registers; rows past the last visible key (and rows of pages outside the pool) become zeros
    const int frow = tid >> 1, fhalf_off = (tid & 1) * (vecs >> 1) * 8, fvecs = vecs >> 1;
    const uint32_t qs_u32 = (uint32_t)__cvta_generic_to_shared(Qs), ks_u32 = (uint32_t)__cvta_generic_to_shared(Ks);
    auto fetch = [&](int kt, uint32_t dst_u32) {
        const int key = kt * LM_KEYS + frow;
        const __nv_bfloat16* src = a.rows;
        int bytes = 0;
        if (key <= last_key && key >= first_key) {         // pages behind the window may be somebody else's by now
            const int page = table[key / a.page_size];
            if ((unsigned)page < (unsigned)a.num_pages) {
                src = a.rows + ((size_t)page * a.page_size + key % a.page_size) * dk + fhalf_off;
                bytes = 16;
            } else {
                atomicExch(a.status, 0x2000000 + seg_begin + tok_off0);
            }
        }
        const uint32_t dst = dst_u32 + (uint32_t)(frow * ldq + fhalf_off) * 2;
        for (int c = 0; c < fvecs; ++c) {
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst + c * 16), "l"(bytes ? src + c * 8 : src), "r"(bytes) : "memory");
        }
        cp_async_commit();
    };
    const uint32_t second = a.stages == 2 ? (uint32_t)(LM_KEYS * ldq * 2) : 0u;     // byte offset of the second key buffer
    // shared-memory addresses of this lane's fragment rows, computed once
    const uint32_t q_frag = qs_u32 + (uint32_t)((warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * ldq + (lane >> 4) * 8) * 2;
    const uint32_t k_frag = (uint32_t)(((lane & 7) + (lane >> 4) * 8) * ldq + ((lane >> 3) & 1) * 8) * 2;
    const uint32_t v_frag = (uint32_t)(((lane & 7) + ((lane >> 3) & 1) * 8) * ldq + col0 + (lane >> 4) * 8) * 2;
    const uint32_t rows16 = (uint32_t)(16 * ldq * 2);
    // rows of this warp that see every key of a tile need no mask for it
    const int warp_min_pos = (warp * 16 + 16 <= valid_rows) ? pos0 + (warp * 16) / nh : -1;
    const int warp_max_pos = pos0 + (min(warp * 16 + 15, valid_rows - 1)) / nh;
    if (kt_begin < kt_end) fetch(kt_begin, ks_u32);
    for (int kt = kt_begin; kt < kt_end; ++kt) {
        const uint32_t kt_u32 = ks_u32 + ((kt - kt_begin) & 1) * second;
        if (a.stages == 2 && kt + 1 < kt_end) {
            fetch(kt + 1, ks_u32 + ((kt + 1 - kt_begin) & 1) * second);     // lands while this tile is multiplied
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                                     // the tile (and, first, the query tile) is in place
        if (warp * 16 < valid_rows) {          // a warp whose 16 rows are all idle only helps to fetch
        float s[LM_KEYS / 8][4];
#pragma unroll
        for (int j = 0; j < LM_KEYS / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
        for (int k0 = 0; k0 < dk; k0 += 16) {
            uint32_t qa[4], kb[LM_KEYS / 16][4];
            ldsm_x4_u32(qa, q_frag + k0 * 2);
#pragma unroll
            for (int jp = 0; jp < LM_KEYS / 16; ++jp) ldsm_x4_u32(kb[jp], kt_u32 + k_frag + jp * rows16 + k0 * 2);
#pragma unroll
            for (int jp = 0; jp < LM_KEYS / 16; ++jp) {
                mma_bf16(s[2 * jp], qa, kb[jp][0], kb[jp][1]);
                mma_bf16(s[2 * jp + 1], qa, kb[jp][2], kb[jp][3]);
            }
        }
        // mask (only tiles that reach past a row's position), running maximum of the raw scores
        if (kt * LM_KEYS + LM_KEYS - 1 > warp_min_pos) {
#pragma unroll
            for (int j = 0; j < LM_KEYS / 8; ++j) {
                const int key = kt * LM_KEYS + 8 * j + 2 * t4;
                if (key > row_pos0) s[j][0] = -INFINITY;
                if (key + 1 > row_pos0) s[j][1] = -INFINITY;
                if (key > row_pos1) s[j][2] = -INFINITY;
                if (key + 1 > row_pos1) s[j][3] = -INFINITY;
            }
        }
        if (a.window > 0 && kt * LM_KEYS <= warp_max_pos - a.window) {       // keys that a row's window has passed
#pragma unroll
            for (int j = 0; j < LM_KEYS / 8; ++j) {
                const int key = kt * LM_KEYS + 8 * j + 2 * t4;
                if (key <= row_pos0 - a.window) s[j][0] = -INFINITY;
                if (key + 1 <= row_pos0 - a.window) s[j][1] = -INFINITY;
                if (key <= row_pos1 - a.window) s[j][2] = -INFINITY;
                if (key + 1 <= row_pos1 - a.window) s[j][3] = -INFINITY;
            }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < LM_KEYS / 8; ++j) {
            mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
            mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // the scale (positive) goes into the exponent: p = 2^(s * scale - maximum)
        const float n0 = fmaxf(m0, mx0 * a.scale_log2), n1 = fmaxf(m1, mx1 * a.scale_log2);
        const float base0 = n0 == -INFINITY ? 0.f : n0, base1 = n1 == -INFINITY ? 0.f : n1;
        const float corr0 = fast_exp2(m0 - base0), corr1 = fast_exp2(m1 - base1);     // 2^-inf = 0
        m0 = n0;
        m1 = n1;
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int j = 0; j < LM_KEYS / 8; ++j) {
            s[j][0] = fast_exp2(fmaf(s[j][0], a.scale_log2, -base0));
            s[j][1] = fast_exp2(fmaf(s[j][1], a.scale_log2, -base0));
            s[j][2] = fast_exp2(fmaf(s[j][2], a.scale_log2, -base1));
            s[j][3] = fast_exp2(fmaf(s[j][3], a.scale_log2, -base1));
            sum0 += s[j][0] + s[j][1];
            sum1 += s[j][2] + s[j][3];
        }
        l0 = l0 * corr0 + sum0;
        l1 = l1 * corr1 + sum1;
        if (__any_sync(0xffffffffu, corr0 != 1.f || corr1 != 1.f)) {       // the maximum moved somewhere in the warp
#pragma unroll
            for (int j = 0; j < LM_CHUNK / 8; ++j) {
                o[j][0] *= corr0; o[j][1] *= corr0; o[j][2] *= corr1; o[j][3] *= corr1;
            }
        }
        // O += P C: the values are the latent part of the key rows
#pragma unroll
        for (int kk = 0; kk < LM_KEYS / 16; ++kk) {
            uint32_t pa[4];
            pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
            pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
            pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int np0 = 0; np0 < LM_CHUNK / 16; np0 += 4) {          // four loads in flight, then their eight products
                if (np0 * 16 < ncols) {
                    uint32_t vb[4][4];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if ((np0 + i) * 16 < ncols) ldsm_x4_trans_u32(vb[i], kt_u32 + v_frag + kk * rows16 + (np0 + i) * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if ((np0 + i) * 16 < ncols) {
                            mma_bf16(o[2 * (np0 + i)], pa, vb[i][0], vb[i][1]);
                            mma_bf16(o[2 * (np0 + i) + 1], pa, vb[i][2], vb[i][3]);
                        }
                }
            }
        }
        }
        __syncthreads();                                     // all warps are done with this tile: it may be overwritten
        if (a.stages == 1 && kt + 1 < kt_end) fetch(kt + 1, ks_u32);
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
#pragma unroll
    for (int half_row = 0; half_row < 2; ++half_row) {
        const int r = half_row ? r1 : r0;
        if (r >= valid_rows) continue;
        const float m = half_row ? m1 : m0, l = half_row ? l1 : l0;
        const size_t row = (size_t)(seg_begin + tok_off0 + r / nh) * a.heads + h0 + r % nh;
        if (a.splits == 1) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16* dst = a.out + row * a.latent + col0;
#pragma unroll
            for (int j = 0; j < LM_CHUNK / 8; ++j)
                if (j * 8 < ncols)
                    *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * t4) = pack_bf16(o[j][2 * half_row] * inv, o[j][2 * half_row + 1] * inv);
        } else {
            float* dst = a.partial_o + (row * a.splits + split) * a.latent + col0;
#pragma unroll
            for (int j = 0; j < LM_CHUNK / 8; ++j)
                if (j * 8 < ncols)
                    *reinterpret_cast<float2*>(dst + j * 8 + 2 * t4) = make_float2(o[j][2 * half_row], o[j][2 * half_row + 1]);
            if (chunk == 0 && t4 == 0) {
                a.partial_ml[(row * a.splits + split) * 2] = m;
                a.partial_ml[(row * a.splits + split) * 2 + 1] = l;
            }
        }
    }
}

// A block takes a query tile from the end of its segment (many keys) and then its partner from the start (few), so
// that all blocks of a long prompt portion walk about the same number of key tiles.
template <int LM_CHUNK>
__global__ void __launch_bounds__(LM_THREADS)
latent_attention_mma_kernel(const LatentMmaArgs a) {
    pdl_wait();
    const int seg = blockIdx.x % a.segments, b = blockIdx.x / a.segments;
    const int first = a.tiles_per_seg - 1 - b, second = a.paired ? b : first;
    latent_attention_tile<LM_CHUNK>(a, seg, first);
    if (second != first) {
        __syncthreads();                      // the first tile's queries are no longer read
        latent_attention_tile<LM_CHUNK>(a, seg, second);
    }
    pdl_launch_dependents();
}

// out[row, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s, splits in their order.
__global__ void latent_attention_merge_kernel(const float* __restrict__ partial_o, const float* __restrict__ partial_ml,
                                              __nv_bfloat16* __restrict__ out, int splits, int latent) {
    __shared__ float wt[64];                  // 2^(m_s - M) / denominator, per split (at most 64 splits)
    pdl_wait();
    pdl_launch_dependents();
    const size_t row = blockIdx.x;
    if (threadIdx.x < 32) {
        const float2* ml = reinterpret_cast<const float2*>(partial_ml) + row * splits;
        const int lane = threadIdx.x;
        const float2 a = lane < splits ? ml[lane] : make_float2(-INFINITY, 0.f);
        const float2 b = lane + 32 < splits ? ml[lane + 32] : make_float2(-INFINITY, 0.f);
        const float M = warp_max(fmaxf(a.x, b.x));
        const float wa = a.x == -INFINITY ? 0.f : exp2f(a.x - M), wb = b.x == -INFINITY ? 0.f : exp2f(b.x - M);
        // the denominator in the order of the splits (one lane adds them up), so that it does not depend on the lanes' tree
        wt[lane] = wa * a.y;
        wt[lane + 32] = wb * b.y;
        __syncwarp();
        float denom = 0.f;
        for (int s = 0; s < splits; ++s) denom += wt[s];
        const float inv = denom > 0.f ? 1.f / denom : 0.f;
        __syncwarp();
        wt[lane] = wa * inv;
        wt[lane + 32] = wb * inv;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < latent; c += blockDim.x) {
        const float* src = partial_o + row * splits * latent + c;
        float acc = 0.f;
#pragma unroll 8
        for (int s = 0; s < splits; ++s) acc = fmaf(wt[s], src[(size_t)s * latent], acc);
        out[row * latent + c] = __float2bfloat16_rn(acc);
    }
}

static int tc_like_sm_count() {
    int device = 0, count = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
    return count > 0 ? count : 1;
}

TTB_EXPORT int ttb_latent_attention_mma_supports(int latent, int extra, int rotary_dim, int window) {
    if (latent < 16 || (latent & 15) || (extra & 15) || extra < 0 || window < 0) return 0;
    if (rotary_dim > extra || (rotary_dim & 1)) return 0;
    const size_t smem = (size_t)(LM_ROWS + LM_KEYS) * (latent + extra + 8) * 2;
    return smem <= 220 * 1024;
}

// Tokens whose heads share a tile, for the caller's split heuristics.
TTB_EXPORT int ttb_latent_attention_mma_tokens_per_tile(int heads) {
    const int hg = heads < LM_ROWS ? heads : LM_ROWS;
    return LM_ROWS / hg > 0 ? LM_ROWS / hg : 1;
}

// q_lat [tokens, heads, latent] and q_rot [tokens, heads, extra] with element strides (token, head, 1), 16-byte
// aligned rows; out [tokens, heads, latent] contiguous; rows [num_pages, page_size, latent + extra]. With
// splits > 1: partial_o tokens * heads * splits * latent floats, partial_ml tokens * heads * splits * 2 floats.
TTB_EXPORT int ttb_latent_attention_mma_ext(const void* q_lat, long long ql_stride_t, long long ql_stride_h, const void* q_rot,
                                        long long qr_stride_t, long long qr_stride_h, void* out, const int* cu_seqlens,
                                        const int* seg_pos0, const void* rows, const int* block_table, int table_width,
                                        int page_size, int num_pages, int segments, int max_seg_len, int tokens, int heads,
                                        int latent, int extra, float scale, const float* sinks, const float* inv_freq,
                                        int rotary_dim, int splits, float* partial_o, float* partial_ml, int merge,
                                        int* status, int window, float amplitude, cudaStream_t stream) {
    if (tokens == 0 || segments == 0) return TTB_OK;
    if (!q_lat || !out || !cu_seqlens || !seg_pos0 || !rows || !block_table || !status) return TTB_ERR_ARGUMENT;
    if (!ttb_latent_attention_mma_supports(latent, extra, rotary_dim, window) || !(scale > 0.f)) return TTB_ERR_UNSUPPORTED;
    if (extra > 0 && (!q_rot || (rotary_dim > 0 && !inv_freq))) return TTB_ERR_ARGUMENT;
    if ((ql_stride_t & 7) || (ql_stride_h & 7) || !aligned16(q_lat) || !aligned16(rows) || !aligned16(out)) return TTB_ERR_ARGUMENT;
    if (splits < 1 || splits > 64 || (splits > 1 && (!partial_o || !partial_ml))) return TTB_ERR_ARGUMENT;
    LatentMmaArgs a;
    a.q_lat = (const __nv_bfloat16*)q_lat; a.ql_stride_t = ql_stride_t; a.ql_stride_h = ql_stride_h;
    a.q_rot = (const __nv_bfloat16*)q_rot; a.qr_stride_t = qr_stride_t; a.qr_stride_h = qr_stride_h;
    a.out = (__nv_bfloat16*)out; a.cu_seqlens = cu_seqlens; a.seg_pos0 = seg_pos0;
    a.rows = (const __nv_bfloat16*)rows; a.block_table = block_table; a.table_width = table_width;
    a.page_size = page_size; a.num_pages = num_pages; a.heads = heads;
    a.heads_per_group = heads < LM_ROWS ? heads : LM_ROWS;
    a.tokens_per_tile = ttb_latent_attention_mma_tokens_per_tile(heads);
    a.tiles_per_seg = (max_seg_len + a.tokens_per_tile - 1) / a.tokens_per_tile;
    const int chunk_cols = latent > LM_CHUNK_SMALL ? LM_CHUNK_LARGE : LM_CHUNK_SMALL;
    a.chunks = (latent + chunk_cols - 1) / chunk_cols;
    a.segments = segments;
    a.latent = latent; a.extra = extra; a.rotary_dim = rotary_dim;
    a.scale_log2 = scale * 1.4426950408889634f; a.sinks = sinks; a.inv_freq = inv_freq;
    a.splits = splits; a.partial_o = partial_o; a.partial_ml = partial_ml; a.status = status;
    a.window = window; a.amplitude = amplitude;
    // with blocks in plenty a block takes a long tile and its short partner (even work); else one tile, longest first
    a.paired = (long long)segments * a.tiles_per_seg >= 16LL * tc_like_sm_count();
    const long long blocks_x = (long long)segments * (a.paired ? (a.tiles_per_seg + 1) / 2 : a.tiles_per_seg);
    const int groups = (heads + a.heads_per_group - 1) / a.heads_per_group;
    if (blocks_x > 2147483647LL || groups * a.chunks > 65535) return TTB_ERR_UNSUPPORTED;
    const size_t tile_bytes = (size_t)LM_KEYS * (latent + extra + 8) * 2;
    a.stages = 3 * tile_bytes <= 96 * 1024 ? 2 : 1;         // two key tiles only while several blocks still fit an SM
    const size_t smem = (size_t)(1 + a.stages) * tile_bytes;
    static TtbOncePerDevice once;
    if (once.pending()) {
        cudaFuncSetAttribute(latent_attention_mma_kernel<LM_CHUNK_SMALL>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        cudaFuncSetAttribute(latent_attention_mma_kernel<LM_CHUNK_LARGE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        once.mark();
    }
    if (chunk_cols == LM_CHUNK_SMALL)
        ttb_launch(latent_attention_mma_kernel<LM_CHUNK_SMALL>, dim3((unsigned)blocks_x, groups * a.chunks, splits), LM_THREADS, smem, stream, a);
    else
        ttb_launch(latent_attention_mma_kernel<LM_CHUNK_LARGE>, dim3((unsigned)blocks_x, groups * a.chunks, splits), LM_THREADS, smem, stream, a);
    int rc = ttb_launch_status();
    if (rc != TTB_OK || splits == 1 || !merge) return rc;      // merge 0: the caller's next kernel takes the partial sums
    ttb_launch(latent_attention_merge_kernel, tokens * heads, 128, 0, stream, (const float*)partial_o,
               (const float*)partial_ml, (__nv_bfloat16*)out, splits, latent);
    return ttb_launch_status();
}

TTB_EXPORT int ttb_latent_attention_mma(const void* q_lat, long long ql_stride_t, long long ql_stride_h, const void* q_rot,
                                        long long qr_stride_t, long long qr_stride_h, void* out, const int* cu_seqlens,
                                        const int* seg_pos0, const void* rows, const int* block_table, int table_width,
                                        int page_size, int num_pages, int segments, int max_seg_len, int tokens, int heads,
                                        int latent, int extra, float scale, const float* sinks, const float* inv_freq,
                                        int rotary_dim, int splits, float* partial_o, float* partial_ml, int merge,
                                        int* status, cudaStream_t stream) {
    return ttb_latent_attention_mma_ext(q_lat, ql_stride_t, ql_stride_h, q_rot, qr_stride_t, qr_stride_h, out, cu_seqlens, seg_pos0,
                                        rows, block_table, table_width, page_size, num_pages, segments, max_seg_len, tokens, heads,
                                        latent, extra, scale, sinks, inv_freq, rotary_dim, splits, partial_o, partial_ml, merge,
                                        status, 0, 1.f, stream);
}
