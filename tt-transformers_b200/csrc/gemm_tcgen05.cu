// C[M, N] = A[M, K] * W[N, K]^T for prefill on the fifth-generation tensor cores (sm_100a):
// operands move from global to shared memory by TMA (cp.async.bulk.tensor, 128-byte swizzle),
// one elected thread issues tcgen05.mma on shared-memory descriptors, the float32 accumulator
// lives in tensor memory (TMEM) and comes back to registers with tcgen05.ld for the epilogue.
//
// Persistent: one block per SM walks over tiles of 128 rows x 256 accumulator columns. Six warps:
//   warp 0      producer: waits for a free stage, arms its mbarrier with the bytes to come, issues the TMA loads
//   warp 1      allocates TMEM (two accumulators of 256 columns); one thread issues the MMAs of each stage
//               (four k-steps of 16, N = 256) and commits them to the stage's "empty" barrier; after a tile's
//               last stage it commits to that accumulator's "full" barrier and goes on with the other one
//   warps 2-5   epilogue: each reads its quarter of the TMEM lanes (a warp may only touch lanes
//               32 * (warp % 4) ..), converts and stores rows of C, then releases the accumulator;
//               it runs under the products of the next tile
// SWIGLU: W holds `up_offset` gate rows followed by as many up rows; a stage holds 128 gate rows and
// their 128 up rows as one 256-row operand, and the epilogue writes silu(gate) * up, so the product's
// intermediate never goes to memory.
//
// No load uses cluster multicast. Every wait on an mbarrier is bounded: after WAIT_LIMIT polls
// the waiting role records an error code in *error_flag and stops; the block then frees its TMEM
// and returns (by then every role has either finished or run out of patience, and no copy of its
// own is in flight). Sizes: any M and N; K a multiple of 8 and row strides of 16 bytes (TMA).
#include <cuda.h>

#include <type_traits>

#include "common.cuh"

#define TC_BM 128
#define TC_BK 64
#define TC_THREADS 192
#define TC_WAIT_LIMIT (1u << 20)

#define TC_ERR_PRODUCER 1
#define TC_ERR_MMA 2
#define TC_ERR_EPILOGUE 3

__device__ __forceinline__ uint32_t tc_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Polls until the barrier's phase `parity` has completed; false after TC_WAIT_LIMIT polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < TC_WAIT_LIMIT; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_c, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_c), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory operand descriptor: K-major tile of rows x 64 bfloat16 as TMA lays it out with the
// 128-byte swizzle; groups of eight rows are 1,024 bytes apart. `addr` is the shared address of
// the first element of the k-step (the tile base plus 32 bytes per k-step of 16).
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);          // start address, 16-byte units
    d |= (uint64_t)0 << 16;                          // leading-dimension offset: not used by swizzled K-major tiles
    d |= (uint64_t)(1024 >> 4) << 32;                // stride between groups of eight rows
    d |= (uint64_t)1 << 46;                          // descriptor version of this architecture
    d |= (uint64_t)2 << 61;                          // 128-byte swizzle
    return d;
}

// 16 bytes of output from consecutive float values.
template <typename TO> __device__ __forceinline__ uint4 pack_chunk(const float* v);
template <> __device__ __forceinline__ uint4 pack_chunk<float>(const float* v) {
    return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
}
template <> __device__ __forceinline__ uint4 pack_chunk<__nv_bfloat16>(const float* v) {
    uint4 r;
    __nv_bfloat162 p;
    p = __floats2bfloat162_rn(v[0], v[1]); r.x = *reinterpret_cast<uint32_t*>(&p);
    p = __floats2bfloat162_rn(v[2], v[3]); r.y = *reinterpret_cast<uint32_t*>(&p);
    p = __floats2bfloat162_rn(v[4], v[5]); r.z = *reinterpret_cast<uint32_t*>(&p);
    p = __floats2bfloat162_rn(v[6], v[7]); r.w = *reinterpret_cast<uint32_t*>(&p);
    return r;
}

// Geometry of one block: it walks over output tiles of 128 rows x TC_BN_ACC accumulator columns.
// Plain product: 256 columns of C. SWIGLU: 128 gate columns and their 128 up columns (the two W row
// tiles lie back to back in the stage and form one 256-row operand), giving 128 columns of output.
struct TcCfg {
    static constexpr int STAGES = 4;
    static constexpr int ACC_COLS = 256;                       // accumulator columns per tile = MMA N
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;          // 16 KB
    static constexpr int B_BYTES = ACC_COLS * TC_BK * 2;       // 32 KB
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * ACC_COLS;             // two accumulators: the epilogue of a tile runs under the next tile's products
    static constexpr int STAGING_BYTES = 4 * 32 * 128;         // the epilogue's transposition buffers: 32 rows x 128 bytes per warp
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /* alignment slack */ + 256 /* barriers */;
};

template <bool SWIGLU, typename TO>
__global__ void __launch_bounds__(TC_THREADS)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                    TO* __restrict__ out, int M, int N, int K, int ldc, int up_offset, int m_tiles, int n_tiles,
                    int* __restrict__ error_flag) {
    using Cfg = TcCfg;
    constexpr int OUT_COLS = SWIGLU ? Cfg::ACC_COLS / 2 : Cfg::ACC_COLS;      // columns of C per tile
    extern __shared__ unsigned char tc_raw[];
    unsigned char* tiles = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* staging = tiles + Cfg::STAGES * Cfg::STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + Cfg::STAGING_BYTES);
    // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * Cfg::STAGES + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k_blocks = (K + TC_BK - 1) / TC_BK;
    const int num_tiles = m_tiles * n_tiles;
    const uint32_t full0 = tc_smem(bars), empty0 = tc_smem(bars + Cfg::STAGES);
    const uint32_t acc_full0 = tc_smem(bars + 2 * Cfg::STAGES), acc_empty0 = tc_smem(bars + 2 * Cfg::STAGES + 2);

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(acc_full0 + 8 * a, 1);
            mbar_init(acc_empty0 + 8 * a, 4);          // one arrival per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tc_smem(tmem_slot)), "r"((uint32_t)Cfg::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();                       // A is the output of the kernel before this one

    // Tiles go round the blocks; consecutive tiles share the W column block (m runs fastest), so the
    // blocks that run side by side read the same weights from L2.
    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;                      // k-blocks loaded so far, over all tiles
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int m0 = (tile % m_tiles) * TC_BM, n0 = (tile / m_tiles) * OUT_COLS;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    const uint32_t round = it / Cfg::STAGES;
                    if (round > 0 && !mbar_wait(empty0 + 8 * s, (round - 1) & 1)) {
                        atomicExch(error_flag, TC_ERR_PRODUCER);
                        tile = num_tiles;
                        break;
                    }
                    const uint32_t bar = full0 + 8 * s;
                    mbar_expect_tx(bar, Cfg::STAGE_BYTES);
                    unsigned char* stage = tiles + s * Cfg::STAGE_BYTES;
                    tma_load_2d(tc_smem(stage), &map_a, kb * TC_BK, m0, bar);
                    if (SWIGLU) {
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES), &map_w, kb * TC_BK, n0, bar);
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES + Cfg::B_BYTES / 2), &map_w, kb * TC_BK, up_offset + n0, bar);
                    } else {
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES), &map_w, kb * TC_BK, n0, bar);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // instruction descriptor: float32 accumulator, bfloat16 operands, both K-major, M = 128, N = 256
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Cfg::ACC_COLS >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
            uint32_t it = 0;
            int local = 0;                        // tiles this block has started
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                if (local >= 2 && !mbar_wait(acc_empty0 + 8 * acc, ((local >> 1) - 1) & 1)) {
                    atomicExch(error_flag, TC_ERR_MMA);
                    break;
                }
                tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    if (!mbar_wait(full0 + 8 * s, (it / Cfg::STAGES) & 1)) {
                        atomicExch(error_flag, TC_ERR_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = tc_smem(tiles + s * Cfg::STAGE_BYTES);
                    const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; ++k)
                        tc_mma(tmem_base + acc * Cfg::ACC_COLS, tc_smem_desc(a_addr + k * 32), tc_smem_desc(b_addr + k * 32),
                               idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    tc_commit(empty0 + 8 * s);         // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                tc_commit(acc_full0 + 8 * acc);
            }
        }
    } else {
        // epilogue: TMEM lane quarter of this warp. A thread holds one row of the accumulator, so
        // storing from registers would write 16 bytes to each of 32 rows per instruction. Instead the
        // warp passes 32 rows x 128 bytes through shared memory (16-byte chunks swizzled by row, free
        // of bank conflicts both ways) and stores whole 128-byte lines, four rows per instruction.
        const int quarter = warp & 3;
        constexpr int CHUNK_ELEMS = 16 / (int)sizeof(TO);            // elements in 16 bytes
        constexpr int LINE_COLS = 8 * CHUNK_ELEMS;                   // columns in 128 bytes of output
        const bool vec = (ldc % CHUNK_ELEMS == 0) && (N % CHUNK_ELEMS == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
        uint4* stage_rows = reinterpret_cast<uint4*>(staging + quarter * 4096);
        int local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const int m0 = (tile % m_tiles) * TC_BM, n0 = (tile / m_tiles) * OUT_COLS;
            const int row0 = m0 + quarter * 32;
            if (tile + (int)gridDim.x >= num_tiles) pdl_launch_dependents();      // this block's last tile
            if (!mbar_wait(acc_full0 + 8 * acc, (local >> 1) & 1)) {
                if (lane == 0) atomicExch(error_flag, TC_ERR_EPILOGUE);
                break;
            }
            tc_fence_after();
            const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_COLS;
#pragma unroll 1
            for (int c0 = 0; c0 < OUT_COLS; c0 += LINE_COLS) {
#pragma unroll
                for (int h = 0; h < LINE_COLS / 32; ++h) {
                    uint32_t accv[32];
                    tc_load32(lane_addr + c0 + h * 32, accv);
                    float v[32];
                    if (SWIGLU) {
                        uint32_t up[32];
                        tc_load32(lane_addr + OUT_COLS + c0 + h * 32, up);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float g = __uint_as_float(accv[j]);
                            v[j] = __fdividef(g, 1.f + __expf(-g)) * __uint_as_float(up[j]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(accv[j]);
                    }
                    if (vec) {
#pragma unroll
                        for (int q = 0; q < 32 / CHUNK_ELEMS; ++q) {
                            const int chunk = h * (32 / CHUNK_ELEMS) + q;
                            stage_rows[lane * 8 + (chunk ^ (lane & 7))] = pack_chunk<TO>(v + q * CHUNK_ELEMS);
                        }
                    } else if (row0 + lane < M) {
                        TO* dst = out + (size_t)(row0 + lane) * ldc + n0 + c0 + h * 32;
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + h * 32 + j < N) dst[j] = from_float<TO>(v[j]);
                    }
                }
                if (vec) {
                    __syncwarp();
                    const int chunk = lane & 7, col = n0 + c0 + chunk * CHUNK_ELEMS;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = i * 4 + (lane >> 3);
                        const uint4 value = stage_rows[r * 8 + (chunk ^ (r & 7))];
                        if (row0 + r < M && col < N)
                            *reinterpret_cast<uint4*>(out + (size_t)(row0 + r) * ldc + col) = value;
                    }
                    __syncwarp();
                }
            }
            // the accumulator has been read: the products of the tile after next may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acc_empty0 + 8 * acc) : "memory");
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)Cfg::TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*TcEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                               const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static TcEncodeFn tc_encode_fn() {
    static TcEncodeFn fn = nullptr;
    static bool looked = false;
    if (!looked) {
        looked = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TcEncodeFn>(p);
    }
    return fn;
}

// A row-major [rows, cols] bfloat16 matrix with row stride ld (elements), fetched in boxes of box_rows x 64.
static bool tc_make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
    TcEncodeFn encode = tc_encode_fn();
    if (!encode) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {TC_BK, (cuuint32_t)box_rows};
    cuuint32_t elem[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int tc_sm_count() {
    static int count = 0;
    if (count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        if (count <= 0) count = 1;
    }
    return count;
}

template <bool SWIGLU, typename TO>
static int tc_launch(const CUtensorMap& map_a, const CUtensorMap& map_w, void* C, int M, int N, int K, int ldc,
                     int up_offset, int* error_flag, cudaStream_t stream) {
    auto kernel = gemm_tcgen05_kernel<SWIGLU, TO>;
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg::SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    constexpr int out_cols = SWIGLU ? TcCfg::ACC_COLS / 2 : TcCfg::ACC_COLS;
    const int m_tiles = (M + TC_BM - 1) / TC_BM, n_tiles = (N + out_cols - 1) / out_cols;
    const int blocks = m_tiles * n_tiles < tc_sm_count() ? m_tiles * n_tiles : tc_sm_count();
    ttb_launch(kernel, dim3(blocks), dim3(TC_THREADS), (size_t)TcCfg::SMEM_BYTES, stream, map_a, map_w, (TO*)C, M, N, K,
               ldc, up_offset, m_tiles, n_tiles, error_flag);
    return ttb_launch_status();
}

// A [M, K], W [N, K] (or [2 * swiglu_rows, K] with swiglu_rows = N gate rows then N up rows), bfloat16, K-contiguous.
// C [M, N] bfloat16 or float32. error_flag: device int that a timed-out wait sets (0 = fine).
TTB_EXPORT int ttb_gemm_tcgen05(const void* A, const void* W, void* C, int out_dtype, int M, int N, int K, int lda,
                                int ldw, int ldc, int swiglu_rows, int* error_flag, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!A || !W || !C || !error_flag) return TTB_ERR_ARGUMENT;
    if (K < 8 || (K & 7) || (lda & 7) || (ldw & 7) || !aligned16(A) || !aligned16(W)) return TTB_ERR_UNSUPPORTED;
    if ((M + TC_BM - 1) / TC_BM > 65535) return TTB_ERR_UNSUPPORTED;
    if (swiglu_rows != 0 && swiglu_rows != N) return TTB_ERR_ARGUMENT;
    CUtensorMap map_a, map_w;
    if (!tc_make_map(&map_a, A, M, K, lda, TC_BM)) return TTB_ERR_UNSUPPORTED;
    if (!tc_make_map(&map_w, W, swiglu_rows ? 2 * N : N, K, ldw, swiglu_rows ? TcCfg::ACC_COLS / 2 : TcCfg::ACC_COLS)) return TTB_ERR_UNSUPPORTED;
    const bool f32 = out_dtype == TTB_DTYPE_F32;
    if (!f32 && out_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    if (swiglu_rows)
        return f32 ? tc_launch<true, float>(map_a, map_w, C, M, N, K, ldc, swiglu_rows, error_flag, stream)
                   : tc_launch<true, __nv_bfloat16>(map_a, map_w, C, M, N, K, ldc, swiglu_rows, error_flag, stream);
    return f32 ? tc_launch<false, float>(map_a, map_w, C, M, N, K, ldc, 0, error_flag, stream)
               : tc_launch<false, __nv_bfloat16>(map_a, map_w, C, M, N, K, ldc, 0, error_flag, stream);
}

// ---------------------------------------------------------------------------- the same product over groups of rows
// Routed experts: the rows of A lie expert by expert (offsets[e] .. offsets[e + 1]), expert e multiplies by its own
// W_e (rows e * rows_per_expert .. of one stacked matrix). The grouping kernel leaves a table of row tiles
// (expert, first row) and their count on the device, so no size is read back by the host; the grid is sized for the
// most tiles there can be. A tile's box of 128 rows may reach into the next expert's rows: those rows are computed
// and not stored. MODE 1: W_e = [gate rows; up rows], the epilogue writes g' sigmoid(alpha g') (u' + 1) with
// g' = min(g, L), u' = clamp(u, -L, L) into the hidden rows (grouped order). MODE 2: W_e = [rows] without a gate, the
// epilogue writes relu(z)^2 into the hidden rows. MODE 0: float32 results go to the row that `sorted` names for each
// grouped row (the pair's own row).
template <int MODE>
__global__ void __launch_bounds__(TC_THREADS)
moe_gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                        void* __restrict__ out_raw, const int* __restrict__ offsets, const int* __restrict__ sorted,
                        const int* __restrict__ tile_info, const int* __restrict__ num_m_tiles, int N, int K, int ldc,
                        int rows_per_expert, int n_tiles, float limit, float alpha, int* __restrict__ error_flag) {
    using Cfg = TcCfg;
    using TO = typename std::conditional<MODE != 0, __nv_bfloat16, float>::type;
    constexpr int OUT_COLS = MODE == 1 ? Cfg::ACC_COLS / 2 : Cfg::ACC_COLS;
    TO* out = reinterpret_cast<TO*>(out_raw);
    extern __shared__ unsigned char tc_raw[];
    unsigned char* tiles = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* staging = tiles + Cfg::STAGES * Cfg::STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + Cfg::STAGING_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * Cfg::STAGES + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k_blocks = (K + TC_BK - 1) / TC_BK;
    const uint32_t full0 = tc_smem(bars), empty0 = tc_smem(bars + Cfg::STAGES);
    const uint32_t acc_full0 = tc_smem(bars + 2 * Cfg::STAGES), acc_empty0 = tc_smem(bars + 2 * Cfg::STAGES + 2);

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::STAGES; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(acc_full0 + 8 * a, 1);
            mbar_init(acc_empty0 + 8 * a, 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(tc_smem(tmem_slot)), "r"((uint32_t)Cfg::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();                       // A, the tile table and its count come from kernels before this one
    const int m_tiles = *num_m_tiles;
    const int num_tiles = m_tiles * n_tiles;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int mt = tile % m_tiles, n0 = (tile / m_tiles) * OUT_COLS;
                const int expert = tile_info[2 * mt], row0 = tile_info[2 * mt + 1];
                const int w_row = expert * rows_per_expert + n0;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    const uint32_t round = it / Cfg::STAGES;
                    if (round > 0 && !mbar_wait(empty0 + 8 * s, (round - 1) & 1)) {
                        atomicExch(error_flag, TC_ERR_PRODUCER);
                        tile = num_tiles;
                        break;
                    }
                    const uint32_t bar = full0 + 8 * s;
                    mbar_expect_tx(bar, Cfg::STAGE_BYTES);
                    unsigned char* stage = tiles + s * Cfg::STAGE_BYTES;
                    tma_load_2d(tc_smem(stage), &map_a, kb * TC_BK, row0, bar);
                    if (MODE == 1) {
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES), &map_w, kb * TC_BK, w_row, bar);
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES + Cfg::B_BYTES / 2), &map_w, kb * TC_BK, w_row + N, bar);
                    } else {
                        tma_load_2d(tc_smem(stage + Cfg::A_BYTES), &map_w, kb * TC_BK, w_row, bar);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Cfg::ACC_COLS >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
            uint32_t it = 0;
            int local = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                if (local >= 2 && !mbar_wait(acc_empty0 + 8 * acc, ((local >> 1) - 1) & 1)) {
                    atomicExch(error_flag, TC_ERR_MMA);
                    break;
                }
                tc_fence_after();
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb, ++it) {
                    const int s = it % Cfg::STAGES;
                    if (!mbar_wait(full0 + 8 * s, (it / Cfg::STAGES) & 1)) {
                        atomicExch(error_flag, TC_ERR_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = tc_smem(tiles + s * Cfg::STAGE_BYTES);
                    const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; ++k)
                        tc_mma(tmem_base + acc * Cfg::ACC_COLS, tc_smem_desc(a_addr + k * 32), tc_smem_desc(b_addr + k * 32),
                               idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    tc_commit(empty0 + 8 * s);
                }
                if (!ok) break;
                tc_commit(acc_full0 + 8 * acc);
            }
        }
    } else {
        const int quarter = warp & 3;
        constexpr int CHUNK_ELEMS = 16 / (int)sizeof(TO);
        constexpr int LINE_COLS = 8 * CHUNK_ELEMS;
        const bool vec = (ldc % CHUNK_ELEMS == 0) && (N % CHUNK_ELEMS == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
        uint4* stage_rows = reinterpret_cast<uint4*>(staging + quarter * 4096);
        int local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const int mt = tile % m_tiles, n0 = (tile / m_tiles) * OUT_COLS;
            const int expert = tile_info[2 * mt];
            const int row0 = tile_info[2 * mt + 1] + quarter * 32, row_end = offsets[expert + 1];
            if (tile + (int)gridDim.x >= num_tiles) pdl_launch_dependents();
            if (!mbar_wait(acc_full0 + 8 * acc, (local >> 1) & 1)) {
                if (lane == 0) atomicExch(error_flag, TC_ERR_EPILOGUE);
                break;
            }
            tc_fence_after();
            // where this lane's row goes: the hidden rows keep the grouped order, results go to the pair's own row
            const long long my_dst = row0 + lane < row_end ? (MODE != 0 ? (long long)(row0 + lane) : (long long)sorted[row0 + lane]) : -1;
            const uint32_t lane_addr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_COLS;
#pragma unroll 1
            for (int c0 = 0; c0 < OUT_COLS; c0 += LINE_COLS) {
#pragma unroll
                for (int h = 0; h < LINE_COLS / 32; ++h) {
                    uint32_t accv[32];
                    tc_load32(lane_addr + c0 + h * 32, accv);
                    float v[32];
                    if (MODE == 1) {
                        uint32_t up[32];
                        tc_load32(lane_addr + OUT_COLS + c0 + h * 32, up);
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (!(limit > 0.f)) {        // no clamps, no unit offset: g sigmoid(alpha g) u
                                const float g = __uint_as_float(accv[j]);
                                v[j] = __fdividef(g, 1.f + __expf(-alpha * g)) * __uint_as_float(up[j]);
                                continue;
                            }
                            const float g = fminf(__uint_as_float(accv[j]), limit);
                            const float u = fminf(fmaxf(__uint_as_float(up[j]), -limit), limit);
                            v[j] = __fdividef(g, 1.f + __expf(-alpha * g)) * (u + 1.f);
                        }
                    } else if (MODE == 2) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float z = fmaxf(__uint_as_float(accv[j]), 0.f);
                            v[j] = z * z;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(accv[j]);
                    }
                    if (vec) {
#pragma unroll
                        for (int q = 0; q < 32 / CHUNK_ELEMS; ++q) {
                            const int chunk = h * (32 / CHUNK_ELEMS) + q;
                            stage_rows[lane * 8 + (chunk ^ (lane & 7))] = pack_chunk<TO>(v + q * CHUNK_ELEMS);
                        }
                    } else if (my_dst >= 0) {
                        TO* dst = out + (size_t)my_dst * ldc + n0 + c0 + h * 32;
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + h * 32 + j < N) dst[j] = from_float<TO>(v[j]);
                    }
                }
                if (vec) {
                    __syncwarp();
                    const int chunk = lane & 7, col = n0 + c0 + chunk * CHUNK_ELEMS;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = i * 4 + (lane >> 3);
                        const uint4 value = stage_rows[r * 8 + (chunk ^ (r & 7))];
                        const long long dst_row = __shfl_sync(0xffffffffu, my_dst, r);
                        if (dst_row >= 0 && col < N)
                            *reinterpret_cast<uint4*>(out + (size_t)dst_row * ldc + col) = value;
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acc_empty0 + 8 * acc) : "memory");
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)Cfg::TMEM_COLS) : "memory");
    }
}

// A [rows, K] in grouped order; W [experts * rows_per_expert, K] (first: rows_per_expert = 2 N, gate then up rows;
// first 2: rows_per_expert = N and relu(z)^2 in the epilogue; otherwise N); C: first ? bfloat16 hidden [rows, N] :
// float32 [rows, N] written by `sorted`. tile_info / num_m_tiles:
// what the grouping kernel left for row tiles of 128. max_m_tiles: the most row tiles there can be.
TTB_EXPORT int ttb_moe_gemm_tcgen05(const void* A, int lda, const void* W, int ldw, void* C, int ldc, int first,
                                    const int* offsets, const int* sorted, const int* tile_info, const int* num_m_tiles,
                                    int rows, int experts, int max_m_tiles, int N, int K, float limit, float alpha,
                                    int* error_flag, cudaStream_t stream) {
    if (rows == 0 || N == 0) return TTB_OK;
    if (!A || !W || !C || !offsets || !sorted || !tile_info || !num_m_tiles || !error_flag) return TTB_ERR_ARGUMENT;
    if (K < 8 || (K & 7) || (lda & 7) || (ldw & 7) || !aligned16(A) || !aligned16(W)) return TTB_ERR_UNSUPPORTED;
    if (first < 0 || first > 2) return TTB_ERR_ARGUMENT;
    const int rows_per_expert = first == 1 ? 2 * N : N;
    if ((long long)experts * rows_per_expert > 2147483647LL) return TTB_ERR_UNSUPPORTED;
    CUtensorMap map_a, map_w;
    if (!tc_make_map(&map_a, A, rows, K, lda, TC_BM)) return TTB_ERR_UNSUPPORTED;
    if (!tc_make_map(&map_w, W, experts * rows_per_expert, K, ldw, first == 1 ? TcCfg::ACC_COLS / 2 : TcCfg::ACC_COLS)) return TTB_ERR_UNSUPPORTED;
    const int out_cols = first == 1 ? TcCfg::ACC_COLS / 2 : TcCfg::ACC_COLS;
    const int n_tiles = (N + out_cols - 1) / out_cols;
    const long long most = (long long)max_m_tiles * n_tiles;
    const int blocks = most < tc_sm_count() ? (int)most : tc_sm_count();
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(moe_gemm_tcgen05_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg::SMEM_BYTES);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(moe_gemm_tcgen05_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg::SMEM_BYTES);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(moe_gemm_tcgen05_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg::SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    if (first == 2)
        ttb_launch(moe_gemm_tcgen05_kernel<2>, dim3(blocks), dim3(TC_THREADS), (size_t)TcCfg::SMEM_BYTES, stream, map_a, map_w,
                   C, offsets, sorted, tile_info, num_m_tiles, N, K, ldc, rows_per_expert, n_tiles, limit, alpha, error_flag);
    else if (first)
        ttb_launch(moe_gemm_tcgen05_kernel<1>, dim3(blocks), dim3(TC_THREADS), (size_t)TcCfg::SMEM_BYTES, stream, map_a, map_w,
                   C, offsets, sorted, tile_info, num_m_tiles, N, K, ldc, rows_per_expert, n_tiles, limit, alpha, error_flag);
    else
        ttb_launch(moe_gemm_tcgen05_kernel<0>, dim3(blocks), dim3(TC_THREADS), (size_t)TcCfg::SMEM_BYTES, stream, map_a, map_w,
                   C, offsets, sorted, tile_info, num_m_tiles, N, K, ldc, rows_per_expert, n_tiles, limit, alpha, error_flag);
    return ttb_launch_status();
}
