// Dense 1-D convolution on the 5th-generation tensor cores (sm_100a).
//
//   y[oc, orow(q)] = epi( sum_{ic,k} W[oc, ic, k] * x[ic, q - p + k*d] )
//
// as an implicit GEMM: M = 128 output positions, N = 128 output channels,
// K = input channels x taps. F16 operands (ggml's F16 arithmetic: both the
// F16 weights and the im2col'd activations are half), F32 accumulation in
// tensor memory.
//
// Operands
//   A  activations, half, chunk-major in HBM: [IC/8][R][8] (8 channels of one
//      row are 16 contiguous bytes). One 3-D TMA box (8 x BR x 8) brings the
//      rows [q0 - p, q0 - p + BR) of 64 channels, halo included, into shared
//      memory as [8 chunks][BR rows][16 B]: the K-major, no-swizzle canonical
//      layout (8-row core matrices 128 B apart, chunks BR*16 B apart). Tap k
//      of the same slab is the same layout starting k*d rows further, so all
//      taps reuse one load.
//   B  weights, packed at upload into the exact shared-memory image of each
//      (tap, 64-channel block, 128-channel tile): [8 chunks][128 oc][16 B],
//      fetched with one bulk copy.
//
// Roles (192 threads, persistent over tiles): warp 0 lane 0 issues the
// copies, warp 1 allocates tensor memory (two 128-column accumulators) and
// lane 0 issues tcgen05.mma, warps 2-5 drain the other accumulator through
// the epilogue (tcgen05.ld 32x32b: warp w owns TMEM lanes 32 (w % 4) ...).
// Every mbarrier wait is bounded in time; on expiry the kernel records an
// error code and the waiting role stops.
#include "kk_kernels.h"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace kk {

constexpr int TC_BM = 128;
constexpr int TC_BN = 128;
constexpr int TC_MAX_BR = 192;                   // rows per slab incl. halo
constexpr int TC_A_BYTES = 8 * TC_MAX_BR * 16;   // 24 KB
constexpr int TC_B_BYTES = 8 * TC_BN * 16;       // 16 KB
constexpr int TC_NSA = 2;                        // A slab stages
constexpr int TC_NSB = 3;                        // B tile stages
constexpr int TC_SMEM = TC_NSA * TC_A_BYTES + TC_NSB * TC_B_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
constexpr int TC_CTAS_PER_SM = 2;  // 2 x 98 KB shared memory, 2 x 256 TMEM columns
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and records `code`) when the phase has not
// completed within TC_WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *err, int code) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (globaltimer() - t0 > TC_WAIT_NS) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y,
                                            int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle (sm_100 layout:
// start >> 4 in [0,14), LBO >> 4 in [16,30), SBO >> 4 in [32,46), version 1
// at bit 46, swizzle mode 0 in [61,64)).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor, kind::f16: D F32 (bit 4), A/B F16 (0), both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------

struct TcParams {
    int IC_blocks;   // input channels / 64 (padded)
    int K, p, d;     // taps, padding, dilation
    int BR;          // slab rows = 127 + (K - 1) d + 1
    int OC;          // real output channels
    int n_tiles;     // OC tiles of 128 in the packed weights
    int n_oc_tiles;  // OC tiles computed
    int64_t m_tiles; // position tiles of 128
    const __half *w; // packed [K][IC_blocks][n_tiles][8][128][8]
    float *out;
    int64_t R_out;
    int64_t n_pos;
    int64_t omul, oadd;
    const float *bias;
    const float *resid;
    int64_t R_resid;
    int resid_half;
    float scale1;
    int accum;
    float scale2;
    int *err;
};

// Persistent: CTA i takes tiles i, i + grid, ... (OC tile fastest, so the
// CTAs working on one slab of positions run close together and share it in
// L2). Warp 0 lane 0: copies. Warp 1: TMEM owner, lane 0 issues MMAs into
// one of two accumulators (128 columns each) so the epilogue of a tile
// overlaps the MMAs of the next. Warps 2-5: epilogue (warp w reads TMEM lanes
// 32 (w % 4) ...).
__global__ void __launch_bounds__(192, 2) k_conv_tc(const __grid_constant__ CUtensorMap amap, TcParams P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;
    uint8_t *sB = smem + TC_NSA * TC_A_BYTES;
    uint64_t *bars = (uint64_t *)(sB + TC_NSB * TC_B_BYTES);
    // A_full[2] A_empty[2] B_full[NSB] B_empty[NSB] acc_full[2] acc_empty[2] tmem slot
    const uint32_t bA_full = smem_u32(bars + 0), bA_empty = smem_u32(bars + 2);
    const uint32_t bB_full = smem_u32(bars + 4), bB_empty = smem_u32(bars + 4 + TC_NSB);
    const uint32_t bAcc_full = smem_u32(bars + 4 + 2 * TC_NSB), bAcc_empty = smem_u32(bars + 6 + 2 * TC_NSB);
    uint32_t *tmem_slot = (uint32_t *)(bars + 8 + 2 * TC_NSB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_tiles_total = P.m_tiles * P.n_oc_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < TC_NSA; ++i) {
            mbar_init(bA_full + 8 * i, 1);
            mbar_init(bA_empty + 8 * i, 1);
        }
        for (int i = 0; i < TC_NSB; ++i) {
            mbar_init(bB_full + 8 * i, 1);
            mbar_init(bB_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bAcc_full + 8 * i, 1);
            mbar_init(bAcc_empty + 8 * i, 4);  // one arrive per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * TC_BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    const uint32_t a_bytes = 8u * (uint32_t)P.BR * 16u;
    const uint32_t lbo_a = (uint32_t)P.BR * 16u;
    const uint32_t lbo_b = (uint32_t)TC_BN * 16u;

    if (warp == 0) {
        if (lane == 0) {
            // producer
            bool ok = true;
            uint32_t ia = 0, ib = 0;  // running slab / tile counters
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
                const int64_t mt = tile / P.n_oc_tiles;
                const int nt = (int)(tile % P.n_oc_tiles);
                const int row0 = (int)(mt * TC_BM - P.p);
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % TC_NSA;
                    if (ia >= TC_NSA) ok = mbar_wait(bA_empty + 8 * sa, ((ia / TC_NSA) & 1) ^ 1, P.err, 11);
                    if (!ok) break;
                    mbar_expect_tx(bA_full + 8 * sa, a_bytes);
                    tma_load_3d(smem_u32(sA + sa * TC_A_BYTES), &amap, bA_full + 8 * sa, 0, row0, 8 * b);
                    for (int k = 0; k < P.K; ++k, ++ib) {
                        const int sb = ib % TC_NSB;
                        if (ib >= TC_NSB) ok = mbar_wait(bB_empty + 8 * sb, ((ib / TC_NSB) & 1) ^ 1, P.err, 12);
                        if (!ok) break;
                        mbar_expect_tx(bB_full + 8 * sb, TC_B_BYTES);
                        const __half *src =
                            P.w + ((((size_t)k * P.IC_blocks + b) * P.n_tiles + nt) * (size_t)(8 * TC_BN * 8));
                        bulk_load(smem_u32(sB + sb * TC_B_BYTES), src, TC_B_BYTES, bB_full + 8 * sb);
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer
            const uint32_t idesc = idesc_f16(TC_BM, TC_BN);
            bool ok = true;
            uint32_t ia = 0, ib = 0, it = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x, ++it) {
                const int ab = it & 1;
                if (it >= 2) ok = mbar_wait(bAcc_empty + 8 * ab, ((it >> 1) & 1) ^ 1, P.err, 17);
                if (!ok) break;
                fence_after_sync();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * TC_BN);
                uint32_t acc = 0;
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % TC_NSA;
                    ok = mbar_wait(bA_full + 8 * sa, (ia / TC_NSA) & 1, P.err, 13);
                    if (!ok) break;
                    fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + sa * TC_A_BYTES);
                    for (int k = 0; k < P.K; ++k, ++ib) {
                        const int sb = ib % TC_NSB;
                        ok = mbar_wait(bB_full + 8 * sb, (ib / TC_NSB) & 1, P.err, 14);
                        if (!ok) break;
                        fence_after_sync();
                        const uint32_t b_base = smem_u32(sB + sb * TC_B_BYTES);
                        const uint32_t a_tap = a_base + (uint32_t)(k * P.d) * 16u;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t ad = sdesc(a_tap + (uint32_t)(2 * ks) * lbo_a, lbo_a, 128);
                            const uint64_t bd = sdesc(b_base + (uint32_t)(2 * ks) * lbo_b, lbo_b, 128);
                            mma_f16(d_tmem, ad, bd, idesc, acc);
                            acc = 1;
                        }
                        mma_commit(bB_empty + 8 * sb);
                    }
                    mma_commit(bA_empty + 8 * sa);
                }
                mma_commit(bAcc_full + 8 * ab);
            }
        }
        __syncwarp();
    } else {
        // epilogue warps 2..5
        const int lg = warp & 3;  // TMEM lane group
        uint32_t it = 0;
        for (int64_t tile = blockIdx.x; tile < n_tiles_total; tile += gridDim.x, ++it) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int n0 = (int)(tile % P.n_oc_tiles) * TC_BN;
            const int ab = it & 1;
            int ok_lane = 0;
            if (lane == 0) ok_lane = mbar_wait(bAcc_full + 8 * ab, (it >> 1) & 1, P.err, 15) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok_lane, 0) == 0) break;
            fence_after_sync();
            const int64_t q = mt * TC_BM + lg * 32 + lane;
            const int64_t orow = q * P.omul + P.oadd;
            const bool row_ok = q < P.n_pos && orow >= 0 && orow < P.R_out;
            const int64_t rrow = P.resid_half ? (orow >> 1) : orow;
            for (int c0 = 0; c0 < TC_BN; c0 += 32) {
                if (n0 + c0 >= P.OC) break;  // warp-uniform
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ab * TC_BN + c0), r);
                if (!row_ok) continue;
                // The residual and the accumulated output may alias the output
                // (in-place updates): read all 32 of this row's values first so
                // the loads overlap, then compute and store.
                const int nj = P.OC - (n0 + c0) < 32 ? P.OC - (n0 + c0) : 32;
                float res[32], old[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int oc = n0 + c0 + j;
                    res[j] = (P.resid && j < nj) ? P.resid[(int64_t)oc * P.R_resid + rrow] : 0.f;
                    old[j] = (P.accum && j < nj) ? P.out[(int64_t)oc * P.R_out + orow] : 0.f;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (j >= nj) break;
                    const int oc = n0 + c0 + j;
                    float v = __uint_as_float(r[j]);
                    if (P.bias) v = __fadd_rn(v, P.bias[oc]);
                    if (P.resid) v = __fadd_rn(res[j], v);
                    if (P.scale1 != 1.0f) v = __fmul_rn(v, P.scale1);
                    if (P.accum) v = __fadd_rn(old[j], v);
                    if (P.scale2 != 1.0f) v = __fmul_rn(v, P.scale2);
                    P.out[(int64_t)oc * P.R_out + orow] = v;
                }
            }
            // hand the accumulator back to the MMA warp
            fence_before_sync();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bAcc_empty + 8 * ab) : "memory");
        }
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TC_BN) : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static int g_num_sms = 148;

cudaError_t conv_tc_init() {
    if (!g_encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return cudaFuncSetAttribute(k_conv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
}

int conv_tc_max_halo() { return TC_MAX_BR - TC_BM; }

cudaError_t conv_tc(const ConvTcArgs &a, cudaStream_t st) {
    const int BR = (TC_BM - 1) + (a.K - 1) * a.d + 1;
    if (BR > TC_MAX_BR || a.IC_pad % 64 != 0 || a.OC > a.n_tiles * TC_BN) return cudaErrorInvalidValue;
    CUtensorMap map;
    cuuint64_t dims[3] = {8, (cuuint64_t)a.R_in, (cuuint64_t)(a.IC_pad / 8)};
    cuuint64_t strides[2] = {16, (cuuint64_t)a.R_in * 16};
    cuuint32_t box[3] = {8, (cuuint32_t)BR, 8};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void *)a.in, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    TcParams P;
    P.IC_blocks = a.IC_pad / 64;
    P.K = a.K;
    P.p = a.p;
    P.d = a.d;
    P.BR = BR;
    P.OC = a.OC;
    P.n_tiles = a.n_tiles;
    P.w = a.w;
    P.out = a.out;
    P.R_out = a.R_out;
    P.n_pos = a.n_pos;
    P.omul = a.omul;
    P.oadd = a.oadd;
    P.bias = a.bias;
    P.resid = a.resid;
    P.R_resid = a.R_resid;
    P.resid_half = a.resid_half;
    P.scale1 = a.scale1;
    P.accum = a.accum;
    P.scale2 = a.scale2;
    P.err = a.err;
    P.n_oc_tiles = (a.OC + TC_BN - 1) / TC_BN;
    P.m_tiles = (a.n_pos + TC_BM - 1) / TC_BM;
    const int64_t tiles = P.m_tiles * P.n_oc_tiles;
    const int64_t slots = (int64_t)g_num_sms * TC_CTAS_PER_SM;
    const unsigned grid = (unsigned)(tiles < slots ? tiles : slots);
    k_conv_tc<<<grid, 192, TC_SMEM, st>>>(map, P);
    return cudaGetLastError();
}

}  // namespace kk
