// Dense 1-D convolution on the 5th-generation tensor cores (sm_100a).
//
//   y[oc, orow(q)] = epi( sum_{ic,k} W[oc, ic, k] * x[ic, q - p + k*d] )
//
// as an implicit GEMM over tiles of 256 output positions x 128 output
// channels, K = input channels x taps. F16 operands (ggml's F16 arithmetic:
// both the F16 weights and the im2col'd activations are half), F32
// accumulation in tensor memory.
//
// Shared-memory operands
//   activations  half, chunk-major in HBM: [IC/8][Ry][8] (8 channels of one row
//      are 16 contiguous bytes) with zero margins of kHalfLo rows before and
//      kHalfHi rows after every chunk. One slab = rows [q0 - p, q0 - p +
//      TC_SLAB) of 64 channels, halo included, is 8 plain bulk copies (one
//      contiguous 5 KB run per chunk) into shared memory as
//      [8 chunks][TC_SLAB rows][16 B]: the K-major, no-swizzle canonical
//      layout (8-row core matrices 128 B apart, chunks TC_SLAB*16 B apart).
//      Tap k is the same layout starting k*d rows further, so all taps reuse
//      one slab.
//   weights  packed at upload into the exact shared-memory image of each
//      (tap, 64-channel block, 128-channel tile): [8 chunks][128 oc][16 B],
//      fetched with one bulk copy.
//
// Two kernels. k_conv_tct (channels x positions, every conv whose output row
// is its position, >= 64 channels): one M = 128 channels x N = 256 positions
// MMA per 16-channel step, weights as operand A, the shifted slab as operand
// B; an epilogue thread owns one channel and 32 consecutive positions.
// k_conv_tc (positions x channels): two M = 128 positions x N = 128 channels
// MMAs per step; its register epilogue serves the strided row maps of the
// ConvTranspose phases, the x2-upsampled shortcut and narrow outputs.
//
// Roles (320 threads, one CTA per SM, persistent over tiles): warp 0 lane 0
// issues the copies, warp 1 allocates tensor memory (two 256-column
// accumulators) and lane 0 issues tcgen05.mma, warps 2-9 drain the other
// accumulator through the epilogue (tcgen05.ld 32x32b: warp w owns TMEM
// lanes 32 (w % 4) ...).
// Every mbarrier wait is bounded in time; on expiry the kernel records an
// error code and the waiting role stops. Before the tensor memory is freed
// the producer waits (bounded) for its last copies and the MMA thread for its
// last MMAs.
#include "kk_kernels.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

namespace kk {

constexpr int TC_BM = 256;                       // positions per tile
constexpr int TC_HM = 128;                       // rows per MMA
constexpr int TC_BN = 128;                       // output channels per tile
constexpr int TC_SLAB = 320;                     // rows per slab incl. halo
constexpr int TC_A_BYTES = 8 * TC_SLAB * 16;     // 40 KB
constexpr int TC_B_BYTES = 8 * TC_BN * 16;       // 16 KB
constexpr int TC_NSA = 2;                        // A slab stages
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_TMEM_COLS = 2 * (TC_BM / TC_HM) * TC_BN;  // 512: two accumulators
constexpr int TC_BLK_BYTES = 32 * 32 * 4;        // one [32 ch][32 positions] F32 epilogue block
constexpr int TC_NSB = 8;                        // weight tile stages of k_conv_tc
constexpr int TC_SMEM = TC_NSA * TC_A_BYTES + TC_NSB * TC_B_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;   // 2 s
constexpr unsigned long long TC_DRAIN_NS = 200000000ull;   // 0.2 s
static_assert(TC_SMEM <= 227 * 1024, "shared memory");
static_assert(TC_SLAB - TC_BM <= kHalfLo + kHalfHi, "slab overhang");

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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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
// completed within `limit_ns`.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *err, int code,
                                          unsigned long long limit_ns = TC_WAIT_NS) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (globaltimer() - t0 > limit_ns) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// 2-D tensor copies of one [32 ch][32 rows] F32 block (x = row, y = channel).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// the shared-memory source of all but the newest N committed stores has been read
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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

// The same load into floats (the accumulator values), for in-place epilogues.
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7]),
          "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]), "=f"(r[14]), "=f"(r[15]),
          "=f"(r[16]), "=f"(r[17]), "=f"(r[18]), "=f"(r[19]), "=f"(r[20]), "=f"(r[21]), "=f"(r[22]),
          "=f"(r[23]), "=f"(r[24]), "=f"(r[25]), "=f"(r[26]), "=f"(r[27]), "=f"(r[28]), "=f"(r[29]),
          "=f"(r[30]), "=f"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------

struct TcParams {
    int IC_blocks;    // input channels / 64 (padded)
    int K, p, d;      // taps, padding, dilation
    int OC;           // real output channels
    int n_tiles;      // OC tiles of 128 in the packed weights
    int n_oc_tiles;   // OC tiles computed
    int mma_n;        // MMA N: 128, or the channel count rounded to 16 when it is smaller
    int phase_oc;     // > 0: output channel n is channel n % phase_oc of phase n / phase_oc
    int64_t m_tiles;  // position tiles of 256
    const __half *a;  // half operand, row 0 of chunk 0
    int64_t R_a;      // chunk stride (rows)
    int a_wrap;       // > 0: K block b >= a_wrap reads operand block b - a_wrap
    float acc_scale;  // the accumulator times this power of two first (1: none)
    const __half *w;  // packed [K][IC_blocks][n_tiles][8][128][8]
    float *out;
    int64_t R_out;
    int64_t n_pos;
    int64_t omul, oadd;
    const float *bias;
    const float *resid;
    int64_t R_resid;
    int resid_half;
    const float *chscale;  // non-null: per output channel, after bias and residual
    float scale1;
    int accum;
    float scale2;
    int *err;
    float2 *part;     // non-null: 32-row block partials of the output, [OC][R_out / 32]
    Batch sb;         // utterances of the output level (each starts on a block boundary)
    int sm, sextra;   // level multiplier and extra rows of the output level
    // k_conv_tcf: the operand is half(snake(adain(x))) of the F32 input x
    // ([IC][R_out], read through a tensor map) on the valid rows of level
    // (sm, sextra), zero elsewhere
    int IC;                              // channels of x (a multiple of 64)
    const float2 *x_ms;                  // [n][IC] (mean, scale)
    const float *x_nw, *x_nb;            // [IC] norm weight and bias
    const float *x_gamma, *x_beta;       // [n][IC]
    const float *x_alpha;                // [IC] Snake alpha
    float nz;                            // -0.0f, opaque to the compiler (packed products)
    unsigned long long nz2;              // two packed -0.0f, the same
    // k_convt_tc: channels per phase in one tile (the tile's MMA N is
    // omul * phase_nc, its rows phase-major)
    int phase_nc;
    // k_conv_tct: non-null, the dynamic tile order (ConvTcArgs::sched)
    int *sched;
};

// Positions x channels, register epilogue (strided row maps). Persistent: CTA
// i takes tiles i, i + grid, ... (OC tile fastest, so the CTAs working on one
// slab of positions run close together and share it in L2; the phases of a
// ConvTranspose tile then write their interleaved rows close in time).
__global__ void __launch_bounds__(TC_THREADS, 1) k_conv_tc(const __grid_constant__ TcParams P) {
    constexpr int NSB = TC_NSB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;
    uint8_t *sB = smem + TC_NSA * TC_A_BYTES;
    uint64_t *bars = (uint64_t *)(sB + NSB * TC_B_BYTES);
    // A_full[2] A_empty[2] B_full[NSB] B_empty[NSB] acc_full[2] acc_empty[2]
    // drain tmem-slot
    const uint32_t bA_full = smem_u32(bars + 0), bA_empty = smem_u32(bars + 2);
    const uint32_t bB_full = smem_u32(bars + 4), bB_empty = smem_u32(bars + 4 + NSB);
    const uint32_t bAcc_full = smem_u32(bars + 4 + 2 * NSB), bAcc_empty = smem_u32(bars + 6 + 2 * NSB);
    const uint32_t bDrain = smem_u32(bars + 8 + 2 * NSB);
    uint32_t *tmem_slot = (uint32_t *)(bars + 9 + 2 * NSB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_tiles_total = P.m_tiles * P.n_oc_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < TC_NSA; ++i) {
            mbar_init(bA_full + 8 * i, 1);
            mbar_init(bA_empty + 8 * i, 1);
        }
        for (int i = 0; i < NSB; ++i) {
            mbar_init(bB_full + 8 * i, 1);
            mbar_init(bB_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bAcc_full + 8 * i, 1);
            mbar_init(bAcc_empty + 8 * i, TC_EPI_WARPS);  // one arrive per epilogue warp
        }
        mbar_init(bDrain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    constexpr uint32_t lbo_a = (uint32_t)TC_SLAB * 16u;
    constexpr uint32_t lbo_b = (uint32_t)TC_BN * 16u;

    if (warp == 0) {
        if (lane == 0) {
            // producer
            bool ok = true;
            uint32_t ia = 0, ib = 0;  // running slab / tile counters
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
                const int64_t mt = tile / P.n_oc_tiles;
                const int nt = (int)(tile % P.n_oc_tiles);
                const int64_t row0 = mt * TC_BM - P.p;  // >= -kHalfLo (checked on the host)
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % TC_NSA;
                    if (ia >= TC_NSA) ok = mbar_wait(bA_empty + 8 * sa, ((ia / TC_NSA) & 1) ^ 1, P.err, 11);
                    if (!ok) break;
                    mbar_expect_tx(bA_full + 8 * sa, TC_A_BYTES);
                    const uint32_t dst = smem_u32(sA + sa * TC_A_BYTES);
                    const int bo = (P.a_wrap > 0 && b >= P.a_wrap) ? b - P.a_wrap : b;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const __half *src = P.a + ((int64_t)(8 * bo + c) * P.R_a + row0) * 8;
                        bulk_load(dst + (uint32_t)c * lbo_a, src, lbo_a, bA_full + 8 * sa);
                    }
                    for (int k = 0; k < P.K; ++k, ++ib) {
                        const int sb = ib % NSB;
                        if (ib >= NSB) ok = mbar_wait(bB_empty + 8 * sb, ((ib / NSB) & 1) ^ 1, P.err, 12);
                        if (!ok) break;
                        mbar_expect_tx(bB_full + 8 * sb, TC_B_BYTES);
                        const __half *src =
                            P.w + ((((size_t)k * P.IC_blocks + b) * P.n_tiles + nt) * (size_t)(8 * TC_BN * 8));
                        bulk_load(smem_u32(sB + sb * TC_B_BYTES), src, TC_B_BYTES, bB_full + 8 * sb);
                    }
                }
            }
            // Drain: the last copy issued into each stage has landed (already
            // consumed on the normal path, so these return at once).
            for (uint32_t i = (ia > TC_NSA ? ia - TC_NSA : 0); i < ia; ++i)
                mbar_wait(bA_full + 8 * (i % TC_NSA), (i / TC_NSA) & 1, P.err, 18, TC_DRAIN_NS);
            for (uint32_t i = (ib > NSB ? ib - NSB : 0); i < ib; ++i)
                mbar_wait(bB_full + 8 * (i % NSB), (i / NSB) & 1, P.err, 18, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer
            const uint32_t idesc = idesc_f16(TC_HM, P.mma_n);
            bool ok = true;
            uint32_t ia = 0, ib = 0, it = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x, ++it) {
                const int ab = it & 1;
                if (it >= 2) ok = mbar_wait(bAcc_empty + 8 * ab, ((it >> 1) & 1) ^ 1, P.err, 17);
                if (!ok) break;
                fence_after_sync();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * 2 * TC_BN);
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % TC_NSA;
                    ok = mbar_wait(bA_full + 8 * sa, (ia / TC_NSA) & 1, P.err, 13);
                    if (!ok) break;
                    fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + sa * TC_A_BYTES);
                    for (int k = 0; k < P.K; ++k, ++ib) {
                        const int sb = ib % NSB;
                        ok = mbar_wait(bB_full + 8 * sb, (ib / NSB) & 1, P.err, 14);
                        if (!ok) break;
                        fence_after_sync();
                        const uint32_t b_base = smem_u32(sB + sb * TC_B_BYTES);
                        const uint32_t a_tap = a_base + (uint32_t)(k * P.d) * 16u;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t bd = sdesc(b_base + (uint32_t)(2 * ks) * lbo_b, lbo_b, 128);
                            const uint32_t acc = (b > 0 || k > 0 || ks > 0) ? 1u : 0u;
#pragma unroll
                            for (int h = 0; h < TC_BM / TC_HM; ++h) {
                                const uint64_t ad =
                                    sdesc(a_tap + (uint32_t)(h * TC_HM) * 16u + (uint32_t)(2 * ks) * lbo_a, lbo_a, 128);
                                mma_f16(d_tmem + (uint32_t)(h * TC_BN), ad, bd, idesc, acc);
                            }
                        }
                        mma_commit(bB_empty + 8 * sb);
                    }
                    mma_commit(bA_empty + 8 * sa);
                }
                if (ok) mma_commit(bAcc_full + 8 * ab);
            }
            // Drain: every MMA issued above has completed before the
            // accumulators are freed.
            mma_commit(bDrain);
            mbar_wait(bDrain, 0, P.err, 19, TC_DRAIN_NS);
        }
        __syncwarp();
    } else {
        // epilogue warps 2..9
        const int ew = warp - 2;
        const int lg = warp & 3;           // TMEM lane group
        const int half = ew >> 2;          // 128-row half of the tile
        const bool has_res = P.resid != nullptr;
        uint32_t it = 0;
        for (int64_t tile = blockIdx.x; tile < n_tiles_total; tile += gridDim.x, ++it) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int n0 = (int)(tile % P.n_oc_tiles) * TC_BN;
            const int ab = it & 1;
            const int64_t qw = mt * TC_BM + half * TC_HM + lg * 32;  // first row of this warp
            // phase-packed transposed conv: this tile's channels belong to
            // phase r, whose output rows are q * omul + oadd + r
            const int ph = P.phase_oc > 0 ? n0 / P.phase_oc : 0;
            const int oc0 = n0 - ph * P.phase_oc;
            int ok_lane = 0;
            if (lane == 0) ok_lane = mbar_wait(bAcc_full + 8 * ab, (it >> 1) & 1, P.err, 15) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok_lane, 0) == 0) break;
            __syncwarp();
            fence_after_sync();
            const int64_t q = qw + lane;
            const int64_t orow = q * P.omul + P.oadd + ph;
            const bool row_ok = q < P.n_pos && orow >= 0 && orow < P.R_out;
            const uint32_t t_base = tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(ab * 2 * TC_BN + half * TC_BN);
            for (int c0 = 0; c0 < TC_BN; c0 += 32) {
                if (n0 + c0 >= P.OC) break;  // warp-uniform
                // every lane takes part in the warp-collective TMEM load and
                // shuffles; row_ok only predicates the memory accesses
                uint32_t r[32];
                tmem_ld32(t_base + (uint32_t)c0, r);
                const int nj = P.OC - (n0 + c0) < 32 ? P.OC - (n0 + c0) : 32;
                const int64_t rrow = P.resid_half ? (orow >> 1) : orow;
                const float b_lane = (P.bias && lane < nj) ? __ldg(P.bias + oc0 + c0 + lane) : 0.f;
                const float s_lane = (P.chscale && lane < nj) ? __ldg(P.chscale + oc0 + c0 + lane) : 1.f;
                // The residual and the accumulated output may alias the
                // output (in-place updates): read all of this row's values
                // first so the loads overlap, then compute and store.
                float res[32], old[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) res[j] = old[j] = 0.f;
                if (has_res) {
                    const float *rp = P.resid + (int64_t)(oc0 + c0) * P.R_resid + rrow;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (row_ok && j < nj) res[j] = rp[(int64_t)j * P.R_resid];
                }
                if (P.accum) {
                    const float *op = P.out + (int64_t)(oc0 + c0) * P.R_out + orow;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (row_ok && j < nj) old[j] = op[(int64_t)j * P.R_out];
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float bj = __shfl_sync(0xffffffffu, b_lane, j);
                    const float sj = __shfl_sync(0xffffffffu, s_lane, j);
                    float v = __uint_as_float(r[j]);
                    if (P.acc_scale != 1.0f) v = __fmul_rn(v, P.acc_scale);
                    if (P.bias) v = __fadd_rn(v, bj);
                    if (has_res) v = __fadd_rn(res[j], v);
                    if (P.chscale) v = __fmul_rn(v, sj);
                    if (P.scale1 != 1.0f) v = __fmul_rn(v, P.scale1);
                    if (P.accum) v = __fadd_rn(old[j], v);
                    if (P.scale2 != 1.0f) v = __fmul_rn(v, P.scale2);
                    if (row_ok && j < nj) P.out[(int64_t)(oc0 + c0 + j) * P.R_out + orow] = v;
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// kernel, channels x positions
// ---------------------------------------------------------------------------
//
// The same convolution with the roles swapped: D[oc][q] = sum W[oc][.] x[.][q]
// with M = 128 output channels (the weight tile is operand A) and N = 256
// positions (the activation slab, shifted by k d rows for tap k, is operand
// B), one MMA per 16-channel step instead of two. Each MMA reads 4 KB of
// weights and 8 KB of activations from shared memory, three quarters of the
// 16 KB that two 128 x 128 MMAs read for the same work, which keeps the tensor
// pipe under the shared-memory bandwidth limit.
// The accumulator holds channels in TMEM lanes and positions in columns, so
// an epilogue thread owns one output channel and 32 consecutive positions:
// exactly a 128-byte run of the channel-major output, read and written with
// float4 accesses, no staging. Output row = position (omul 1, oadd 0).

// STAGED (output row = position over the whole level, TMA maps available):
// each warp moves [32 channels][32 positions] blocks through shared memory
// with a 128-byte swizzle (thread = channel writes and reads its 128-byte row
// without bank conflicts) and TMA loads / stores of whole 4 KB blocks, the
// residual prefetched one block ahead. Otherwise each thread reads and writes
// its 128-byte run of the output directly.
__host__ __device__ constexpr int tt_nsa(bool staged) { return staged ? 2 : 3; }  // activation slab stages
// weight tile stages: the weight stream of the k = 7 / 11 tiles is bound by
// the bytes in flight from L2 (staged: 5 stages, 226 KB of shared memory in
// all, made stage-1 k = 11 3.5 % faster than 4)
__host__ __device__ constexpr int tt_nsw(bool staged) { return staged ? 5 : 6; }
__host__ __device__ constexpr int tt_smem(bool staged) {
    return tt_nsa(staged) * TC_A_BYTES + tt_nsw(staged) * TC_B_BYTES + (staged ? TC_EPI_WARPS * 2 * TC_BLK_BYTES : 0) +
           1024 /*barriers*/ + 1024 /*align*/;
}
static_assert(tt_smem(true) <= 227 * 1024 && tt_smem(false) <= 227 * 1024, "shared memory");

// Byte offset of 16-byte chunk i of row r in a 128-byte-swizzled block (the
// layout TMA reads and writes with CU_TENSOR_MAP_SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz128(int r, int i) { return (uint32_t)(r * 128 + ((i ^ (r & 7)) << 4)); }

// Instance-norm partials of one output channel over the 32-position blocks
// of a tile: (S, M2) with S the sum of the block's k rows that are valid rows
// of its utterance and M2 = sum (v - S / k)^2, both in FP32; (0, 0) for a
// block of gap rows. Every utterance starts on a block boundary, so a block
// belongs to at most one utterance. The utterance and its rows are the same
// for the 32 lanes of a warp (they share positions and differ in channel).
struct BlockStats {
    int u;           // utterance whose slot holds the current block
    int64_t lo, hi;  // its valid rows

    __device__ __forceinline__ void set_utt(const TcParams &P, int uu) {
        u = uu;
        lo = (int64_t)P.sm * __ldg(P.sb.offT + uu);
        hi = lo + (int64_t)P.sm * __ldg(P.sb.T + uu) + P.sextra;
    }
    __device__ __forceinline__ void begin(const TcParams &P, int64_t p) { set_utt(P, utt_of_row(P.sb, P.sm, p)); }
    // v[j] = output at position p0 + j
    __device__ __forceinline__ float2 block(const TcParams &P, const float (&v)[32], int64_t p0) {
        for (int guard = 0; guard < P.sb.n && u + 1 < P.sb.n; ++guard) {
            if ((int64_t)P.sm * __ldg(P.sb.offT + u + 1) > p0) break;
            set_utt(P, u + 1);
        }
        if (p0 >= lo && p0 + 32 <= hi) {
            float2 a[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int j = 0; j < 32; j += 2) a[(j >> 1) & 1] = f2add(a[(j >> 1) & 1], make_float2(v[j], v[j + 1]));
            const float S = (a[0].x + a[0].y) + (a[1].x + a[1].y);
            const float nmb = S * (-1.0f / 32.0f);
            float2 q[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float2 dv = f2add(make_float2(v[j], v[j + 1]), make_float2(nmb, nmb));
                q[(j >> 1) & 1] = f2fma(dv, dv, q[(j >> 1) & 1]);
            }
            return make_float2(S, (q[0].x + q[0].y) + (q[1].x + q[1].y));
        }
        // the block ends the utterance, or holds gap rows only
        const int j0 = p0 >= lo ? 0 : (int)(lo - p0 < 32 ? lo - p0 : 32);
        const int j1 = hi <= p0 ? 0 : (int)(hi - p0 < 32 ? hi - p0 : 32);
        if (j1 <= j0) return make_float2(0.f, 0.f);
        float S = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j >= j0 && j < j1) S += v[j];
        const float mb = __fdiv_rn(S, (float)(j1 - j0));
        float M2 = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j >= j0 && j < j1) {
                const float dv = v[j] - mb;
                M2 = fmaf(dv, dv, M2);
            }
        return make_float2(S, M2);
    }
};

// Pairs of block partials as one 16-byte store: blocks 2i and 2i + 1 of a
// thread's four are adjacent in part (the position half of a tile starts on
// a multiple of 128 rows, and R_out / 32 is a multiple of 4).
__device__ __forceinline__ void store_part(const TcParams &P, float2 q, float2 &prev, int c, bool chan_ok, int64_t p0,
                                           int cc) {
    if (cc & 1) {
        if (chan_ok && p0 < P.R_out)
            *reinterpret_cast<float4 *>(P.part + (int64_t)c * (P.R_out >> 5) + (p0 >> 5) - 1) =
                make_float4(prev.x, prev.y, q.x, q.y);
    } else {
        prev = q;
    }
}

template <bool STAGED>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_conv_tct(const __grid_constant__ TcParams P, const __grid_constant__ CUtensorMap omap,
               const __grid_constant__ CUtensorMap rmap) {
    constexpr int NSA = tt_nsa(STAGED), NSW = tt_nsw(STAGED);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;                     // activation slabs
    uint8_t *sW = smem + NSA * TC_A_BYTES;  // weight tiles
    uint8_t *sE = sW + NSW * TC_B_BYTES;    // STAGED: two 4 KB blocks per epilogue warp (1 KB aligned)
    uint64_t *bars = (uint64_t *)(sE + (STAGED ? TC_EPI_WARPS * 2 * TC_BLK_BYTES : 0));
    // A_full[NSA] A_empty[NSA] W_full[NSW] W_empty[NSW] acc_full[2] acc_empty[2]
    // drain res[8 warps][2] tmem-slot sched_full[4] sched_empty[4] sched_tile[4]
    const uint32_t bA_full = smem_u32(bars), bA_empty = smem_u32(bars + NSA);
    const uint32_t bW_full = smem_u32(bars + 2 * NSA), bW_empty = smem_u32(bars + 2 * NSA + NSW);
    const uint32_t bAcc_full = smem_u32(bars + 2 * NSA + 2 * NSW);
    const uint32_t bAcc_empty = smem_u32(bars + 2 * NSA + 2 * NSW + 2);
    const uint32_t bDrain = smem_u32(bars + 2 * NSA + 2 * NSW + 4);
    const uint32_t bRes = smem_u32(bars + 2 * NSA + 2 * NSW + 5);
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * NSA + 2 * NSW + 5 + 2 * TC_EPI_WARPS);
    // dynamic tile order: the producer publishes each tile index (-1: no
    // more) in a 4-slot ring that the MMA thread and the epilogue warps read
    const uint32_t bS_full = smem_u32(bars + 2 * NSA + 2 * NSW + 6 + 2 * TC_EPI_WARPS);
    const uint32_t bS_empty = bS_full + 8 * 4;
    volatile int64_t *s_tile = (volatile int64_t *)(bars + 2 * NSA + 2 * NSW + 14 + 2 * TC_EPI_WARPS);
    const bool dyn = P.sched != nullptr;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_tiles_total = P.m_tiles * P.n_oc_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) {
            mbar_init(bS_full + 8 * i, 1);
            mbar_init(bS_empty + 8 * i, 1 + TC_EPI_WARPS);
        }
        for (int i = 0; i < NSA; ++i) {
            mbar_init(bA_full + 8 * i, 1);
            mbar_init(bA_empty + 8 * i, 1);
        }
        for (int i = 0; i < NSW; ++i) {
            mbar_init(bW_full + 8 * i, 1);
            mbar_init(bW_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bAcc_full + 8 * i, 1);
            mbar_init(bAcc_empty + 8 * i, TC_EPI_WARPS);
        }
        mbar_init(bDrain, 1);
        for (int i = 0; i < 2 * TC_EPI_WARPS; ++i) mbar_init(bRes + 8 * i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    constexpr uint32_t lbo_a = (uint32_t)TC_SLAB * 16u;  // activation chunk stride
    constexpr uint32_t lbo_w = (uint32_t)TC_BN * 16u;    // weight chunk stride

    if (warp == 0) {
        if (lane == 0) {
            // producer (and, in the dynamic order, the tile scheduler)
            bool ok = true;
            uint32_t ia = 0, iw = 0;
            int64_t tile = blockIdx.x;
            for (uint32_t it = 0; ok; ++it) {
                if (dyn) {
                    const int q = it & 3;
                    if (it >= 4) ok = mbar_wait(bS_empty + 8 * q, ((it >> 2) & 1) ^ 1, P.err, 22);
                    if (!ok) break;
                    s_tile[q] = tile < n_tiles_total ? tile : -1;
                    mbar_arrive(bS_full + 8 * q);
                }
                if (tile >= n_tiles_total) break;
                const int64_t mt = tile / P.n_oc_tiles;
                const int nt = (int)(tile % P.n_oc_tiles);
                // the next tile, asked for before this one's copies are issued
                tile = dyn ? (int64_t)gridDim.x + atomicAdd(P.sched, 1) : tile + gridDim.x;
                const int64_t row0 = mt * TC_BM - P.p;  // >= -kHalfLo (checked on the host)
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % NSA;
                    if (ia >= NSA) ok = mbar_wait(bA_empty + 8 * sa, ((ia / NSA) & 1) ^ 1, P.err, 11);
                    if (!ok) break;
                    mbar_expect_tx(bA_full + 8 * sa, TC_A_BYTES);
                    const uint32_t dst = smem_u32(sA + sa * TC_A_BYTES);
                    const int bo = (P.a_wrap > 0 && b >= P.a_wrap) ? b - P.a_wrap : b;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const __half *src = P.a + ((int64_t)(8 * bo + c) * P.R_a + row0) * 8;
                        bulk_load(dst + (uint32_t)c * lbo_a, src, lbo_a, bA_full + 8 * sa);
                    }
                    for (int k = 0; k < P.K; ++k, ++iw) {
                        const int sw = iw % NSW;
                        if (iw >= NSW) ok = mbar_wait(bW_empty + 8 * sw, ((iw / NSW) & 1) ^ 1, P.err, 12);
                        if (!ok) break;
                        mbar_expect_tx(bW_full + 8 * sw, TC_B_BYTES);
                        const __half *src =
                            P.w + ((((size_t)k * P.IC_blocks + b) * P.n_tiles + nt) * (size_t)(8 * TC_BN * 8));
                        bulk_load(smem_u32(sW + sw * TC_B_BYTES), src, TC_B_BYTES, bW_full + 8 * sw);
                    }
                }
            }
            for (uint32_t i = (ia > NSA ? ia - NSA : 0); i < ia; ++i)
                mbar_wait(bA_full + 8 * (i % NSA), (i / NSA) & 1, P.err, 18, TC_DRAIN_NS);
            for (uint32_t i = (iw > NSW ? iw - NSW : 0); i < iw; ++i)
                mbar_wait(bW_full + 8 * (i % NSW), (i / NSW) & 1, P.err, 18, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: A = weights (M = 128 channels), B = activations (N = 256 positions)
            const uint32_t idesc = idesc_f16(TC_BN, TC_BM);
            bool ok = true;
            uint32_t ia = 0, iw = 0, it = 0;
            int64_t tile = blockIdx.x;
            for (; ok; ++it) {
                if (dyn) {
                    const int q = it & 3;
                    ok = mbar_wait(bS_full + 8 * q, (it >> 2) & 1, P.err, 23);
                    if (!ok) break;
                    tile = s_tile[q];
                    mbar_arrive(bS_empty + 8 * q);
                    if (tile < 0) break;
                } else if (it > 0) {
                    tile += gridDim.x;
                }
                if (tile >= n_tiles_total) break;
                const int ab = it & 1;
                if (it >= 2) ok = mbar_wait(bAcc_empty + 8 * ab, ((it >> 1) & 1) ^ 1, P.err, 17);
                if (!ok) break;
                fence_after_sync();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * TC_BM);
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % NSA;
                    ok = mbar_wait(bA_full + 8 * sa, (ia / NSA) & 1, P.err, 13);
                    if (!ok) break;
                    fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + sa * TC_A_BYTES);
                    for (int k = 0; k < P.K; ++k, ++iw) {
                        const int sw = iw % NSW;
                        ok = mbar_wait(bW_full + 8 * sw, (iw / NSW) & 1, P.err, 14);
                        if (!ok) break;
                        fence_after_sync();
                        const uint32_t w_base = smem_u32(sW + sw * TC_B_BYTES);
                        const uint32_t x_tap = a_base + (uint32_t)(k * P.d) * 16u;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t wd = sdesc(w_base + (uint32_t)(2 * ks) * lbo_w, lbo_w, 128);
                            const uint64_t xd = sdesc(x_tap + (uint32_t)(2 * ks) * lbo_a, lbo_a, 128);
                            mma_f16(d_tmem, wd, xd, idesc, (b > 0 || k > 0 || ks > 0) ? 1u : 0u);
                        }
                        mma_commit(bW_empty + 8 * sw);
                    }
                    mma_commit(bA_empty + 8 * sa);
                }
                if (ok) mma_commit(bAcc_full + 8 * ab);
            }
            mma_commit(bDrain);
            mbar_wait(bDrain, 0, P.err, 19, TC_DRAIN_NS);
        }
        __syncwarp();
    } else {
        // epilogue warps 2..9: warp w reads TMEM lanes 32 (w % 4) .. (its 32
        // channels) and the position half (w - 2) / 4 of the tile
        const int lq = warp & 3;
        const int ew = warp - 2;
        const int hsel = ew >> 2;
        const bool has_res = P.resid != nullptr;
        uint8_t *blk = sE + ew * 2 * TC_BLK_BYTES;  // STAGED: this warp's two blocks
        const uint32_t bR = bRes + 8 * 2 * ew;
        uint32_t it = 0;
        uint32_t ci = 0, n_res = 0;  // STAGED: blocks done / residual blocks requested
        bool stop = false;
        int64_t tile = blockIdx.x;
        for (; !stop; ++it) {
            if (dyn) {
                const int q = it & 3;
                int64_t tv = -1;
                int okl = 1;
                if (lane == 0) {
                    okl = mbar_wait(bS_full + 8 * q, (it >> 2) & 1, P.err, 24) ? 1 : 0;
                    if (okl) {
                        tv = s_tile[q];
                        mbar_arrive(bS_empty + 8 * q);
                    }
                }
                if (__shfl_sync(0xffffffffu, okl, 0) == 0) break;
                tile = __shfl_sync(0xffffffffu, tv, 0);
                if (tile < 0) break;
            } else if (it > 0) {
                tile += gridDim.x;
            }
            if (tile >= n_tiles_total) break;
            const int64_t mt = tile / P.n_oc_tiles;
            const int n0 = (int)(tile % P.n_oc_tiles) * TC_BN;
            const int ab = it & 1;
            const int c_lo = n0 + 32 * lq;                       // first channel of this warp
            const int64_t pw = mt * TC_BM + hsel * 128;          // first position of this warp
            BlockStats bs;
            float2 prev_part = make_float2(0.f, 0.f);  // the tile's previous block partial
            if (P.part) bs.begin(P, pw);
            if (STAGED && has_res && lane == 0) {
                // the residual of this tile's first block, requested before the
                // accumulator is ready
                bulk_wait_read<0>();
                mbar_expect_tx(bR + 8 * (ci & 1), TC_BLK_BYTES);
                tma_load_2d(smem_u32(blk + (ci & 1) * TC_BLK_BYTES), &rmap, bR + 8 * (ci & 1), (int)pw, c_lo);
                ++n_res;
            }
            int ok_lane = 0;
            if (lane == 0) ok_lane = mbar_wait(bAcc_full + 8 * ab, (it >> 1) & 1, P.err, 15) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok_lane, 0) == 0) break;
            __syncwarp();
            fence_after_sync();
            const int c = c_lo + lane;  // this thread's output channel
            const bool chan_ok = c < P.OC;
            const float bias = (P.bias && chan_ok) ? P.bias[c] : 0.f;
            const float chs = (P.chscale && chan_ok) ? P.chscale[c] : 1.f;
            const uint32_t t_base = tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(ab * TC_BM + hsel * 128);
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t r[32];  // r[j] = D[c][p0 + j]
                tmem_ld32(t_base + (uint32_t)(32 * cc), r);
                const int64_t p0 = pw + 32 * cc;
                if (STAGED) {
                    const int s = ci & 1;
                    uint8_t *buf = blk + s * TC_BLK_BYTES;
                    if (has_res) {
                        if (lane == 0 && cc < 3) {
                            // next block's residual into the other buffer
                            bulk_wait_read<0>();
                            mbar_expect_tx(bR + 8 * (s ^ 1), TC_BLK_BYTES);
                            tma_load_2d(smem_u32(blk + (s ^ 1) * TC_BLK_BYTES), &rmap, bR + 8 * (s ^ 1),
                                        (int)(p0 + 32), c_lo);
                            ++n_res;
                        }
                        // every lane waits: each reader needs its own acquire of
                        // the bytes the copy engine wrote
                        if (!__all_sync(0xffffffffu, mbar_wait(bR + 8 * s, (ci >> 1) & 1, P.err, 20))) {
                            stop = true;
                            break;
                        }
                    } else {
                        if (lane == 0) bulk_wait_read<1>();  // this buffer's previous store has read it
                        __syncwarp();
                    }
                    // row `lane` of the block = channel c: 8 chunks of 4 positions
                    float res[32], old[32];
                    if (has_res) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 t = *reinterpret_cast<const float4 *>(buf + swz128(lane, i));
                            res[4 * i] = t.x, res[4 * i + 1] = t.y, res[4 * i + 2] = t.z, res[4 * i + 3] = t.w;
                        }
                    }
                    if (P.accum && chan_ok && p0 < P.n_pos) {
                        // n_pos == R_out here, a multiple of 128: the block's 32
                        // positions exist and the run is 16-byte aligned
                        const float4 *op = reinterpret_cast<const float4 *>(P.out + (int64_t)c * P.R_out + p0);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 t = op[i];
                            old[4 * i] = t.x, old[4 * i + 1] = t.y, old[4 * i + 2] = t.z, old[4 * i + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) old[j] = 0.f;
                    }
                    float v[32];
                    // element pairs in packed FP32: the same roundings as one op each
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float2 x = make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        // a power of two: exact, contracted or not
                        if (P.acc_scale != 1.0f) x = f2mul(x, make_float2(P.acc_scale, P.acc_scale));
                        if (P.bias) x = f2add(x, make_float2(bias, bias));
                        if (has_res) x = f2add(make_float2(res[j], res[j + 1]), x);
                        // scalar products: a packed product feeding a packed add may be contracted
                        if (P.chscale) x = make_float2(__fmul_rn(x.x, chs), __fmul_rn(x.y, chs));
                        if (P.scale1 != 1.0f) x = make_float2(__fmul_rn(x.x, P.scale1), __fmul_rn(x.y, P.scale1));
                        if (P.accum) x = f2add(make_float2(old[j], old[j + 1]), x);
                        if (P.scale2 != 1.0f) x = make_float2(__fmul_rn(x.x, P.scale2), __fmul_rn(x.y, P.scale2));
                        v[j] = x.x;
                        v[j + 1] = x.y;
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<float4 *>(buf + swz128(lane, i)) =
                            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        // positions past R_out and channels past OC are clipped by the map
                        tma_store_2d(&omap, smem_u32(buf), (int)p0, c_lo);
                        bulk_commit();
                    }
                    ++ci;
                    if (P.part) store_part(P, bs.block(P, v, p0), prev_part, c, chan_ok, p0, cc);
                } else {
                    // memory work only where the channel and rows exist; every
                    // lane reaches the __syncwarp below before the next TMEM load
                    float v[32];
                    if (chan_ok && p0 < P.n_pos) {
                        float *op = P.out + (int64_t)c * P.R_out + p0;
                        // resid_half: the nearest x2 upsample of the residual,
                        // row p / 2 (p0 is even)
                        const int rs = P.resid_half ? 1 : 0;
                        const float *rp = has_res ? P.resid + (int64_t)c * P.R_resid + (p0 >> rs) : nullptr;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            float x = 0.f;
                            if (p0 + j < P.n_pos) {
                                x = __uint_as_float(r[j]);
                                if (P.acc_scale != 1.0f) x = __fmul_rn(x, P.acc_scale);
                                if (P.bias) x = __fadd_rn(x, bias);
                                if (has_res) x = __fadd_rn(rp[j >> rs], x);
                                if (P.chscale) x = __fmul_rn(x, chs);
                                if (P.scale1 != 1.0f) x = __fmul_rn(x, P.scale1);
                                if (P.accum) x = __fadd_rn(op[j], x);
                                if (P.scale2 != 1.0f) x = __fmul_rn(x, P.scale2);
                                op[j] = x;
                            }
                            v[j] = x;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = 0.f;
                    }
                    __syncwarp();
                    if (P.part) store_part(P, bs.block(P, v, p0), prev_part, c, chan_ok, p0, cc);
                }
            }
            if (stop) break;
            fence_before_sync();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bAcc_empty + 8 * ab) : "memory");
        }
        if (STAGED) {
            if (lane == 0) {
                // residual blocks requested but not used (only after an error)
                for (uint32_t i = ci; i < n_res; ++i)
                    mbar_wait(bR + 8 * (i & 1), (i >> 1) & 1, P.err, 21, TC_DRAIN_NS);
                bulk_wait_all();  // every output block written
            }
            __syncwarp();
        }
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
    if (dyn && threadIdx.x == 0) {
        // this CTA's producer asks for no more tiles; the last CTA to get here
        // leaves the counters at zero for the next launch
        __threadfence();
        if (atomicAdd(P.sched + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(P.sched, 0);
            atomicExch(P.sched + 1, 0);
        }
    }
}

// ---------------------------------------------------------------------------
// k_conv_tcf: k_conv_tct with the operand prologue inside. The activation
// slab is formed in shared memory from the F32 input instead of being read
// from a half operand in HBM:
//   warp 0 lane 0   copies F32 pieces [64 channels][32 rows] of x (tensor
//                   map, 128-byte swizzle, rows < 0 or >= R read as zero)
//                   into a ring of TF_NP pieces;
//   warp 2 lane 0   copies the weight tiles;
//   warps 7..14     (transform) turn each piece into half(snake(adain(x)))
//                   with the k_prologue_h arithmetic (one rounding per
//                   operation, packed in FP32 pairs), zero on rows that are
//                   not valid rows of an utterance, and store it into the
//                   K-major slab: warp t owns channels 8t..8t+7 of the 64;
//   warp 1          MMAs as in k_conv_tct;
//   warps 3..6      the staged epilogue of k_conv_tct, each warp over all
//                   256 positions of its 32 channels.
// The slab starts at the tile's first input row rounded down to a multiple
// of 4 (the tensor copy's row coordinate must be 16-byte aligned); the MMA
// start address skips the 0..3 extra rows.
// ---------------------------------------------------------------------------

constexpr int TF_EPI_WARPS = 4;
constexpr int TF_XF_WARPS = 8;
constexpr int TF_XF_WARP0 = 3 + TF_EPI_WARPS;              // first transform warp
constexpr int TF_THREADS = 32 * (TF_XF_WARP0 + TF_XF_WARPS);  // 480
constexpr int TF_NP = 8;                                   // F32 piece stages
constexpr int TF_PIECE_BYTES = 64 * 32 * 4;                // [64 ch][32 rows] F32
constexpr int TF_PIECES = TC_SLAB / 32;                    // pieces per slab
constexpr int TF_NSA = 2;
constexpr int TF_NSW = 3;
constexpr int TF_SMEM = TF_NSA * TC_A_BYTES + TF_NSW * TC_B_BYTES + TF_EPI_WARPS * 2 * TC_BLK_BYTES +
                        TF_NP * TF_PIECE_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
static_assert(TF_SMEM <= 227 * 1024, "shared memory");
static_assert(TC_SLAB % 32 == 0, "slab of whole pieces");

// AdaIN + Snake terms of a channel pair for one utterance (k_prologue_h).
struct XfPrm {
    float2 nmean, scale, nw, nb, g, be, al, ia;  // nmean = -mean
};

__device__ __forceinline__ XfPrm xf_load(const TcParams &P, int u, int c) {
    XfPrm q;
    const float2 m0 = P.x_ms[(int64_t)u * P.IC + c], m1 = P.x_ms[(int64_t)u * P.IC + c + 1];
    q.nmean = make_float2(-m0.x, -m1.x);
    q.scale = make_float2(m0.y, m1.y);
    q.nw = make_float2(P.x_nw[c], P.x_nw[c + 1]);
    q.nb = make_float2(P.x_nb[c], P.x_nb[c + 1]);
    q.g = make_float2(P.x_gamma[(int64_t)u * P.IC + c], P.x_gamma[(int64_t)u * P.IC + c + 1]);
    q.be = make_float2(P.x_beta[(int64_t)u * P.IC + c], P.x_beta[(int64_t)u * P.IC + c + 1]);
    q.al = make_float2(P.x_alpha[c], P.x_alpha[c + 1]);
    q.ia = make_float2(__fdiv_rn(1.0f, q.al.x), __fdiv_rn(1.0f, q.al.y));
    return q;
}


// Packed product a * b rounded once, as fma(a, b, z) with z = -0.0f from a
// kernel parameter: the assembler can neither simplify it back to a multiply
// nor contract it into the add that follows (it does both for a literal
// -0 or a packed mul.rn), so every step keeps its own rounding.
__device__ __forceinline__ float2 f2mul_sep(float2 a, float2 b, float z) {
    float2 r;
    asm("{\n .reg .b64 ra, rb, rz, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mov.b64 rz, {%6, %6};\n fma.rn.f32x2 rd, ra, rb, rz;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(z));
    return r;
}

// x[c][r] of a [64 ch][32 rows] F32 piece in the 128-byte swizzle
__device__ __forceinline__ float xf_piece(const uint8_t *pc, int c, int r) {
    return *reinterpret_cast<const float *>(pc + c * 128 + (((r >> 2) ^ (c & 7)) << 4) + (r & 3) * 4);
}

__device__ __forceinline__ int64_t floor4(int64_t v) { return v - (((v % 4) + 4) % 4); }

// One lane's share of an edge piece: rows 8 i + rr (i = 0..3) of channels
// cl and cl + 1, as half(snake(adain(x))) with the terms q of one utterance,
// written for the rows g with sel_lo <= g < sel_hi: the value where
// lo <= g < hi, else zero. The k_prologue_h expressions with one rounding
// per operation, in packed FP32 pairs; all 32 lanes call this together (one
// warp-wide polynomial test). dst = the slab chunk at the piece's first row
// plus the lane's channel-pair offset.
__device__ __forceinline__ void xf_edge(const uint8_t *pc, uint8_t *dst, int cl, int rr, const XfPrm &q, int64_t g0,
                                        int64_t lo, int64_t hi, int64_t sel_lo, int64_t sel_hi, float z) {
    float2 w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rw = 8 * i + rr;
        const float2 x = make_float2(xf_piece(pc, cl, rw), xf_piece(pc, cl + 1, rw));
        float2 v = f2mul_sep(f2add(x, q.nmean), q.scale, z);
        v = f2add(f2mul_sep(v, q.nw, z), q.nb);
        v = f2add(v, f2mul_sep(v, q.g, z));
        w[i] = f2add(v, q.be);
    }
    float2 t[4];
    bool small = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        t[i] = f2mul_sep(w[i], q.al, z);
        small = small && fabsf(t[i].x) < kSnakeFast && fabsf(t[i].y) < kSnakeFast;
    }
    float2 s2[4];
    if (__all_sync(0xffffffffu, small)) {
        // snake_p in pairs
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 r2 = f2mul_sep(t[i], t[i], z);
            float2 p = f2fma(make_float2(-4.2755596e-06f, -4.2755596e-06f), r2,
                             make_float2(1.4109348e-04f, 1.4109348e-04f));
            p = f2fma(p, r2, make_float2(-3.1746032e-03f, -3.1746032e-03f));
            p = f2fma(p, r2, make_float2(4.4444446e-02f, 4.4444446e-02f));
            p = f2fma(p, r2, make_float2(-3.3333334e-01f, -3.3333334e-01f));
            p = f2fma(p, r2, make_float2(1.0f, 1.0f));
            s2[i] = f2mul_sep(r2, p, z);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) s2[i] = make_float2(snake_sin2(t[i].x), snake_sin2(t[i].y));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t g = g0 + 8 * i + rr;
        const float2 v = f2add(w[i], f2mul_sep(s2[i], q.ia, z));
        const __half2 h = __floats2half2_rn(v.x, v.y);
        const uint32_t hb = *reinterpret_cast<const uint32_t *>(&h);
        if (g >= sel_lo && g < sel_hi)
            *reinterpret_cast<uint32_t *>(dst + (8 * i + rr) * 16) = (g >= lo && g < hi) ? hb : 0u;
    }
}

// One channel's AdaIN + Snake terms as loaded (prefetched a slab ahead)...
struct XfRaw {
    float2 ms;
    float nw, nb, g, be, al;
};
__device__ __forceinline__ XfRaw xf_raw(const TcParams &P, int u, int c) {
    XfRaw r;
    r.ms = P.x_ms[(int64_t)u * P.IC + c];
    r.nw = P.x_nw[c];
    r.nb = P.x_nb[c];
    r.g = P.x_gamma[(int64_t)u * P.IC + c];
    r.be = P.x_beta[(int64_t)u * P.IC + c];
    r.al = P.x_alpha[c];
    return r;
}
// ... and each broadcast to both halves of a pair (nmean = -mean)
struct XfP {
    p2_t nmean, scale, nw, nb, g, be, al, ia;
};
__device__ __forceinline__ XfP xf_bc(const XfRaw &r) {
    XfP q;
    q.nmean = p2_bc(-r.ms.x);
    q.scale = p2_bc(r.ms.y);
    q.nw = p2_bc(r.nw);
    q.nb = p2_bc(r.nb);
    q.g = p2_bc(r.g);
    q.be = p2_bc(r.be);
    q.al = p2_bc(r.al);
    q.ia = p2_bc(__fdiv_rn(1.0f, r.al));
    return q;
}

// A piece whose 32 rows are all valid rows of one utterance: lane = ch +
// 8 q owns channel c (= 8 t + ch of the slab) at rows 8 i + 2 q and the row
// after (i = 0..3), one 8-byte load per pair; the k_prologue_h expressions
// with one rounding per operation; one warp-wide polynomial test for the
// piece (all 32 lanes call this together). dst = the warp's slab chunk at
// the piece's first row.
__device__ __forceinline__ void xf_rows(const uint8_t *pc, uint8_t *dst, int c, int ch, int q, const XfP &p, p2_t z) {
    p2_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 8 * i + 2 * q;
        const p2_t x = *reinterpret_cast<const p2_t *>(pc + c * 128 + (((r >> 2) ^ (c & 7)) << 4) + (r & 3) * 4);
        p2_t v = p2_fma(p2_add(x, p.nmean), p.scale, z);
        v = p2_add(p2_fma(v, p.nw, z), p.nb);
        v = p2_add(v, p2_fma(v, p.g, z));
        w[i] = p2_add(v, p.be);
    }
    p2_t t[4];
    bool small = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        t[i] = p2_fma(w[i], p.al, z);
        const float2 tf = p2_unpack(t[i]);
        small = small && fabsf(tf.x) < kSnakeFast && fabsf(tf.y) < kSnakeFast;
    }
    p2_t s2[4];
    if (__all_sync(0xffffffffu, small)) {
        // snake_p in pairs
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const p2_t r2 = p2_fma(t[i], t[i], z);
            p2_t pp = p2_fma(p2_bc(-4.2755596e-06f), r2, p2_bc(1.4109348e-04f));
            pp = p2_fma(pp, r2, p2_bc(-3.1746032e-03f));
            pp = p2_fma(pp, r2, p2_bc(4.4444446e-02f));
            pp = p2_fma(pp, r2, p2_bc(-3.3333334e-01f));
            pp = p2_fma(pp, r2, p2_bc(1.0f));
            s2[i] = p2_fma(r2, pp, z);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 tf = p2_unpack(t[i]);
            s2[i] = p2_pack(snake_sin2(tf.x), snake_sin2(tf.y));
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = p2_unpack(p2_add(w[i], p2_fma(s2[i], p.ia, z)));
        const int r = 8 * i + 2 * q;
        *reinterpret_cast<__half *>(dst + r * 16 + ch * 2) = __float2half_rn(v.x);
        *reinterpret_cast<__half *>(dst + (r + 1) * 16 + ch * 2) = __float2half_rn(v.y);
    }
}

__global__ void __launch_bounds__(TF_THREADS, 1)
    k_conv_tcf(const __grid_constant__ TcParams P, const __grid_constant__ CUtensorMap omap,
               const __grid_constant__ CUtensorMap rmap, const __grid_constant__ CUtensorMap xmap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;                                   // half slabs
    uint8_t *sW = sA + TF_NSA * TC_A_BYTES;               // weight tiles
    uint8_t *sE = sW + TF_NSW * TC_B_BYTES;               // epilogue blocks, two per warp
    uint8_t *sF = sE + TF_EPI_WARPS * 2 * TC_BLK_BYTES;   // F32 pieces (1 KB aligned)
    uint64_t *bars = (uint64_t *)(sF + TF_NP * TF_PIECE_BYTES);
    // F_full[NP] F_empty[NP] A_full[NSA] A_empty[NSA] W_full[NSW] W_empty[NSW]
    // acc_full[2] acc_empty[2] drain res[4 warps][2] tmem-slot
    const uint32_t bF_full = smem_u32(bars), bF_empty = smem_u32(bars + TF_NP);
    const uint32_t bA_full = smem_u32(bars + 2 * TF_NP), bA_empty = smem_u32(bars + 2 * TF_NP + TF_NSA);
    const uint32_t bW_full = smem_u32(bars + 2 * TF_NP + 2 * TF_NSA);
    const uint32_t bW_empty = smem_u32(bars + 2 * TF_NP + 2 * TF_NSA + TF_NSW);
    const uint32_t bAcc_full = smem_u32(bars + 2 * TF_NP + 2 * TF_NSA + 2 * TF_NSW);
    const uint32_t bAcc_empty = bAcc_full + 16;
    const uint32_t bDrain = bAcc_full + 32;
    const uint32_t bRes = bAcc_full + 40;
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * TF_NP + 2 * TF_NSA + 2 * TF_NSW + 5 + 2 * TF_EPI_WARPS);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_tiles_total = P.m_tiles * P.n_oc_tiles;
    const int IC_blocks = P.IC / 64;

    if (threadIdx.x == 0) {
        for (int i = 0; i < TF_NP; ++i) {
            mbar_init(bF_full + 8 * i, 1);
            mbar_init(bF_empty + 8 * i, TF_XF_WARPS);
        }
        for (int i = 0; i < TF_NSA; ++i) {
            mbar_init(bA_full + 8 * i, TF_XF_WARPS);
            mbar_init(bA_empty + 8 * i, 1);
        }
        for (int i = 0; i < TF_NSW; ++i) {
            mbar_init(bW_full + 8 * i, 1);
            mbar_init(bW_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bAcc_full + 8 * i, 1);
            mbar_init(bAcc_empty + 8 * i, TF_EPI_WARPS);
        }
        mbar_init(bDrain, 1);
        for (int i = 0; i < 2 * TF_EPI_WARPS; ++i) mbar_init(bRes + 8 * i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    constexpr uint32_t lbo_a = (uint32_t)TC_SLAB * 16u;  // activation chunk stride
    constexpr uint32_t lbo_w = (uint32_t)TC_BN * 16u;    // weight chunk stride

    if (warp == 0) {
        if (lane == 0) {
            // F32 pieces of x
            bool ok = true;
            uint32_t ip = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
                const int64_t mt = tile / P.n_oc_tiles;
                const int64_t r0a = floor4(mt * TC_BM - P.p);
                for (int b = 0; b < IC_blocks && ok; ++b) {
                    for (int j = 0; j < TF_PIECES; ++j, ++ip) {
                        const int sp = ip % TF_NP;
                        if (ip >= TF_NP) ok = mbar_wait(bF_empty + 8 * sp, ((ip / TF_NP) & 1) ^ 1, P.err, 31);
                        if (!ok) break;
                        mbar_expect_tx(bF_full + 8 * sp, TF_PIECE_BYTES);
                        tma_load_2d(smem_u32(sF + sp * TF_PIECE_BYTES), &xmap, bF_full + 8 * sp, (int)(r0a + 32 * j),
                                    64 * b);
                    }
                }
            }
            for (uint32_t i = (ip > TF_NP ? ip - TF_NP : 0); i < ip; ++i)
                mbar_wait(bF_full + 8 * (i % TF_NP), (i / TF_NP) & 1, P.err, 38, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == 2) {
        if (lane == 0) {
            // weight tiles
            bool ok = true;
            uint32_t iw = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
                const int nt = (int)(tile % P.n_oc_tiles);
                for (int b = 0; b < IC_blocks && ok; ++b) {
                    for (int k = 0; k < P.K; ++k, ++iw) {
                        const int sw = iw % TF_NSW;
                        if (iw >= TF_NSW) ok = mbar_wait(bW_empty + 8 * sw, ((iw / TF_NSW) & 1) ^ 1, P.err, 32);
                        if (!ok) break;
                        mbar_expect_tx(bW_full + 8 * sw, TC_B_BYTES);
                        const __half *src =
                            P.w + ((((size_t)k * IC_blocks + b) * P.n_tiles + nt) * (size_t)(8 * TC_BN * 8));
                        bulk_load(smem_u32(sW + sw * TC_B_BYTES), src, TC_B_BYTES, bW_full + 8 * sw);
                    }
                }
            }
            for (uint32_t i = (iw > TF_NSW ? iw - TF_NSW : 0); i < iw; ++i)
                mbar_wait(bW_full + 8 * (i % TF_NSW), (i / TF_NSW) & 1, P.err, 38, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: A = weights (M = 128 channels), B = the formed slab (N = 256 positions)
            const uint32_t idesc = idesc_f16(TC_BN, TC_BM);
            bool ok = true;
            uint32_t ia = 0, iw = 0, it = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x, ++it) {
                const int64_t mt = tile / P.n_oc_tiles;
                const int64_t row0 = mt * TC_BM - P.p;
                const uint32_t shift = (uint32_t)(row0 - floor4(row0));  // 0..3 rows
                const int ab = it & 1;
                if (it >= 2) ok = mbar_wait(bAcc_empty + 8 * ab, ((it >> 1) & 1) ^ 1, P.err, 37);
                if (!ok) break;
                fence_after_sync();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * TC_BM);
                for (int b = 0; b < IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % TF_NSA;
                    ok = mbar_wait(bA_full + 8 * sa, (ia / TF_NSA) & 1, P.err, 33);
                    if (!ok) break;
                    fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + sa * TC_A_BYTES);
                    for (int k = 0; k < P.K; ++k, ++iw) {
                        const int sw = iw % TF_NSW;
                        ok = mbar_wait(bW_full + 8 * sw, (iw / TF_NSW) & 1, P.err, 34);
                        if (!ok) break;
                        fence_after_sync();
                        const uint32_t w_base = smem_u32(sW + sw * TC_B_BYTES);
                        const uint32_t x_tap = a_base + (shift + (uint32_t)(k * P.d)) * 16u;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t wd = sdesc(w_base + (uint32_t)(2 * ks) * lbo_w, lbo_w, 128);
                            const uint64_t xd = sdesc(x_tap + (uint32_t)(2 * ks) * lbo_a, lbo_a, 128);
                            mma_f16(d_tmem, wd, xd, idesc, (b > 0 || k > 0 || ks > 0) ? 1u : 0u);
                        }
                        mma_commit(bW_empty + 8 * sw);
                    }
                    mma_commit(bA_empty + 8 * sa);
                }
                if (ok) mma_commit(bAcc_full + 8 * ab);
            }
            mma_commit(bDrain);
            mbar_wait(bDrain, 0, P.err, 39, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp < TF_XF_WARP0) {
        // epilogue warps 3..6: warp w reads TMEM lanes 32 (w % 4) .. (its 32
        // channels) over all 256 positions of the tile
        const int lq = warp & 3;
        const int ew = warp - 3;
        const bool has_res = P.resid != nullptr;
        uint8_t *blk = sE + ew * 2 * TC_BLK_BYTES;
        const uint32_t bR = bRes + 8 * 2 * ew;
        uint32_t it = 0;
        uint32_t ci = 0, n_res = 0;  // blocks done / residual blocks requested
        bool stop = false;
        for (int64_t tile = blockIdx.x; tile < n_tiles_total && !stop; tile += gridDim.x, ++it) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int n0 = (int)(tile % P.n_oc_tiles) * TC_BN;
            const int ab = it & 1;
            const int c_lo = n0 + 32 * lq;
            const int64_t pw = mt * TC_BM;
            BlockStats bs;
            float2 prev_part = make_float2(0.f, 0.f);
            if (P.part) bs.begin(P, pw);
            if (has_res && lane == 0) {
                bulk_wait_read<0>();
                mbar_expect_tx(bR + 8 * (ci & 1), TC_BLK_BYTES);
                tma_load_2d(smem_u32(blk + (ci & 1) * TC_BLK_BYTES), &rmap, bR + 8 * (ci & 1), (int)pw, c_lo);
                ++n_res;
            }
            int ok_lane = 0;
            if (lane == 0) ok_lane = mbar_wait(bAcc_full + 8 * ab, (it >> 1) & 1, P.err, 35) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok_lane, 0) == 0) break;
            __syncwarp();
            fence_after_sync();
            const int c = c_lo + lane;
            const bool chan_ok = c < P.OC;
            const float bias = (P.bias && chan_ok) ? P.bias[c] : 0.f;
            const uint32_t t_base = tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(ab * TC_BM);
            for (int cc = 0; cc < 8; ++cc) {
                float v[32];  // the accumulator, then the output, in place
                tmem_ld32f(t_base + (uint32_t)(32 * cc), v);
                const int64_t p0 = pw + 32 * cc;
                const int s = ci & 1;
                uint8_t *buf = blk + s * TC_BLK_BYTES;
                if (has_res) {
                    if (lane == 0 && cc < 7) {
                        bulk_wait_read<0>();
                        mbar_expect_tx(bR + 8 * (s ^ 1), TC_BLK_BYTES);
                        tma_load_2d(smem_u32(blk + (s ^ 1) * TC_BLK_BYTES), &rmap, bR + 8 * (s ^ 1), (int)(p0 + 32),
                                    c_lo);
                        ++n_res;
                    }
                    if (!__all_sync(0xffffffffu, mbar_wait(bR + 8 * s, (ci >> 1) & 1, P.err, 36))) {
                        stop = true;
                        break;
                    }
                } else {
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float2 x0 = make_float2(v[4 * i], v[4 * i + 1]);
                    float2 x1 = make_float2(v[4 * i + 2], v[4 * i + 3]);
                    if (P.bias) {
                        x0 = f2add(x0, make_float2(bias, bias));
                        x1 = f2add(x1, make_float2(bias, bias));
                    }
                    if (has_res) {
                        const float4 t = *reinterpret_cast<const float4 *>(buf + swz128(lane, i));
                        x0 = f2add(make_float2(t.x, t.y), x0);
                        x1 = f2add(make_float2(t.z, t.w), x1);
                    }
                    v[4 * i] = x0.x, v[4 * i + 1] = x0.y, v[4 * i + 2] = x1.x, v[4 * i + 3] = x1.y;
                    *reinterpret_cast<float4 *>(buf + swz128(lane, i)) = make_float4(x0.x, x0.y, x1.x, x1.y);
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&omap, smem_u32(buf), (int)p0, c_lo);
                    bulk_commit();
                }
                ++ci;
                if (P.part) store_part(P, bs.block(P, v, p0), prev_part, c, chan_ok, p0, cc);
            }
            if (stop) break;
            fence_before_sync();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bAcc_empty + 8 * ab) : "memory");
        }
        if (lane == 0) {
            for (uint32_t i = ci; i < n_res; ++i) mbar_wait(bR + 8 * (i & 1), (i >> 1) & 1, P.err, 40, TC_DRAIN_NS);
            bulk_wait_all();
        }
        __syncwarp();
    } else {
        // transform warps: warp t forms channels 8t..8t+7 of each 64-channel
        // slab. Whole-utterance pieces: lane = ch + 8 q (xf_rows); pieces at
        // utterance edges: lane = (row rr = lane / 4, channel pair cp = lane
        // % 4) (xf_edge). The next slab's terms are loaded while this one is
        // formed.
        const int tw = warp - TF_XF_WARP0;  // channel chunk
        const int rr = lane >> 2, cp = lane & 3;
        const int ch = lane & 7, q8 = lane >> 3;
        const int cl = 8 * tw + 2 * cp;  // edge pieces: the lane's first channel within the slab
        const int c1 = 8 * tw + ch;      // whole pieces: the lane's channel within the slab
        uint32_t ip = 0, is = 0;
        bool ok = true;
        int64_t tile = blockIdx.x;
        int b = 0;
        int u_cur = 0;
        XfRaw raw_cur{};
        if (tile < n_tiles_total) {
            const int64_t r0 = floor4((tile / P.n_oc_tiles) * TC_BM - P.p);
            u_cur = utt_of_row(P.sb, P.sm, r0 > 0 ? r0 : 0);
            raw_cur = xf_raw(P, u_cur, c1);
        }
        while (tile < n_tiles_total && ok) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int64_t r0a = floor4(mt * TC_BM - P.p);
            // the slab after this one, and its terms
            int64_t tile_n = tile;
            int b_n = b + 1;
            if (b_n == IC_blocks) {
                b_n = 0;
                tile_n += gridDim.x;
            }
            int u_next = 0;
            XfRaw raw_next{};
            if (tile_n < n_tiles_total) {
                const int64_t r0n = floor4((tile_n / P.n_oc_tiles) * TC_BM - P.p);
                u_next = utt_of_row(P.sb, P.sm, r0n > 0 ? r0n : 0);
                raw_next = xf_raw(P, u_next, 64 * b_n + c1);
            }
            const int sa = is % TF_NSA;
            if (is >= TF_NSA) {
                int okl = 1;
                if (lane == 0) okl = mbar_wait(bA_empty + 8 * sa, ((is / TF_NSA) & 1) ^ 1, P.err, 41) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
                if (!ok) break;
            }
            const int cg = 64 * b + cl;  // edge pieces: global channel
            int u = u_cur;
            int64_t lo = (int64_t)P.sm * __ldg(P.sb.offT + u);
            int64_t hi = lo + (int64_t)P.sm * __ldg(P.sb.T + u) + P.sextra;
            int64_t lo_n = u + 1 < P.sb.n ? (int64_t)P.sm * __ldg(P.sb.offT + u + 1) : INT64_MAX;
            XfP pf = xf_bc(raw_cur);
            uint8_t *slab = sA + sa * TC_A_BYTES + tw * lbo_a;
            for (int j = 0; j < TF_PIECES; ++j, ++ip) {
                const int sp = ip % TF_NP;
                // every lane acquires the bytes the copy wrote
                if (!__all_sync(0xffffffffu, mbar_wait(bF_full + 8 * sp, (ip / TF_NP) & 1, P.err, 42))) {
                    ok = false;
                    break;
                }
                const int64_t g0 = r0a + 32 * j;
                for (int guard = 0; guard < P.sb.n && g0 >= lo_n; ++guard) {
                    ++u;
                    lo = lo_n;
                    hi = lo + (int64_t)P.sm * __ldg(P.sb.T + u) + P.sextra;
                    lo_n = u + 1 < P.sb.n ? (int64_t)P.sm * __ldg(P.sb.offT + u + 1) : INT64_MAX;
                    pf = xf_bc(xf_raw(P, u, 64 * b + c1));
                }
                const uint8_t *pc = sF + sp * TF_PIECE_BYTES;
                if (g0 >= lo && g0 + 32 <= hi) {
                    xf_rows(pc, slab + 32 * j * 16, c1, ch, q8, pf, P.nz2);
                } else {
                    // gap rows, an utterance's end, or the next one's start
                    // (rows of this utterance's slot, then the next one's)
                    uint8_t *dst = slab + 32 * j * 16 + cp * 4;
                    xf_edge(pc, dst, cl, rr, xf_load(P, u, cg), g0, lo, hi, INT64_MIN, lo_n, P.nz);
                    if (lo_n < g0 + 32) {
                        const int64_t hi_n = lo_n + (int64_t)P.sm * __ldg(P.sb.T + u + 1) + P.sextra;
                        xf_edge(pc, dst, cl, rr, xf_load(P, u + 1, cg), g0, lo_n, hi_n, lo_n, INT64_MAX, P.nz);
                    }
                }
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bF_empty + 8 * sp) : "memory");
            }
            if (!ok) break;
            // the slab's generic stores, visible to the tensor cores
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bA_full + 8 * sa) : "memory");
            ++is;
            raw_cur = raw_next;
            u_cur = u_next;
            tile = tile_n;
            b = b_n;
        }
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// kernel, transposed convolution with row-contiguous output
// ---------------------------------------------------------------------------
//
// ConvTranspose1d with stride S as S phase convolutions of 2 taps over the
// input (phase r writes output rows S q + oadd + r), all S phases of NC
// channels in one tile: D[q][r NC + c] = one M = 128 positions x N = S NC MMA
// per 16-channel step, the activation slab as operand A and the phase-major
// weight rows as operand B. The S phases of a position are adjacent output
// rows, so an epilogue warp (32 positions, NC / 2 channels) holds, per
// channel, the 32 S consecutive output rows [S q0 + oadd, S q0 + oadd + 32 S)
// of its positions. The residual of those rows arrives by bulk copies (a
// 16-byte aligned superset of the run) in a shared run buffer, the
// accumulator and bias are added into it in row order, and the run is
// written out as whole 128-byte stores, where the per-phase register
// epilogue of k_conv_tc writes every S-th float (partial L2 sectors).
//
// With two taps the MMA work per tile is small and the tile pipeline sets
// the pace: at batch 64 the stride-6 upsampler took 0.52 ms with no MMA and
// no stores (operand copies and the epilogue's TMEM reads and run staging
// alone), 0.79 ms complete. Where the weights of one channel group fit in
// shared memory next to the slabs (stride 6: NC = 16, N = 96, 2 taps x 256
// channels = 96 KB) they stay resident: the grid is a multiple of the
// channel groups, so every tile of a CTA has the same group and only the
// slabs stream. More epilogue warps (16: more runs in flight) took it from
// 0.80 to 0.73 ms; an L2 prefetch of the residual two tiles ahead made it
// slower (0.88 ms).
//
// Roles (64 + 32 EW threads): warp 0 lane 0 copies, warp 1 lane 0 issues the
// MMAs into two accumulators of up to 256 columns, warps 2 .. EW + 1 run the
// epilogue, EW / 4 of them per TMEM lane group (warp w: lanes 32 (w % 4) ..,
// channel part (w - 2) / 4 of the tile).
constexpr int CT_BM = 128;                          // positions per tile
constexpr int CT_SLAB = 136;                        // slab rows: 128 + the taps' halo, rounded to 8
constexpr int CT_A_BYTES = 8 * CT_SLAB * 16;        // 17 KB

// One instance: S phases, NC channels per phase in a tile (MMA N = S NC), G
// channels per epilogue pass, NRB run buffers per epilogue warp (2: the next
// pass's residual lands while this one is written out; 1: after it), RES:
// resident weights (at most CT_RES_TILES (tap, 64-channel block) tiles),
// else NSW streamed weight stages; EW epilogue warps.
constexpr int CT_RES_TILES = 8;
template <int S_, int NC_, int G_, int NRB_, bool RES_, int NSA_, int NSW_, int EW_>
struct CtCfg {
    static constexpr int S = S_, NC = NC_, G = G_, NRB = NRB_, NSA = NSA_, NSW = NSW_, EW = EW_;
    static constexpr bool RES = RES_;
    static constexpr int N = S * NC;
    static constexpr int NCW = NC / (EW / 4);  // channels of one epilogue warp
    static constexpr int THREADS = 64 + 32 * EW;
    static constexpr int BX = 32 * S + 4;  // rows of a run buffer: a run and its 16-byte alignment
    static constexpr int RUN = G * BX;     // floats per run buffer
    static constexpr int W_TILE = N * 128;
    static constexpr int W_SLOTS = RES ? CT_RES_TILES : NSW;
    static constexpr int SMEM = NSA * CT_A_BYTES + W_SLOTS * W_TILE + EW * NRB * RUN * 4 + 1024 /*barriers*/ +
                                1024 /*align*/;
    static_assert(S % 2 == 0 && G * S <= 48 && EW % 4 == 0 && NC % (EW / 4) == 0 && NCW % G == 0 && N % 16 == 0 &&
                      N <= 256,
                  "shape");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};
using CtCfg6 = CtCfg<6, 16, 4, 1, true, 3, 0, 16>;    // stride 6, weights resident: N = 96
using CtCfg6s = CtCfg<6, 16, 4, 2, false, 2, 4, 16>;   // stride 6, streamed (split F32: 3x the blocks)
using CtCfg10 = CtCfg<10, 16, 4, 2, false, 2, 4, 8>;  // stride 10 (256 x 512 weights): N = 160, streamed

// tcgen05.ld 32x32b of N consecutive columns, without the wait
template <int N>
__device__ __forceinline__ void tmem_ld_nowait(uint32_t taddr, float (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld_nowait<4>(uint32_t taddr, float (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld_nowait<8>(uint32_t taddr, float (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) k_convt_tc(const __grid_constant__ TcParams P) {
    constexpr int S = C::S, NC = C::NC, N = C::N, G = C::G, BX = C::BX, NRB = C::NRB;
    constexpr int NSA = C::NSA, NWB = C::RES ? 1 : C::NSW;  // weight barriers
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;
    uint8_t *sW = sA + NSA * CT_A_BYTES;
    float *sE = (float *)(sW + C::W_SLOTS * C::W_TILE);
    uint64_t *bars = (uint64_t *)(sE + C::EW * NRB * C::RUN);
    // A_full[NSA] A_empty[NSA] W_full[NWB] W_empty[NWB] acc_full[2] acc_empty[2] drain
    // res[EW warps][NRB] tmem-slot
    const uint32_t bA_full = smem_u32(bars), bA_empty = smem_u32(bars + NSA);
    const uint32_t bW_full = smem_u32(bars + 2 * NSA), bW_empty = smem_u32(bars + 2 * NSA + NWB);
    const uint32_t bAcc_full = smem_u32(bars + 2 * NSA + 2 * NWB);
    const uint32_t bAcc_empty = smem_u32(bars + 2 * NSA + 2 * NWB + 2);
    const uint32_t bDrain = smem_u32(bars + 2 * NSA + 2 * NWB + 4);
    const uint32_t bRes = smem_u32(bars + 2 * NSA + 2 * NWB + 5);
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * NSA + 2 * NWB + 5 + NRB * C::EW);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_tiles_total = P.m_tiles * P.n_oc_tiles;
    const int n_wt = P.K * P.IC_blocks;  // weight tiles of a channel group

    if (threadIdx.x == 0) {
        for (int i = 0; i < NSA; ++i) {
            mbar_init(bA_full + 8 * i, 1);
            mbar_init(bA_empty + 8 * i, 1);
        }
        for (int i = 0; i < NWB; ++i) {
            mbar_init(bW_full + 8 * i, 1);
            mbar_init(bW_empty + 8 * i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(bAcc_full + 8 * i, 1);
            mbar_init(bAcc_empty + 8 * i, C::EW);
        }
        mbar_init(bDrain, 1);
        for (int i = 0; i < NRB * C::EW; ++i) mbar_init(bRes + 8 * i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    constexpr uint32_t lbo_a = (uint32_t)CT_SLAB * 16u;  // slab chunk stride
    constexpr uint32_t lbo_w = (uint32_t)N * 16u;        // weight chunk stride
    constexpr uint32_t w_bytes = (uint32_t)C::W_TILE;    // one weight tile
    // packed weight tile (tap k, block b) of channel group nt
    auto w_src = [&](int k, int b, int nt) {
        return P.w + (((size_t)k * P.IC_blocks + b) * P.n_tiles + nt) * (size_t)N * 64;
    };

    if (warp == 0) {
        if (lane == 0) {
            // producer
            bool ok = true;
            uint32_t ia = 0, iw = 0;
            if (C::RES && (int64_t)blockIdx.x < n_tiles_total) {
                // every tile of this CTA has channel group blockIdx.x % n_oc_tiles
                const int nt = (int)(blockIdx.x % P.n_oc_tiles);
                mbar_expect_tx(bW_full, w_bytes * (uint32_t)n_wt);
                for (int b = 0; b < P.IC_blocks; ++b)
                    for (int k = 0; k < P.K; ++k)
                        bulk_load(smem_u32(sW + (b * P.K + k) * C::W_TILE), w_src(k, b, nt), w_bytes, bW_full);
                iw = 1;
            }
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
                const int64_t mt = tile / P.n_oc_tiles;
                const int nt = (int)(tile % P.n_oc_tiles);
                const int64_t row0 = mt * CT_BM - P.p;  // >= -kHalfLo (checked on the host)
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % NSA;
                    if (ia >= NSA) ok = mbar_wait(bA_empty + 8 * sa, ((ia / NSA) & 1) ^ 1, P.err, 11);
                    if (!ok) break;
                    mbar_expect_tx(bA_full + 8 * sa, CT_A_BYTES);
                    const uint32_t dst = smem_u32(sA + sa * CT_A_BYTES);
                    const int bo = (P.a_wrap > 0 && b >= P.a_wrap) ? b - P.a_wrap : b;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const __half *src = P.a + ((int64_t)(8 * bo + c) * P.R_a + row0) * 8;
                        bulk_load(dst + (uint32_t)c * lbo_a, src, lbo_a, bA_full + 8 * sa);
                    }
                    if (!C::RES) {
                        for (int k = 0; k < P.K; ++k, ++iw) {
                            const int sw = iw % NWB;
                            if (iw >= NWB) ok = mbar_wait(bW_empty + 8 * sw, ((iw / NWB) & 1) ^ 1, P.err, 12);
                            if (!ok) break;
                            mbar_expect_tx(bW_full + 8 * sw, w_bytes);
                            bulk_load(smem_u32(sW + sw * C::W_TILE), w_src(k, b, nt), w_bytes, bW_full + 8 * sw);
                        }
                    }
                }
            }
            for (uint32_t i = (ia > NSA ? ia - NSA : 0); i < ia; ++i)
                mbar_wait(bA_full + 8 * (i % NSA), (i / NSA) & 1, P.err, 18, TC_DRAIN_NS);
            for (uint32_t i = (iw > NWB ? iw - NWB : 0); i < iw; ++i)
                mbar_wait(bW_full + 8 * (i % NWB), (i / NWB) & 1, P.err, 18, TC_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: A = activations (M = 128 positions), B = weights (N = S NC phase rows)
            const uint32_t idesc = idesc_f16(CT_BM, N);
            bool ok = true;
            uint32_t ia = 0, iw = 0, it = 0;
            if (C::RES && (int64_t)blockIdx.x < n_tiles_total) ok = mbar_wait(bW_full, 0, P.err, 14);
            for (int64_t tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x, ++it) {
                const int ab = it & 1;
                if (it >= 2) ok = mbar_wait(bAcc_empty + 8 * ab, ((it >> 1) & 1) ^ 1, P.err, 17);
                if (!ok) break;
                fence_after_sync();
                const uint32_t d_tmem = tmem + (uint32_t)(ab * 256);
                for (int b = 0; b < P.IC_blocks && ok; ++b, ++ia) {
                    const int sa = ia % NSA;
                    ok = mbar_wait(bA_full + 8 * sa, (ia / NSA) & 1, P.err, 13);
                    if (!ok) break;
                    fence_after_sync();
                    const uint32_t a_base = smem_u32(sA + sa * CT_A_BYTES);
                    for (int k = 0; k < P.K; ++k) {
                        uint32_t w_base;
                        int sw = 0;
                        if (C::RES) {
                            w_base = smem_u32(sW + (b * P.K + k) * C::W_TILE);
                        } else {
                            sw = iw % NWB;
                            ok = mbar_wait(bW_full + 8 * sw, (iw / NWB) & 1, P.err, 14);
                            if (!ok) break;
                            fence_after_sync();
                            w_base = smem_u32(sW + sw * C::W_TILE);
                        }
                        const uint32_t a_tap = a_base + (uint32_t)(k * P.d) * 16u;
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t ad = sdesc(a_tap + (uint32_t)(2 * ks) * lbo_a, lbo_a, 128);
                            const uint64_t wd = sdesc(w_base + (uint32_t)(2 * ks) * lbo_w, lbo_w, 128);
                            mma_f16(d_tmem, ad, wd, idesc, (b > 0 || k > 0 || ks > 0) ? 1u : 0u);
                        }
                        if (!C::RES) {
                            mma_commit(bW_empty + 8 * sw);
                            ++iw;
                        }
                    }
                    mma_commit(bA_empty + 8 * sa);
                }
                if (ok) mma_commit(bAcc_full + 8 * ab);
            }
            mma_commit(bDrain);
            mbar_wait(bDrain, 0, P.err, 19, TC_DRAIN_NS);
        }
        __syncwarp();
    } else {
        // epilogue warps 2 .. EW + 1
        const int lg = warp & 3;            // TMEM lane group: positions 32 lg .. of the tile
        const int hsel = (warp - 2) >> 2;   // channel part of the tile
        constexpr int ncw = C::NCW;         // channels of this warp
        constexpr int n_pass = ncw / G;
        const int ew = warp - 2;
        // NRB run buffers [G][BX]; a run of 32 S output rows starts d0 < 4
        // floats into its buffer, at the 16-byte boundary below it. Item n
        // (a tile's pass) uses buffer n % NRB.
        float *runs = sE + ew * NRB * C::RUN;
        const uint32_t bR = bRes + 8 * NRB * ew;  // their barriers
        const bool has_res = P.resid != nullptr;
        // lane 0: the residual of item (tile, pass g) into buffer s: channels
        // c_lo + g G + j, rows [x0, x0 + BX) clipped to [0, R_resid) (the
        // clipped rows are no output rows of the run), one bulk copy each
        uint32_t n_issued = 0;
        auto fetch = [&](int64_t tile, int g, int s) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int nt = (int)(tile % P.n_oc_tiles);
            const int64_t x0 = ((mt * CT_BM + 32 * lg) * S + P.oadd) & ~(int64_t)3;
            const int64_t lo = x0 > 0 ? x0 : 0;
            const int64_t hi = x0 + BX < P.R_resid ? x0 + BX : P.R_resid;
            const uint32_t bytes = hi > lo ? (uint32_t)(hi - lo) * 4u : 0u;
            fence_proxy_async();  // this buffer's earlier reads and writes come first
            mbar_expect_tx(bR + 8 * s, bytes * G);
            if (bytes) {
                const int c0 = nt * NC + hsel * ncw + g * G;
                const uint32_t dst = smem_u32(runs + s * C::RUN + (lo - x0));
                for (int j = 0; j < G; ++j)
                    bulk_load(dst + (uint32_t)(j * BX * 4), P.resid + (int64_t)(c0 + j) * P.R_resid + lo, bytes,
                              bR + 8 * s);
            }
            ++n_issued;
        };
        // lane 0: the residual of the item after (tile, g) into buffer s
        auto fetch_next = [&](int64_t tile, int g, int s) {
            if (g + 1 < n_pass)
                fetch(tile, g + 1, s);
            else if (tile + gridDim.x < n_tiles_total)
                fetch(tile + gridDim.x, 0, s);
        };
        if (has_res && lane == 0 && (int64_t)blockIdx.x < n_tiles_total) fetch(blockIdx.x, 0, 0);
        uint32_t it = 0, n = 0;  // tiles and items (tile, pass) done
        bool stop = false;
        for (int64_t tile = blockIdx.x; tile < n_tiles_total && !stop; tile += gridDim.x, ++it) {
            const int64_t mt = tile / P.n_oc_tiles;
            const int nt = (int)(tile % P.n_oc_tiles);
            const int ab = it & 1;
            const int64_t pw = mt * CT_BM + 32 * lg;  // first position of this warp
            const int64_t orow0 = pw * S + P.oadd;    // its first output row
            const int d0 = (int)(orow0 - (orow0 & ~(int64_t)3));
            const int c_lo = nt * NC + hsel * ncw;    // its first output channel
            int ok_lane = 0;
            if (lane == 0) ok_lane = mbar_wait(bAcc_full + 8 * ab, (it >> 1) & 1, P.err, 15) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok_lane, 0) == 0) break;
            __syncwarp();
            fence_after_sync();
            // row lane + 32 k of the run: position pw + (lane + 32 k) / S, phase (lane + 32 k) % S
            bool row_ok[S];
#pragma unroll
            for (int k = 0; k < S; ++k) {
                const int i = lane + 32 * k;
                const int64_t o = orow0 + i;
                row_ok[k] = pw + i / S < P.n_pos && o >= 0 && o < P.R_out;
            }
            const uint32_t t_base = tmem + ((uint32_t)(32 * lg) << 16) + (uint32_t)(ab * 256 + hsel * ncw);
            for (int g = 0; g < n_pass; ++g, ++n) {
                const int s = (int)(n % NRB);
                float *run = runs + s * C::RUN + d0;
                // with two buffers, the next item's residual into the other
                // one (its reads ended at the previous item's last __syncwarp)
                if (NRB == 2 && has_res && lane == 0) fetch_next(tile, g, s ^ 1);
                float v[S][G];  // v[r][j] = D[position pw + lane][phase r, channel c_lo + g G + j]
#pragma unroll
                for (int r = 0; r < S; ++r) tmem_ld_nowait<G>(t_base + (uint32_t)(r * NC + g * G), v[r]);
                tmem_ld_wait();
                if (g == n_pass - 1) {
                    // the tile's accumulator values are all in registers: hand it back
                    fence_before_sync();
                    __syncwarp();
                    if (lane == 0)
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bAcc_empty + 8 * ab) : "memory");
                }
                // every lane waits: each reader needs its own acquire of the
                // bytes the copies wrote
                if (has_res && !__all_sync(0xffffffffu, mbar_wait(bR + 8 * s, (n / NRB) & 1, P.err, 20))) {
                    stop = true;
                    break;
                }
                // accumulator (+ bias) into the run, row S lane + r of channel
                // j: residual + value, or the value alone
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    const float bj = P.bias ? __ldg(P.bias + c_lo + g * G + j) : 0.f;
                    float *rj = run + j * BX + S * lane;
#pragma unroll
                    for (int r = 0; r < S; ++r) {
                        float x = v[r][j];
                        if (P.acc_scale != 1.0f) x = __fmul_rn(x, P.acc_scale);
                        if (P.bias) x = __fadd_rn(x, bj);
                        rj[r] = has_res ? __fadd_rn(rj[r], x) : x;
                    }
                }
                __syncwarp();
                // whole 128-byte runs of each channel's output row
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    float *op = P.out + (int64_t)(c_lo + g * G + j) * P.R_out + orow0 + lane;
                    const float *rj = run + j * BX + lane;
#pragma unroll
                    for (int k = 0; k < S; ++k)
                        if (row_ok[k]) op[32 * k] = rj[32 * k];
                }
                __syncwarp();  // the run is read before this buffer's next copy or write
                // with one buffer, the next item's residual into it now
                if (NRB == 1 && has_res && lane == 0) fetch_next(tile, g, s);
            }
        }
        // a copy issued for an item that never ran (a wait that ran out) lands
        // before the CTA ends
        if (has_res && lane == 0)
            for (uint32_t i = n; i < n_issued; ++i)
                mbar_wait(bR + 8 * (i % NRB), (i / NRB) & 1, P.err, 18, TC_DRAIN_NS);
    }

    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int g_num_sms = 0;
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

cudaError_t conv_tc_init() {
    if (!g_num_sms) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
    }
    if (!g_encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    cudaError_t e = cudaFuncSetAttribute(k_conv_tct<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, tt_smem(true));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_conv_tct<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, tt_smem(false));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_conv_tcf, cudaFuncAttributeMaxDynamicSharedMemorySize, TF_SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_convt_tc<CtCfg6>, cudaFuncAttributeMaxDynamicSharedMemorySize, CtCfg6::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_convt_tc<CtCfg6s>, cudaFuncAttributeMaxDynamicSharedMemorySize, CtCfg6s::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_convt_tc<CtCfg10>, cudaFuncAttributeMaxDynamicSharedMemorySize, CtCfg10::SMEM);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_conv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
}

int conv_tc_max_halo() { return TC_SLAB - TC_BM; }

// The instances of k_convt_tc: 16 channels per phase in a tile for strides 6
// (N = 96) and 10 (N = 160).
int convt_phase_nc(int S, int OC) {
    const int nc = (S == 6 || S == 10) ? 16 : 0;
    return nc > 0 && OC % nc == 0 ? nc : 0;
}

template <class C>
static void launch_convt(const TcParams &P, int64_t tiles, cudaStream_t st) {
    const int64_t slots = g_num_sms > 0 ? g_num_sms : 148;
    int64_t grid = tiles < slots ? tiles : slots;
    // resident weights: a grid of whole channel-group rounds keeps every tile
    // of a CTA in one group (tiles is a multiple of n_oc_tiles)
    if (C::RES) grid = grid / P.n_oc_tiles * P.n_oc_tiles;
    k_convt_tc<C><<<(unsigned)grid, C::THREADS, C::SMEM, st>>>(P);
}

// k_convt_tc launch (ConvTcArgs::phase_nc > 0).
static cudaError_t conv_tc_transposed(const ConvTcArgs &a, cudaStream_t st) {
    const int S = (int)a.omul, NC = a.phase_nc;
    if (NC != convt_phase_nc(S, a.OC) || a.n_tiles != a.OC / NC || a.K < 1 || a.d < 1 || a.p < 0 ||
        a.p > kHalfLo || (a.K - 1) * a.d > CT_SLAB - CT_BM || a.IC_pad % 64 != 0 || a.n_pos < 1 ||
        a.R_in < half_stride(0) || a.a_wrap < 0 || a.a_wrap >= a.IC_pad / 64 || a.phase_oc != 0 || a.resid_half ||
        a.accum || a.scale1 != 1.0f || a.scale2 != 1.0f || a.chscale || a.stats || a.x)
        return cudaErrorInvalidValue;
    // the residual arrives by bulk copies of 16-byte aligned row runs
    if (a.resid && (a.R_resid < a.R_out || a.R_resid % 4 != 0 || ((uintptr_t)a.resid & 15)))
        return cudaErrorInvalidValue;
    TcParams P;
    memset(&P, 0, sizeof(P));
    P.IC_blocks = a.IC_pad / 64;
    P.K = a.K;
    P.p = a.p;
    P.d = a.d;
    P.OC = a.OC;
    P.n_tiles = a.n_tiles;
    P.n_oc_tiles = a.n_tiles;
    P.mma_n = S * NC;
    P.phase_nc = NC;
    P.m_tiles = (a.n_pos + CT_BM - 1) / CT_BM;
    // the last slab stays inside the operand's chunk (rows < R + kHalfHi)
    const int64_t rows = a.R_in - kHalfLo - kHalfHi;
    if (a.n_pos > rows || (P.m_tiles - 1) * CT_BM - a.p + CT_SLAB > rows + kHalfHi) return cudaErrorInvalidValue;
    P.a = a.in;
    P.R_a = a.R_in;
    P.a_wrap = a.a_wrap;
    P.acc_scale = a.acc_scale == 0.0f ? 1.0f : a.acc_scale;
    P.w = a.w;
    P.out = a.out;
    P.R_out = a.R_out;
    P.n_pos = a.n_pos;
    P.omul = a.omul;
    P.oadd = a.oadd;
    P.bias = a.bias;
    P.resid = a.resid;
    P.R_resid = a.R_resid;
    P.scale1 = 1.0f;
    P.scale2 = 1.0f;
    P.err = a.err;
    const int64_t tiles = P.m_tiles * P.n_oc_tiles;
    if (S == 6 && a.K * P.IC_blocks <= CT_RES_TILES && P.n_oc_tiles <= (g_num_sms > 0 ? g_num_sms : 148))
        launch_convt<CtCfg6>(P, tiles, st);
    else if (S == 6)
        launch_convt<CtCfg6s>(P, tiles, st);
    else
        launch_convt<CtCfg10>(P, tiles, st);
    return cudaGetLastError();
}

// 2-D map of an F32 [C][R] tensor in 32 x 32 boxes (x = position, y =
// channel) with the 128-byte swizzle of the channel-major staging.
static bool block_map_swz(CUtensorMap *m, const float *base, int64_t R, int C) {
    if (((uintptr_t)base & 15) || (R & 3)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)C};
    cuuint64_t strides[1] = {(cuuint64_t)R * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map of the F32 input [C][R] of k_conv_tcf in [64 ch][32 rows] pieces,
// 128-byte swizzle; rows outside [0, R) read as zero.
static bool piece_map(CUtensorMap *m, const float *base, int64_t R, int C) {
    if (((uintptr_t)base & 15) || (R & 3)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)R, (cuuint64_t)C};
    cuuint64_t strides[1] = {(cuuint64_t)R * 4};
    cuuint32_t box[2] = {32, 64};
    cuuint32_t estr[2] = {1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool conv_tc_fusable(const ConvTcArgs &a) {
    return g_encode && a.x && a.x_ms && a.x_nw && a.x_nb && a.x_gamma && a.x_beta && a.x_alpha && a.omul == 1 &&
           a.oadd == 0 && a.phase_oc == 0 && !a.resid_half && a.accum == 0 && a.scale1 == 1.0f &&
           a.scale2 == 1.0f && a.OC >= 64 && a.OC <= a.n_tiles * TC_BN && a.n_pos == a.R_out &&
           a.R_out % 128 == 0 && (!a.resid || a.R_resid == a.R_out) && a.IC_pad >= 64 && a.IC_pad % 64 == 0 &&
           a.K >= 1 && a.d >= 1 && a.p >= 0 && (a.K - 1) * a.d + 3 <= TC_SLAB - TC_BM && a.sb.n >= 1 && a.sm >= 4 &&
           a.sextra >= 0 && a.a_wrap == 0 && (a.acc_scale == 0.0f || a.acc_scale == 1.0f) && !a.chscale;
}

// k_conv_tcf launch: the operand formed from x inside the conv.
static cudaError_t conv_tc_fused(const ConvTcArgs &a, cudaStream_t st) {
    if (!conv_tc_fusable(a)) return cudaErrorInvalidValue;
    TcParams P;
    memset(&P, 0, sizeof(P));
    P.IC_blocks = a.IC_pad / 64;
    P.K = a.K;
    P.p = a.p;
    P.d = a.d;
    P.OC = a.OC;
    P.n_tiles = a.n_tiles;
    P.n_oc_tiles = (a.OC + TC_BN - 1) / TC_BN;
    P.mma_n = TC_BN;
    P.m_tiles = (a.n_pos + TC_BM - 1) / TC_BM;
    P.w = a.w;
    P.out = a.out;
    P.R_out = a.R_out;
    P.n_pos = a.n_pos;
    P.omul = 1;
    P.bias = a.bias;
    P.resid = a.resid;
    P.R_resid = a.R_resid;
    P.scale1 = 1.0f;
    P.scale2 = 1.0f;
    P.err = a.err;
    P.sb = a.sb;
    P.sm = a.sm;
    P.sextra = a.sextra;
    P.IC = a.IC_pad;
    P.x_ms = a.x_ms;
    P.x_nw = a.x_nw;
    P.x_nb = a.x_nb;
    P.x_gamma = a.x_gamma;
    P.x_beta = a.x_beta;
    P.x_alpha = a.x_alpha;
    P.nz = -0.0f;
    P.nz2 = 0x8000000080000000ull;
    const bool fused_stats = a.stats && a.part && a.stats_aligned;
    P.part = fused_stats ? a.part : nullptr;
    CUtensorMap omap, rmap, xmap;
    memset(&omap, 0, sizeof(omap));
    memset(&rmap, 0, sizeof(rmap));
    memset(&xmap, 0, sizeof(xmap));
    if (!block_map_swz(&omap, a.out, a.R_out, a.OC) ||
        !block_map_swz(&rmap, a.resid ? a.resid : a.out, a.R_out, a.OC) || !piece_map(&xmap, a.x, a.R_out, a.IC_pad))
        return cudaErrorInvalidValue;
    const int64_t tiles = P.m_tiles * P.n_oc_tiles;
    const int64_t slots = g_num_sms > 0 ? g_num_sms : 148;
    const unsigned grid = (unsigned)(tiles < slots ? tiles : slots);
    k_conv_tcf<<<grid, TF_THREADS, TF_SMEM, st>>>(P, omap, rmap, xmap);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !a.stats) return e;
    if (fused_stats)
        stats_blocks(a.part, a.R_out / 32, a.OC, a.sm, a.sextra, a.sb, a.stats, st);
    else
        stats(a.out, a.R_out, a.OC, a.sm, a.sextra, a.sb, a.stats, st);
    return cudaGetLastError();
}

cudaError_t conv_tc(const ConvTcArgs &a, cudaStream_t st) {
    if (a.x) return conv_tc_fused(a, st);
    if (a.phase_nc > 0) return conv_tc_transposed(a, st);
    const int halo = (a.K - 1) * a.d;
    if (a.K < 1 || a.d < 1 || a.p < 0 || halo > TC_SLAB - TC_BM || a.p > kHalfLo || a.IC_pad % 64 != 0 ||
        a.OC > a.n_tiles * TC_BN || a.n_pos < 1 || a.R_in < half_stride(0) || a.a_wrap < 0 ||
        a.a_wrap >= a.IC_pad / 64)
        return cudaErrorInvalidValue;
    TcParams P;
    memset(&P, 0, sizeof(P));
    P.IC_blocks = a.IC_pad / 64;
    P.K = a.K;
    P.p = a.p;
    P.d = a.d;
    P.OC = a.OC;
    P.n_tiles = a.n_tiles;
    P.n_oc_tiles = (a.OC + TC_BN - 1) / TC_BN;
    P.mma_n = a.OC < TC_BN ? (a.OC + 15) / 16 * 16 : TC_BN;
    P.phase_oc = a.phase_oc;
    if (a.phase_oc < 0 || (a.phase_oc > 0 && (a.phase_oc % TC_BN != 0 || a.OC % a.phase_oc != 0)))
        return cudaErrorInvalidValue;
    P.m_tiles = (a.n_pos + TC_BM - 1) / TC_BM;
    // the last slab must stay inside the chunk: rows < R + kHalfHi where the
    // operand has R = R_in - kHalfLo - kHalfHi rows
    const int64_t rows = a.R_in - kHalfLo - kHalfHi;
    if (a.n_pos > rows || (P.m_tiles - 1) * TC_BM - a.p + TC_SLAB > rows + kHalfHi) return cudaErrorInvalidValue;
    P.a = a.in;
    P.R_a = a.R_in;
    P.a_wrap = a.a_wrap;
    P.acc_scale = a.acc_scale == 0.0f ? 1.0f : a.acc_scale;
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
    P.chscale = a.chscale;
    P.scale1 = a.scale1;
    P.accum = a.accum;
    P.scale2 = a.scale2;
    P.err = a.err;
    P.part = nullptr;
    P.sb = a.sb;
    P.sm = a.sm;
    P.sextra = a.sextra;
    if (a.stats && (a.sb.n < 1 || a.sm < 1 || a.sextra < 0 || a.omul != 1 || a.oadd != 0 || a.phase_oc != 0))
        return cudaErrorInvalidValue;
    const int64_t tiles = P.m_tiles * P.n_oc_tiles;
    const int64_t slots = g_num_sms > 0 ? g_num_sms : 148;
    const unsigned grid = (unsigned)(tiles < slots ? tiles : slots);
    // channels x positions kernel where output row = position
    // (a residual upsampled x2 by resid_half only on the unstaged epilogue;
    // its rows up to n_pos / 2 exist)
    if (a.omul == 1 && a.oadd == 0 && a.phase_oc == 0 && a.OC >= 64 && a.n_pos <= a.R_out &&
        (!a.resid || (a.resid_half ? 2 * a.R_resid >= a.n_pos : a.R_resid >= a.n_pos))) {
        CUtensorMap omap, rmap;
        memset(&omap, 0, sizeof(omap));
        memset(&rmap, 0, sizeof(rmap));
        // staged blocks where every position of the level is written
        const bool staged = g_encode && !a.resid_half && a.n_pos == a.R_out && a.R_out % 32 == 0 &&
                            (!a.resid || a.R_resid == a.R_out) &&
                            block_map_swz(&omap, a.out, a.R_out, a.OC) &&
                            block_map_swz(&rmap, a.resid ? a.resid : a.out, a.R_out, a.OC);
        // block partials where every position is written and the utterances
        // start on block boundaries (then R_out is a multiple of 128)
        const bool fused = a.stats && a.part && a.stats_aligned && a.n_pos == a.R_out && a.R_out % 128 == 0;
        if (fused) P.part = a.part;
        P.sched = a.sched;
        if (staged)
            k_conv_tct<true><<<grid, TC_THREADS, tt_smem(true), st>>>(P, omap, rmap);
        else
            k_conv_tct<false><<<grid, TC_THREADS, tt_smem(false), st>>>(P, omap, rmap);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess || !a.stats) return e;
        if (fused)
            stats_blocks(a.part, a.R_out / 32, a.OC, a.sm, a.sextra, a.sb, a.stats, st);
        else
            stats(a.out, a.R_out, a.OC, a.sm, a.sextra, a.sb, a.stats, st);
        return cudaGetLastError();
    }
    k_conv_tc<<<grid, TC_THREADS, TC_SMEM, st>>>(P);
    cudaError_t e = cudaGetLastError();
    // this kernel keeps no partials: a separate pass over the written output
    if (e == cudaSuccess && a.stats) {
        stats(a.out, a.R_out, a.OC, a.sm, a.sextra, a.sb, a.stats, st);
        e = cudaGetLastError();
    }
    return e;
}

// The bounded wait of the convolution kernels, made to run out: one thread
// initialises an mbarrier that expects one arrival, which nothing makes, and
// waits on it with mbar_wait. After limit_ns the wait records
// kErrWaitSelftest in *err and returns false, and the kernel ends; the
// context stays usable and the host reads the status as for a real expiry.
__global__ void k_wait_selftest(int *err, unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_wait(b, 0, err, kErrWaitSelftest, limit_ns);
}

cudaError_t wait_selftest(int *err, unsigned long long limit_ns, cudaStream_t st) {
    if (limit_ns > TC_WAIT_NS) return cudaErrorInvalidValue;
    k_wait_selftest<<<1, 32, 0, st>>>(err, limit_ns);
    return cudaGetLastError();
}

}  // namespace kk
