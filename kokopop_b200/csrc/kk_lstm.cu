// Bidirectional LSTM stack (prosody duration encoder) and the durations ->
// frames alignment.
//
// Layout: the sequences of a batch are packed time-major, row = t * B + b
// (B sequences, t < max length), channel-major [C][R] like every other
// activation of the library, so the input projection W_ih x + b_ih is one
// K = 1 convolution over all rows and both directions (output channels
// [forward 4H | backward 4H]) on the existing convolution kernels.
//
// Recurrence (cpu_lstm_contiguous, src/arch/kokoro/lstm_fused.cpp:200-247):
// one thread-block cluster of 8 CTAs per (direction, group of Bc sequences).
// CTA r of the cluster owns hidden units [32 r, 32 r + 32) and their four
// gate rows of W_hh (128 rows x 256, F32, 130 KB padded) in shared memory
// for the whole sequence. Local row lr = 4 u + q holds gate q (i, f, g, o) of
// local unit u, so warp w owns units 4w .. 4w + 3 with all their gates.
// Per step:
//   * every CTA waits on its own mbarrier for the previous h of all 256
//     units (the cluster's stores, below), bounded in time;
//   * two threads per gate row each sum one half of the 256-term dot
//     (fixed order: interleaved FMA partial sums, then their pairwise sum,
//     then the two halves); the reference's AVX2 build reorders this sum
//     too (lstm_fused.cpp:93-123), and the parity bound covers it;
//   * the gate sum is (b_hh + pre) + dot as in the reference, the pre-gates
//     having been loaded from global memory one step ahead; the gate's
//     activation is applied by its own thread;
//   * the warp's lanes update the cells of its 4 units (c stays in
//     registers) after a __syncwarp, write h to global memory, and store it
//     into the h buffer of every CTA of the cluster with st.async, each
//     store completing bytes on the receiving CTA's mbarrier.
// No block-wide or cluster-wide barrier runs inside the step loop: a CTA's
// buffer for step s + 2 is written only after every CTA has sent its h for
// step s + 1, which each sends after finishing its dot of step s + 1 that
// read the other buffer, so the double buffer needs no further fence.
#include "kk_kernels.h"

#include <atomic>

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace kk {

constexpr int kLstmH = 256;        // hidden units per direction
constexpr int kLstmCl = 8;         // CTAs per cluster
constexpr int kLstmUnits = 32;     // hidden units per CTA
constexpr int kLstmRows = 128;     // gate rows per CTA (4 gates x 32 units)
constexpr int kLstmThreads = 256;  // two threads per gate row
constexpr int kLstmHalf = kLstmH / 2;    // terms of the dot per thread
constexpr int kWStride = kLstmH + 8;     // W row stride in shared memory (floats): conflict-free 16-byte loads
constexpr unsigned long long kLstmWaitNs = 1000000000ull;  // 1 s per wait, then kErrLstmWait

size_t lstm_rec_smem(int Bc) {
    return sizeof(float) * ((size_t)kLstmRows * kWStride + 2 * (size_t)Bc * kLstmH + (size_t)kLstmRows * Bc);
}

// lstm_fused.cpp:60-68: branch-stable logistic, with CUDA's single-precision
// expf (the reference calls the C library's; both are within a few ulp)
__device__ __forceinline__ float sigmoid_stable(float x) {
    if (x >= 0.0f) {
        const float z = expf(-x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
    }
    const float z = expf(x);
    return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

__device__ __forceinline__ uint32_t lstm_smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t lstm_clock_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of parity `parity` of the mbarrier at `bar`; false
// after kLstmWaitNs.
__device__ __forceinline__ bool lstm_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = lstm_clock_ns();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (lstm_clock_ns() - t0 > kLstmWaitNs) return false;
    }
}

// this CTA's shared address `local` as seen in the shared memory of CTA
// `rank` of the cluster
__device__ __forceinline__ uint32_t lstm_mapa(uint32_t local, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// 4-byte store into another CTA's shared memory that completes its bytes on
// that CTA's mbarrier
__device__ __forceinline__ void lstm_st_async(uint32_t remote, float v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote),
                 "r"(__float_as_uint(v)), "r"(remote_bar)
                 : "memory");
}

// non-finite -> 0, clamp to +-lim
__device__ __forceinline__ float sanitize(float x, float lim) {
    if (!isfinite(x)) return 0.0f;
    return fminf(fmaxf(x, -lim), lim);
}

// Pre-gates of step s for the sequences jj = part, part + 2, ... of the
// group (the ones this thread adds into its gate values), 0 past a sequence.
template <int BC>
__device__ __forceinline__ void lstm_load_pre(float (&p)[(BC + 1) / 2], const float *pre, int64_t B, int b0,
                                              const int *lens, int d, int s, int part) {
#pragma unroll
    for (int i = 0; i < (BC + 1) / 2; ++i) {
        const int jj = 2 * i + part;
        float v = 0.0f;
        if (jj < BC) {
            const int L = lens[jj];
            if (s < L) {
                const int t = d ? L - 1 - s : s;
                v = pre[(int64_t)t * B + b0 + jj];
            }
        }
        p[i] = v;
    }
}

template <int BC>
__global__ void __cluster_dims__(kLstmCl, 1, 1) __launch_bounds__(kLstmThreads, 1)
    k_lstm_rec(const LstmRecArgs a) {
    constexpr int NA = BC >= 4 ? 1 : 4 / BC;  // interleaved partial sums per sequence
    constexpr int NP = (4 * BC + 31) / 32;    // (unit, sequence) cells per lane
    constexpr int NH = (BC + 1) / 2;          // sequences whose pre-gates a thread adds
    constexpr uint32_t kBytes = (uint32_t)kLstmH * BC * 4;  // h of one step, all units
    cg::cluster_group cluster = cg::this_cluster();
    const int cr = (int)cluster.block_rank();
    const int cid = blockIdx.x / kLstmCl;
    const int d = cid & 1, grp = cid >> 1;
    const int b0 = grp * BC;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    extern __shared__ __align__(16) float sm[];
    float *W = sm;                          // [128 local rows][kWStride]
    float *hb = W + kLstmRows * kWStride;   // [2][BC][256]: h of the previous step, double-buffered
    float *gb = hb + 2 * BC * kLstmH;       // [128 local rows][BC]: activated gates
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ int lens[BC];
    const float *whh = d ? a.whh[1] : a.whh[0];
    const float *bhh = d ? a.bhh[1] : a.bhh[0];
    // local row lr = 4 u + q <-> gate row j = q * 256 + 32 cr + u, in natural
    // k order; the two threads of a row take alternate 16-byte chunks, and
    // the 264-float stride (8 banks apart) puts the 8 threads of each
    // quarter-warp's 16-byte loads on 32 distinct banks
    for (int idx = tid; idx < kLstmRows * kLstmH; idx += kLstmThreads) {
        const int lr = idx / kLstmH, k = idx % kLstmH;
        const int j = (lr & 3) * kLstmH + kLstmUnits * cr + (lr >> 2);
        W[lr * kWStride + k] = whh[(int64_t)j * kLstmH + k];
    }
    for (int idx = tid; idx < BC * kLstmH; idx += kLstmThreads) hb[idx] = 0.0f;  // h(-1) = 0
    if (tid < BC) lens[tid] = b0 + tid < a.B ? a.len[b0 + tid] : 0;
    const uint32_t bar0 = lstm_smem_u32(&bar[0]);
    if (tid == 0) {
        // one arrival per phase (the expect below); the phase completes when
        // all kBytes of a step's h have been stored by the cluster
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int b = 0; b < 2; ++b)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8 * b), "r"(kBytes)
                         : "memory");
    }
    cluster.sync();  // every CTA's barriers are armed before any store reaches them

    const int lr = tid >> 1, part = tid & 1;  // gate row and dot half of this thread
    const int q = lr & 3;
    const int jrow = q * kLstmH + kLstmUnits * cr + (lr >> 2);
    const float bias = bhh[jrow];
    const float *pre = a.pre + ((int64_t)d * 4 * kLstmH + jrow) * a.R;
    const float *wrow = W + lr * kWStride + 4 * part;
    float pcur[NH], pnext[NH];
    lstm_load_pre<BC>(pcur, pre, a.B, b0, lens, d, 0, part);
    float c[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) c[j] = 0.0f;

    bool ok = true;
    for (int s = 0; s < a.max_len; ++s) {
        const int cb = s & 1, nb = cb ^ 1;
        if (s > 0) {
            ok = __all_sync(0xffffffffu, lstm_wait(bar0 + 8 * cb, ((s - 1) >> 1) & 1));
            if (!ok) {
                if (lane == 0) atomicCAS(a.err, 0, kErrLstmWait);
                break;
            }
            // the next phase of this buffer (step s + 2's h) can only start
            // after this CTA has sent step s + 1's, later than this
            if (tid == 0)
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar0 + 8 * cb),
                             "r"(kBytes)
                             : "memory");
        }
        // next step's pre-gates, a step ahead of their use
        lstm_load_pre<BC>(pnext, pre, a.B, b0, lens, d, s + 1, part);
        // dot products: this thread's 32 chunks of 4 terms (half of 256)
        const float *hp = hb + cb * BC * kLstmH + 4 * part;
        float acc[BC][NA];
#pragma unroll
        for (int jj = 0; jj < BC; ++jj)
#pragma unroll
            for (int i = 0; i < NA; ++i) acc[jj][i] = 0.0f;
#pragma unroll 4
        for (int ch = 0; ch < kLstmHalf / 4; ++ch) {
            const float4 w4 = *reinterpret_cast<const float4 *>(wrow + 8 * ch);
#pragma unroll
            for (int jj = 0; jj < BC; ++jj) {
                const float4 h4 = *reinterpret_cast<const float4 *>(hp + jj * kLstmH + 8 * ch);
                if (NA == 4) {
                    acc[jj][0] = fmaf(w4.x, h4.x, acc[jj][0]);
                    acc[jj][1 % NA] = fmaf(w4.y, h4.y, acc[jj][1 % NA]);
                    acc[jj][2 % NA] = fmaf(w4.z, h4.z, acc[jj][2 % NA]);
                    acc[jj][3 % NA] = fmaf(w4.w, h4.w, acc[jj][3 % NA]);
                } else {
                    acc[jj][0] = fmaf(w4.x, h4.x, acc[jj][0]);
                    acc[jj][1 % NA] = fmaf(w4.y, h4.y, acc[jj][1 % NA]);
                    acc[jj][0] = fmaf(w4.z, h4.z, acc[jj][0]);
                    acc[jj][1 % NA] = fmaf(w4.w, h4.w, acc[jj][1 % NA]);
                }
            }
        }
        // gate values: the partial sums in a fixed order, the two halves
        // (lower half first on both threads), then (b_hh + pre) + dot
#pragma unroll
        for (int jj = 0; jj < BC; ++jj) {
            float sum = acc[jj][0];
            if (NA == 2) sum = __fadd_rn(acc[jj][0], acc[jj][1 % NA]);
            if (NA == 4) sum = __fadd_rn(__fadd_rn(acc[jj][0], acc[jj][1 % NA]), __fadd_rn(acc[jj][2 % NA], acc[jj][3 % NA]));
            const float other = __shfl_xor_sync(0xffffffffu, sum, 1);
            const float dot = part == 0 ? __fadd_rn(sum, other) : __fadd_rn(other, sum);
            if ((jj & 1) == part) {
                const float x = sanitize(__fadd_rn(__fadd_rn(bias, pcur[jj >> 1]), dot), 80.0f);
                gb[lr * BC + jj] = q == 2 ? tanhf(x) : sigmoid_stable(x);
            }
        }
        __syncwarp();
        // cells of the warp's 4 units: cell p = lane + 32 j is unit
        // 4 warp + p / BC of sequence p % BC
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int p = lane + 32 * j;
            if (p < 4 * BC) {
                const int ul = 4 * warp + p / BC, jj = p % BC;
                const float *g4 = gb + (4 * ul) * BC + jj;
                const float ig = g4[0], fg = g4[BC], gg = g4[2 * BC], og = g4[3 * BC];
                const int L = lens[jj];
                const bool live = s < L;
                const float cn = sanitize(__fadd_rn(__fmul_rn(fg, c[j]), __fmul_rn(ig, gg)), 50.0f);
                float hv = __fmul_rn(og, tanhf(cn));
                if (!isfinite(hv)) hv = 0.0f;
                if (!live) hv = 0.0f;
                else c[j] = cn;
                const int unit = kLstmUnits * cr + ul;
                if (live) {
                    const int t = d ? L - 1 - s : s;
                    a.hout[(int64_t)(d * kLstmH + unit) * a.R + (int64_t)t * a.B + b0 + jj] = hv;
                }
                // every CTA of the cluster, this one included, gets the value
                const uint32_t dst = lstm_smem_u32(hb + nb * BC * kLstmH + jj * kLstmH + unit);
#pragma unroll
                for (int r = 0; r < kLstmCl; ++r) lstm_st_async(lstm_mapa(dst, r), hv, lstm_mapa(bar0 + 8 * nb, r));
            }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < NH; ++i) pcur[i] = pnext[i];
    }
    // the last step's stores into this CTA complete before it leaves the
    // cluster
    if (ok) {
        const int s = a.max_len;
        if (!__all_sync(0xffffffffu, lstm_wait(bar0 + 8 * (s & 1), ((s - 1) >> 1) & 1)) && lane == 0)
            atomicCAS(a.err, 0, kErrLstmWait);
    }
    cluster.sync();
}

template <int BC>
static cudaError_t launch_rec(const LstmRecArgs &a, int n_clusters, cudaStream_t st) {
    const size_t smem = lstm_rec_smem(BC);
    cudaError_t e = cudaFuncSetAttribute(k_lstm_rec<BC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_lstm_rec<BC><<<n_clusters * kLstmCl, kLstmThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <int BC>
static int max_clusters_of() {
    const size_t smem = lstm_rec_smem(BC);
    if (cudaFuncSetAttribute(k_lstm_rec<BC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kLstmCl * 64);
    cfg.blockDim = dim3(kLstmThreads);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_lstm_rec<BC>, &cfg) != cudaSuccess) n = 0;
    return n;
}

int lstm_max_clusters(int Bc) {
    constexpr int kDev = 64;
    static std::atomic<int> cache[kDev][6];  // 0 = not yet asked; -1 = query failed
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const int i = Bc == 1 ? 0 : Bc == 2 ? 1 : Bc == 4 ? 2 : Bc == 8 ? 3 : Bc == 16 ? 4 : Bc == 32 ? 5 : -1;
    if (i < 0) return 0;
    if (dev >= 0 && dev < kDev) {
        const int v = cache[dev][i].load(std::memory_order_relaxed);
        if (v != 0) return v < 0 ? 0 : v;
    }
    int n = 0;
    switch (Bc) {
        case 1: n = max_clusters_of<1>(); break;
        case 2: n = max_clusters_of<2>(); break;
        case 4: n = max_clusters_of<4>(); break;
        case 8: n = max_clusters_of<8>(); break;
        case 16: n = max_clusters_of<16>(); break;
        default: n = max_clusters_of<32>(); break;
    }
    cudaGetLastError();  // a failed query leaves no sticky error behind
    if (dev >= 0 && dev < kDev) cache[dev][i].store(n > 0 ? n : -1, std::memory_order_relaxed);
    return n;
}

cudaError_t lstm_recurrence(const LstmRecArgs &a, cudaStream_t st) {
    if (a.B < 1 || a.max_len < 1) return cudaSuccess;
    if (!a.err) return cudaErrorInvalidValue;
    const int groups = (a.B + a.Bc - 1) / a.Bc;
    const int n_clusters = 2 * groups;
    switch (a.Bc) {
        case 1: return launch_rec<1>(a, n_clusters, st);
        case 2: return launch_rec<2>(a, n_clusters, st);
        case 4: return launch_rec<4>(a, n_clusters, st);
        case 8: return launch_rec<8>(a, n_clusters, st);
        case 16: return launch_rec<16>(a, n_clusters, st);
        case 32: return launch_rec<32>(a, n_clusters, st);
        default: return cudaErrorInvalidValue;
    }
}

// ---------------------------------------------------------------------------
// packing
// ---------------------------------------------------------------------------

// x: per sequence [len_b][D] feature-fastest, back to back (offsets cum[b]);
// X: [C][R] with row t * B + b. Channels [D, D + Ds) take the sequence's style
// vector (the duration encoder's concat); rows past a sequence stay as they
// are (zero from the caller's memset).
__global__ void k_lstm_pack(const float *__restrict__ x, int D, const float *__restrict__ style, int Ds,
                            float *__restrict__ X, int64_t R, const int32_t *__restrict__ len,
                            const int64_t *__restrict__ cum, int B) {
    const int b = blockIdx.y;
    const int L = len[b];
    const int C = D + Ds;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)L * C;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(idx / C), c = (int)(idx % C);
        const float v = c < D ? x[(cum[b] + t) * D + c] : style[(int64_t)b * Ds + (c - D)];
        X[(int64_t)c * R + (int64_t)t * B + b] = v;
    }
}

// inverse: out[cum[b] + t][c] = X[c][t * B + b], c < C
__global__ void k_lstm_unpack(const float *__restrict__ X, int64_t R, int C, float *__restrict__ out,
                              const int32_t *__restrict__ len, const int64_t *__restrict__ cum, int B) {
    const int b = blockIdx.y;
    const int L = len[b];
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)L * C;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(idx / C), c = (int)(idx % C);
        out[(cum[b] + t) * C + c] = X[(int64_t)c * R + (int64_t)t * B + b];
    }
}

// X [C][R] in the LSTM layout (row t * B + b) -> dst [C][R_dst] at rows
// m * offT[b] + t of a packed ragged level (t < len[b]); other rows untouched.
__global__ void k_lstm_to_level(const float *__restrict__ X, int64_t R, int B, const int32_t *__restrict__ len,
                                float *__restrict__ dst, int64_t R_dst, const int64_t *__restrict__ offT, int m) {
    const int b = blockIdx.y, c = blockIdx.z;
    const int L = len[b];
    const int64_t o = (int64_t)m * offT[b];
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x)
        dst[(int64_t)c * R_dst + o + t] = X[(int64_t)c * R + (int64_t)t * B + b];
}

void lstm_to_level(const float *X, int64_t R, int C, int B, const int32_t *len, int max_len, float *dst,
                   int64_t R_dst, const int64_t *offT, int m, cudaStream_t st) {
    int bx = (max_len + 255) / 256;
    if (bx > 64) bx = 64;
    if (bx < 1) bx = 1;
    k_lstm_to_level<<<dim3(bx, B, C), 256, 0, st>>>(X, R, B, len, dst, R_dst, offT, m);
}

void lstm_pack(const float *x, int D, const float *style, int Ds, float *X, int64_t R, const int32_t *len,
               const int64_t *cum, int B, int max_len, cudaStream_t st) {
    int bx = (int)(((int64_t)max_len * (D + Ds) + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_lstm_pack<<<dim3(bx, B), 256, 0, st>>>(x, D, style, Ds, X, R, len, cum, B);
}

void lstm_unpack(const float *X, int64_t R, int C, float *out, const int32_t *len, const int64_t *cum, int B,
                 int max_len, cudaStream_t st) {
    int bx = (int)(((int64_t)max_len * C + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_lstm_unpack<<<dim3(bx, B), 256, 0, st>>>(X, R, C, out, len, cum, B);
}

// ---------------------------------------------------------------------------
// AdaLayerNorm (ada_layer_norm, src/arch/kokoro/graph_ops.cpp:865-886)
// ---------------------------------------------------------------------------

// gamma / beta of one AdaLayerNorm per sequence: linear (graph_ops.cpp:636-654)
// with the sequential F32 sum, the style rounded to half for an F16 weight.
// w: [C][Ds] values; out: [B][C].
__global__ void k_style_linear(const float *__restrict__ w, const float *__restrict__ bias, int f16,
                               const float *__restrict__ style, int Ds, int C, float *__restrict__ out) {
    const int b = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float *s = style + (int64_t)b * Ds;
    const float *wr = w + (int64_t)c * Ds;
    float acc = 0.0f;
    for (int i = 0; i < Ds; ++i) {
        const float x = f16 ? round_f16(s[i]) : s[i];
        acc = __fadd_rn(acc, __fmul_rn(wr[i], x));
    }
    out[(int64_t)b * C + c] = __fadd_rn(acc, bias[c]);
}

void style_linear(const float *w, const float *bias, int f16, const float *style, int Ds, int C, int B, float *out,
                  cudaStream_t st) {
    k_style_linear<<<dim3((C + 127) / 128, B), 128, 0, st>>>(w, bias, f16, style, Ds, C, out);
}

// ggml_norm over the D features of each row (mean, then the variance of
// x - mean, sums in double), then (y + y * gamma) + beta; result into X rows
// (channels [0, D)). One block of 256 threads handles 32 rows: lane = row,
// warp = channel slice.
__global__ void __launch_bounds__(256) k_ada_layer_norm(const float *__restrict__ h, int64_t R, int D,
                                                        const float *__restrict__ gamma,
                                                        const float *__restrict__ beta, float *__restrict__ X,
                                                        const int32_t *__restrict__ len, int B, float eps) {
    __shared__ double part[8][33];
    __shared__ float stat[2][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * 32 + lane;
    const int b = (int)(row % B);
    const int64_t t = row / B;
    const bool live = row < R && t < len[b];
    // pass 1: mean
    double s = 0.0;
    if (live)
        for (int c = w; c < D; c += 8) s += (double)h[(int64_t)c * R + row];
    part[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        double tot = 0.0;
        for (int i = 0; i < 8; ++i) tot += part[i][lane];
        stat[0][lane] = __fdiv_rn((float)tot, (float)D);
    }
    __syncthreads();
    const float mean = stat[0][lane];
    // pass 2: variance of x - mean
    s = 0.0;
    if (live)
        for (int c = w; c < D; c += 8) {
            const float v = __fsub_rn(h[(int64_t)c * R + row], mean);
            s += (double)__fmul_rn(v, v);
        }
    __syncthreads();
    part[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        double tot = 0.0;
        for (int i = 0; i < 8; ++i) tot += part[i][lane];
        const float var = (float)(tot / (double)D);
        stat[1][lane] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const float scale = stat[1][lane];
    if (row >= R) return;
    for (int c = w; c < D; c += 8) {
        float v = 0.0f;
        if (live) {
            const float y = __fmul_rn(__fsub_rn(h[(int64_t)c * R + row], mean), scale);
            v = __fadd_rn(__fadd_rn(y, __fmul_rn(y, gamma[(int64_t)b * D + c])), beta[(int64_t)b * D + c]);
        }
        X[(int64_t)c * R + row] = v;
    }
}

void ada_layer_norm(const float *h, int64_t R, int D, const float *gamma, const float *beta, float *X,
                    const int32_t *len, int B, cudaStream_t st) {
    k_ada_layer_norm<<<(unsigned)((R + 31) / 32), 256, 0, st>>>(h, R, D, gamma, beta, X, len, B, 1e-5f);
}

// ---------------------------------------------------------------------------
// R11: durations -> frames, alignment (src/arch/kokoro/kokoro.cpp:115-193,
// :669-674)
// ---------------------------------------------------------------------------

// frames[i] = clamp(int(lrint(d[i] / speed)), 1, 50); non-finite -> 1. The
// speed was sanitised on the host (non-finite or <= 0 -> 1).
__global__ void k_duration_frames(const float *__restrict__ d, int64_t n, float speed, int32_t *__restrict__ frames) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = __fdiv_rn(d[i], speed);
        int r = 1;
        if (isfinite(v)) {
            // lrint rounds to nearest-even into a 64-bit long; the reference
            // then narrows it to int (two's-complement truncation)
            const long long l = __float2ll_rn(v);
            const int n32 = (int)(unsigned int)(unsigned long long)l;
            r = n32 < 1 ? 1 : (n32 > 50 ? 50 : n32);
        }
        frames[i] = r;
    }
}

// exclusive prefix sum of frames (one block; n up to a few thousand tokens)
// and the frame -> token map; start[n] = total.
__global__ void k_duration_scan(const int32_t *__restrict__ frames, int64_t n, int64_t *__restrict__ start) {
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        __shared__ int64_t buf[1024];
        const int64_t i = base + threadIdx.x;
        buf[threadIdx.x] = i < n ? frames[i] : 0;
        __syncthreads();
        for (int off = 1; off < (int)blockDim.x; off <<= 1) {
            const int64_t v = threadIdx.x >= (unsigned)off ? buf[threadIdx.x - off] : 0;
            __syncthreads();
            buf[threadIdx.x] += v;
            __syncthreads();
        }
        const int64_t incl = buf[threadIdx.x];
        const int64_t excl = incl - (i < n ? frames[i] : 0);
        if (i < n) start[i] = carry + excl;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) start[n] = carry;
}

// en[f][:] = hidden[token(f)][:]: the one-hot alignment matmul d . mask is
// a copy of the frame's token row.
__global__ void k_align_gather(const float *__restrict__ hidden, int64_t D, const int32_t *__restrict__ frames,
                               const int64_t *__restrict__ start, int64_t n, float *__restrict__ en) {
    const int64_t i = blockIdx.y;  // token
    if (i >= n) return;
    const int64_t f0 = start[i];
    const int nf = frames[i];
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)nf * D;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / D, c = idx % D;
        en[(f0 + r) * D + c] = hidden[i * D + c];
    }
}

void duration_frames(const float *d, int64_t n, float speed, int32_t *frames, int64_t *start, cudaStream_t st) {
    int bx = (int)((n + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_duration_frames<<<bx, 256, 0, st>>>(d, n, speed, frames);
    k_duration_scan<<<1, 1024, 0, st>>>(frames, n, start);
}

void align_gather(const float *hidden, int64_t D, const int32_t *frames, const int64_t *start, int64_t n, float *en,
                  cudaStream_t st) {
    if (n < 1) return;
    int bx = (int)((50 * D + 255) / 256);
    if (bx > 64) bx = 64;
    k_align_gather<<<dim3(bx, (unsigned)n), 256, 0, st>>>(hidden, D, frames, start, n, en);
}

}  // namespace kk
