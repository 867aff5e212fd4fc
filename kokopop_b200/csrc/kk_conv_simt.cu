// Dense 1-D convolution as a CUDA-core implicit GEMM over the packed
// channel-major layout (F32 accumulation). It serves the small-channel
// convolutions that do not fill a tensor-core tile (noise_convs with 22 input
// channels, conv_post with 22 outputs) and is the F32-exact cross-check for
// the tensor-core path.
//
// Block tile: 128 output positions x 64 output channels, 256 threads, each
// thread 8 positions x 4 channels. The K loop walks 8 input channels at a
// time with the input slab (positions plus halo) and the weights staged in
// shared memory.
#include "kk_kernels.h"

namespace kk {

constexpr int CS_BM = 128;
constexpr int CS_BN = 64;
constexpr int CS_ICB = 8;
constexpr int CS_MAX_SMEM = 96 * 1024;

__global__ void __launch_bounds__(256) k_conv_simt(ConvArgs a) {
    extern __shared__ float sm[];
    const int span = (CS_BM - 1) * a.s + (a.K - 1) * a.d + 1;
    float *xs = sm;                    // [ICB][span]
    float *ws = sm + CS_ICB * span;    // [BN][ICB][K]
    const int64_t q0 = (int64_t)blockIdx.x * CS_BM;
    const int oc0 = blockIdx.y * CS_BN;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const int64_t in0 = q0 * a.s - a.p;
    const int wsz = CS_BN * CS_ICB * a.K;
    for (int ic0 = 0; ic0 < a.IC; ic0 += CS_ICB) {
        __syncthreads();
        for (int i = tid; i < CS_ICB * span; i += 256) {
            const int ic = i / span, q = i - ic * span;
            const int64_t r = in0 + q;
            float v = 0.f;
            if (ic0 + ic < a.IC && r >= 0 && r < a.R_in) v = a.in[(int64_t)(ic0 + ic) * a.R_in + r];
            if (a.round16) v = round_f16(v);
            xs[i] = v;
        }
        for (int i = tid; i < wsz; i += 256) {
            const int o = i / (CS_ICB * a.K);
            const int rem = i - o * CS_ICB * a.K;
            const int ic = rem / a.K, k = rem - ic * a.K;
            float v = 0.f;
            if (oc0 + o < a.OC && ic0 + ic < a.IC) v = a.w[((int64_t)(oc0 + o) * a.IC + ic0 + ic) * a.K + k];
            ws[i] = v;
        }
        __syncthreads();
        for (int ic = 0; ic < CS_ICB; ++ic) {
            for (int k = 0; k < a.K; ++k) {
                float wv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) wv[j] = ws[((ty * 4 + j) * CS_ICB + ic) * a.K + k];
                const float *xp = xs + ic * span + k * a.d;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float xv = xp[(tx + 16 * i) * a.s];
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv, wv[j], acc[i][j]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int oc = oc0 + ty * 4 + j;
        if (oc >= a.OC) continue;
        const float bias = a.bias ? a.bias[oc] : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t q = q0 + tx + 16 * i;
            if (q >= a.n_pos) continue;
            const int64_t orow = q * a.omul + a.oadd;
            if (orow < 0 || orow >= a.R_out) continue;
            float v = acc[i][j];
            if (a.bias) v = __fadd_rn(v, bias);
            if (a.resid) {
                const int64_t rr = a.resid_half ? (orow >> 1) : orow;
                v = __fadd_rn(a.resid[(int64_t)oc * a.R_resid + rr], v);
            }
            if (a.scale1 != 1.0f) v = __fmul_rn(v, a.scale1);
            float *o = a.out + (int64_t)oc * a.R_out + orow;
            if (a.accum) v = __fadd_rn(*o, v);
            if (a.scale2 != 1.0f) v = __fmul_rn(v, a.scale2);
            *o = v;
        }
    }
}

cudaError_t conv_simt_init() {
    return cudaFuncSetAttribute(k_conv_simt, cudaFuncAttributeMaxDynamicSharedMemorySize, CS_MAX_SMEM);
}

void conv_simt(const ConvArgs &a, cudaStream_t st) {
    const int span = (CS_BM - 1) * a.s + (a.K - 1) * a.d + 1;
    const size_t smem = sizeof(float) * ((size_t)CS_ICB * span + (size_t)CS_BN * CS_ICB * a.K);
    dim3 grid((unsigned)((a.n_pos + CS_BM - 1) / CS_BM), (a.OC + CS_BN - 1) / CS_BN);
    k_conv_simt<<<grid, 256, smem, st>>>(a);
}

}  // namespace kk
