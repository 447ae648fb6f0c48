// k_gemm.cu -- dequant-GEMM on CUDA cores (fp32) for token batches larger
// than the GEMV handles: y[m][n] (epi)= x[m][:] . W[n][:] (tensor.go:253-298).
//
// 64 tokens x 64 weight rows per CTA, K in steps of 64.  Each step, half the
// CTA decodes 64 rows x 64 elements of GGUF blocks into a shared fp32 tile
// (the exact dequant, so the products match the reference's operands) while
// the other half stages the activation tile; then every thread accumulates a
// 4x4 register tile.  A SwiGLU pair decodes both gate and up tiles.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "quant.cuh"

namespace acm {

constexpr int GB = 64;      // tile edge (tokens and rows)
constexpr int GK = 64;      // K step
constexpr int GPAD = 4;

template <int T, bool PAIR>
__global__ void __launch_bounds__(256) k_gemm_simt(const GemmDesc d) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    extern __shared__ __align__(16) float gsm[];
    float(*As)[GB + GPAD] = reinterpret_cast<float(*)[GB + GPAD]>(gsm);
    float(*Ws)[GK][GB + GPAD] = reinterpret_cast<float(*)[GK][GB + GPAD]>(gsm + GK * (GB + GPAD));
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int n0 = blockIdx.x * GB, m0 = blockIdx.y * GB;
    const int K = (int)d.k, N = (int)d.n, M = d.m;
    const int64_t rb = row_bytes(T, K);
    const uint8_t *w1 = static_cast<const uint8_t *>(d.w);
    const uint8_t *w2 = static_cast<const uint8_t *>(d.w2);
    float acc[4][4], acc2[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = acc2[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += GK) {
        // weight tiles: 64 rows x 2 runs of 32 per matrix
        {
            const int task = tid & 127, mat = tid >> 7;
            if (PAIR || mat == 0) {
                const int rr = task >> 1, run = (k0 >> 5) + (task & 1);
                const int n = n0 + rr;
                float v[32];
                if (n < N && run * 32 < K) {
                    dequant_run32<T>((mat ? w2 : w1) + (int64_t)n * rb, run, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = 0.f;
                }
                const int kk = (task & 1) * 32;
#pragma unroll
                for (int i = 0; i < 32; i++) Ws[PAIR ? mat : 0][kk + i][rr] = v[i];
            }
            if (!PAIR && mat == 1) {
                // activation tile: 64 tokens x 64 k, 128 threads x 32 floats
                const int mm = task >> 1, kk = (task & 1) * 32;
                const int m = m0 + mm;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (m < M && k0 + kk + i < K)
                        xv = *reinterpret_cast<const float4 *>(d.x + (int64_t)m * d.ldx + k0 + kk + i);
                    As[kk + i][mm] = xv.x;
                    As[kk + i + 1][mm] = xv.y;
                    As[kk + i + 2][mm] = xv.z;
                    As[kk + i + 3][mm] = xv.w;
                }
            }
        }
        if (PAIR) {
            for (int e = tid; e < GB * (GK / 4); e += 256) {
                const int mm = e / (GK / 4), kk = (e % (GK / 4)) * 4;
                const int m = m0 + mm;
                float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
                if (m < M && k0 + kk < K) xv = *reinterpret_cast<const float4 *>(d.x + (int64_t)m * d.ldx + k0 + kk);
                As[kk][mm] = xv.x;
                As[kk + 1][mm] = xv.y;
                As[kk + 2][mm] = xv.z;
                As[kk + 3][mm] = xv.w;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < GK; k++) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[k][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Ws[0][k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            if (PAIR) {
                const float4 c = *reinterpret_cast<const float4 *>(&Ws[1][k][tx * 4]);
                const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc2[i][j] = fmaf(av[i], cv[j], acc2[i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + tx * 4 + j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (d.bias) v += d.bias[n];
            float *yp = d.y + (int64_t)(d.yrow ? d.yrow[m] : m) * d.ldy + n;
            if (d.epi == EPI_ADD) {
                *yp += v;
            } else if (d.epi == EPI_SWIGLU) {
                const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-v)));
                *yp = __fmul_rn(__fmul_rn(v, sg), acc2[i][j]);
            } else {
                *yp = v;
            }
        }
    }
}

cudaError_t gemm_launch(const GemmDesc &d, cudaStream_t st) {
    if (!type_ok(d.type) || d.k % 32 || d.k % blk_elems(d.type) || d.m <= 0 || d.n <= 0 || (d.ldx % 4))
        return cudaErrorInvalidValue;
    const bool pair = d.w2 != nullptr;
    if (pair != (d.epi == EPI_SWIGLU)) return cudaErrorInvalidValue;
    dim3 grid((unsigned)((d.n + GB - 1) / GB), (unsigned)((d.m + GB - 1) / GB));
    const size_t smem = (size_t)(pair ? 3 : 2) * GK * (GB + GPAD) * sizeof(float);
    static std::atomic<bool> attr[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
#define ACM_GA(T)                                                                                       \
    cudaFuncSetAttribute(k_gemm_simt<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 << 10); \
    cudaFuncSetAttribute(k_gemm_simt<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 << 10);
        ACM_GA(T_F32) ACM_GA(T_F16) ACM_GA(T_Q4_0) ACM_GA(T_Q5_0) ACM_GA(T_Q8_0) ACM_GA(T_Q4_K) ACM_GA(T_Q5_K)
        ACM_GA(T_Q6_K)
#undef ACM_GA
        attr[dev & 63] = true;
    }
    switch (d.type) {
#define ACM_GM(T)                                                       \
    case T:                                                             \
        if (pair) launch_pdl(k_gemm_simt<T, true>, grid, dim3(256), smem, st, d);     \
        else launch_pdl(k_gemm_simt<T, false>, grid, dim3(256), smem, st, d);         \
        break;
        ACM_GM(T_F32) ACM_GM(T_F16) ACM_GM(T_Q4_0) ACM_GM(T_Q5_0) ACM_GM(T_Q8_0) ACM_GM(T_Q4_K) ACM_GM(T_Q5_K)
        ACM_GM(T_Q6_K)
#undef ACM_GM
    }
    return launched(1);
}

}  // namespace acm
