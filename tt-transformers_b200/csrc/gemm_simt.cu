// C[M, N] = A[M, K] * W[N, K]^T on the CUDA cores with float32 multiply-adds: the matrix
// product of the true 32-bit mode (no tensor-core or reduced-precision mode), and the
// fallback for bfloat16 shapes that the tensor-core kernels refuse. Any M, N, K.
// Every output element sums its K products in the same order whatever M is, so a
// token's result does not depend on the batch it is in.
#include "common.cuh"

#define GS_BM 64
#define GS_BN 64
#define GS_BK 16
#define GS_THREADS 256

__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
    const float4 r = *reinterpret_cast<const float4*>(p);
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(r.x << 16); v[1] = __uint_as_float(r.x & 0xffff0000u);
    v[2] = __uint_as_float(r.y << 16); v[3] = __uint_as_float(r.y & 0xffff0000u);
}

// VEC: K, lda and ldw are multiples of 4 and both bases are 16-byte aligned, so four
// consecutive k of a row can be fetched with one load.
template <typename TA, typename TC, bool VEC>
__global__ void __launch_bounds__(GS_THREADS)
gemm_simt_kernel(const TA* __restrict__ A, const TA* __restrict__ W, TC* __restrict__ C, int M, int N, int K,
                 int lda, int ldw, int ldc, long long batch_a = 0, long long batch_w = 0, long long batch_c = 0) {
    A += (size_t)blockIdx.z * batch_a;       // one product per blockIdx.z (a single product: one z, strides 0)
    W += (size_t)blockIdx.z * batch_w;
    C += (size_t)blockIdx.z * batch_c;
    __shared__ float As[GS_BK][GS_BM + 4];
    __shared__ float Ws[GS_BK][GS_BN + 4];
    const int m0 = blockIdx.y * GS_BM, n0 = blockIdx.x * GS_BN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;   // 16 x 16 threads, each a 4 x 4 patch
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    // loading: 64 rows x 16 k = 1024 elements per operand, 4 per thread
    const int load_row = threadIdx.x / 4;          // 0..63
    const int load_k = (threadIdx.x % 4) * 4;      // 0,4,8,12
    for (int k0 = 0; k0 < K; k0 += GS_BK) {
        const int am = m0 + load_row, wn = n0 + load_row;
        if (VEC) {
            float a[4] = {0.f, 0.f, 0.f, 0.f}, w[4] = {0.f, 0.f, 0.f, 0.f};
            if (am < M && k0 + load_k < K) load4(A + (size_t)am * lda + k0 + load_k, a);
            if (wn < N && k0 + load_k < K) load4(W + (size_t)wn * ldw + k0 + load_k, w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                As[load_k + e][load_row] = a[e];
                Ws[load_k + e][load_row] = w[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k = k0 + load_k + e;
                As[load_k + e][load_row] = (am < M && k < K) ? to_float(A[(size_t)am * lda + k]) : 0.f;
                Ws[load_k + e][load_row] = (wn < N && k < K) ? to_float(W[(size_t)wn * ldw + k]) : 0.f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < GS_BK; ++kk) {
            float a[4], w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) w[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N) C[(size_t)m * ldc + n] = from_float<TC>(acc[i][j]);
        }
    }
}

// in_dtype: type of A and W; out_dtype: type of C (float32 output from bfloat16 inputs is allowed).
TTB_EXPORT int ttb_gemm_simt(const void* A, const void* W, void* C, int in_dtype, int out_dtype, int M, int N, int K,
                             int lda, int ldw, int ldc, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!A || !W || !C || K < 1) return TTB_ERR_ARGUMENT;
    dim3 grid((N + GS_BN - 1) / GS_BN, (M + GS_BM - 1) / GS_BM);
    if (grid.y > 65535) return TTB_ERR_UNSUPPORTED;
    const bool vec = (K % 4 == 0) && (lda % 4 == 0) && (ldw % 4 == 0) && aligned16(A) && aligned16(W);
#define GS_LAUNCH(TA, TC)                                                                                          \
    do {                                                                                                           \
        if (vec) gemm_simt_kernel<TA, TC, true><<<grid, GS_THREADS, 0, stream>>>((const TA*)A, (const TA*)W, (TC*)C, M, N, K, lda, ldw, ldc); \
        else gemm_simt_kernel<TA, TC, false><<<grid, GS_THREADS, 0, stream>>>((const TA*)A, (const TA*)W, (TC*)C, M, N, K, lda, ldw, ldc);    \
    } while (0)
    if (in_dtype == TTB_DTYPE_F32 && out_dtype == TTB_DTYPE_F32) GS_LAUNCH(float, float);
    else if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_BF16) GS_LAUNCH(__nv_bfloat16, __nv_bfloat16);
    else if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_F32) GS_LAUNCH(__nv_bfloat16, float);
    else return TTB_ERR_UNSUPPORTED;
#undef GS_LAUNCH
    return ttb_launch_status();
}

// `batch` products at once: product b reads A + b * batch_a (rows lda apart), W + b * batch_w, and writes
// C + b * batch_c, all strides in elements. Per-head products (x[t, h, :] times W[h]) are this with batch_a the
// head stride of x and lda its token stride.
TTB_EXPORT int ttb_gemm_simt_batched(const void* A, const void* W, void* C, int in_dtype, int out_dtype, int batch, int M,
                                     int N, int K, int lda, int ldw, int ldc, long long batch_a, long long batch_w,
                                     long long batch_c, cudaStream_t stream) {
    if (M == 0 || N == 0 || batch == 0) return TTB_OK;
    if (!A || !W || !C || K < 1) return TTB_ERR_ARGUMENT;
    dim3 grid((N + GS_BN - 1) / GS_BN, (M + GS_BM - 1) / GS_BM, batch);
    if (grid.y > 65535 || batch > 65535) return TTB_ERR_UNSUPPORTED;
    const bool vec = (K % 4 == 0) && (lda % 4 == 0) && (ldw % 4 == 0) && (batch_a % 4 == 0) && (batch_w % 4 == 0) &&
                     aligned16(A) && aligned16(W);
#define GS_LAUNCH(TA, TC)                                                                                          \
    do {                                                                                                           \
        if (vec) gemm_simt_kernel<TA, TC, true><<<grid, GS_THREADS, 0, stream>>>((const TA*)A, (const TA*)W, (TC*)C, M, N, K, lda, ldw, ldc, batch_a, batch_w, batch_c); \
        else gemm_simt_kernel<TA, TC, false><<<grid, GS_THREADS, 0, stream>>>((const TA*)A, (const TA*)W, (TC*)C, M, N, K, lda, ldw, ldc, batch_a, batch_w, batch_c);    \
    } while (0)
    if (in_dtype == TTB_DTYPE_F32 && out_dtype == TTB_DTYPE_F32) GS_LAUNCH(float, float);
    else if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_BF16) GS_LAUNCH(__nv_bfloat16, __nv_bfloat16);
    else if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_F32) GS_LAUNCH(__nv_bfloat16, float);
    else return TTB_ERR_UNSUPPORTED;
#undef GS_LAUNCH
    return ttb_launch_status();
}
