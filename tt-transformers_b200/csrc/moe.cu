// A routed feed-forward: router, grouping of (token, choice) pairs by expert, both products of the experts over
// those groups, and the weighted sum per token.
//
// route_top: z = W_r h in float32 (one block per token; every logit is summed in the same order whatever the batch
//   holds); the `top` largest logits are chosen, the lower index among equals; their weights are the softmax over
//   the chosen logits only. An optional extra row of W_r gives the shared expert's gate sigmoid(w . h).
// moe_align: counts the pairs of every expert and lays their indices out expert by expert (one block; no host read).
// moe_group_gemm: C = A W_e^T over the rows of each expert, with float32 accumulation on the CUDA cores. FIRST:
//   rows are gathered from the tokens, W_e = [gate rows; up rows], and the epilogue writes
//   g' * sigmoid(alpha g') * (u' + 1) with g' = min(g, L), u' = clamp(u, -L, L). Otherwise: rows are the pairs'
//   hidden vectors and the result goes to the pair's own row, float32. A pair's numbers do not depend on which other
//   pairs share its tile.
// moe_combine: out[t] = sum_j weight[t, j] * pair_out[t, j] (+ gate[t] * shared[t]) in float32, in the order of j.
// glu_clamped: the same activation on a dense [rows, 2 inter] product (the shared expert).
#include "common.cuh"

#define RT_THREADS 128
#define RT_MAX_EXPERTS 1024

template <typename T>
__global__ void __launch_bounds__(RT_THREADS)
route_top_kernel(const T* __restrict__ x, int ldx, const float* __restrict__ w_router, int width, int experts, int top,
                 int shared, int* __restrict__ choice, float* __restrict__ weight, float* __restrict__ shared_gate) {
    extern __shared__ float rt_smem[];
    float* h = rt_smem;                   // [width]
    float* z = rt_smem + width;           // [experts + 1]
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    for (int c = threadIdx.x; c < width; c += RT_THREADS) h[c] = to_float(x[(size_t)t * ldx + c]);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int e = warp; e < experts + (shared ? 1 : 0); e += RT_THREADS / 32) {
        const float* w = w_router + (size_t)e * width;
        float s = 0.f;
        for (int c = lane; c < width; c += 32) s = fmaf(h[c], w[c], s);
        s = warp_sum(s);
        if (lane == 0) z[e] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float best_first = 0.f, denom = 0.f;
        for (int j = 0; j < top; ++j) {
            int best = -1;
            float best_z = -INFINITY;
            for (int e = 0; e < experts; ++e) {
                const float v = z[e];
                if (best < 0 || v > best_z) {
                    bool taken = false;
                    for (int i = 0; i < j; ++i) taken |= choice[(size_t)t * top + i] == e;
                    if (!taken) { best = e; best_z = v; }
                }
            }
            choice[(size_t)t * top + j] = best;
            if (j == 0) best_first = best_z;
            const float p = expf(best_z - best_first);
            weight[(size_t)t * top + j] = p;
            denom += p;
        }
        for (int j = 0; j < top; ++j) weight[(size_t)t * top + j] /= denom;
        if (shared) shared_gate[t] = 1.f / (1.f + expf(-z[experts]));
    }
}

TTB_EXPORT int ttb_route_top(const void* x, int dtype, int ldx, const float* w_router, int tokens, int width, int experts,
                             int top, int shared, int* choice, float* weight, float* shared_gate, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!x || !w_router || !choice || !weight || (shared && !shared_gate)) return TTB_ERR_ARGUMENT;
    if (experts < 1 || experts > RT_MAX_EXPERTS || top < 1 || top > experts) return TTB_ERR_UNSUPPORTED;
    const size_t smem = (size_t)(width + experts + 1) * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(route_top_kernel<__nv_bfloat16>, tokens, RT_THREADS, smem, stream, (const __nv_bfloat16*)x, ldx, w_router,
                   width, experts, top, shared, choice, weight, shared_gate);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(route_top_kernel<float>, tokens, RT_THREADS, smem, stream, (const float*)x, ldx, w_router, width, experts,
                   top, shared, choice, weight, shared_gate);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// ---------------------------------------------------------------- grouping
// offsets[e] .. offsets[e + 1]: where expert e's pairs lie in `sorted`; pairs of one expert in increasing order
// of their index (token * top + choice rank), so the layout is the same whenever the choices are.
__global__ void __launch_bounds__(1024)
moe_align_kernel(const int* __restrict__ choice, int pairs, int experts, int* __restrict__ offsets, int* __restrict__ sorted) {
    extern __shared__ int al_smem[];
    int* count = al_smem;                 // [experts + 1]
    pdl_wait();
    pdl_launch_dependents();
    for (int e = threadIdx.x; e <= experts; e += blockDim.x) count[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int e = choice[p];
        if ((unsigned)e < (unsigned)experts) atomicAdd(&count[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < experts; ++e) {
            const int c = count[e];
            count[e] = run;
            offsets[e] = run;
            run += c;
        }
        offsets[experts] = run;
    }
    __syncthreads();
    // one warp per expert walks the pairs in order and writes those of its expert (stable, no atomics)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int e = warp; e < experts; e += nwarps) {
        int at = count[e];
        for (int p0 = 0; p0 < pairs; p0 += 32) {
            const int p = p0 + lane;
            const bool mine = p < pairs && choice[p] == e;
            const unsigned ballot = __ballot_sync(0xffffffffu, mine);
            if (mine) sorted[at + __popc(ballot & ((1u << lane) - 1))] = p;
            at += __popc(ballot);
        }
    }
}

TTB_EXPORT int ttb_moe_align(const int* choice, int pairs, int experts, int* offsets, int* sorted, cudaStream_t stream) {
    if (pairs == 0) return TTB_OK;
    if (!choice || !offsets || !sorted || experts < 1 || experts > RT_MAX_EXPERTS) return TTB_ERR_ARGUMENT;
    ttb_launch(moe_align_kernel, 1, 1024, (size_t)(experts + 1) * sizeof(int), stream, choice, pairs, experts, offsets, sorted);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the experts' products (CUDA cores, float32 sums)
#define MG_BM 32
#define MG_BN 64
#define MG_BK 16
#define MG_THREADS 128

__device__ __forceinline__ float glu_clamped(float g, float u, float limit, float alpha) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
    return g / (1.f + expf(-alpha * g)) * (u + 1.f);
}

// Tile blockIdx.y of the pairs: walks the experts' groups in tiles of MG_BM rows. Returns false past the last tile.
__device__ __forceinline__ bool mg_find_tile(const int* offsets, int experts, int tile, int& expert, int& row0, int& row_end) {
    int seen = 0;
    for (int e = 0; e < experts; ++e) {
        const int begin = offsets[e], end = offsets[e + 1];
        const int tiles = (end - begin + MG_BM - 1) / MG_BM;
        if (tile < seen + tiles) {
            expert = e;
            row0 = begin + (tile - seen) * MG_BM;
            row_end = end;
            return true;
        }
        seen += tiles;
    }
    return false;
}

template <typename TA, typename TC, bool FIRST>
__global__ void __launch_bounds__(MG_THREADS)
moe_group_gemm_kernel(const TA* __restrict__ A, int lda, const TA* __restrict__ W, long long w_expert_stride, int ldw,
                      TC* __restrict__ C, int ldc, const int* __restrict__ offsets, const int* __restrict__ sorted,
                      int experts, int top, int N, int K, float limit, float alpha) {
    __shared__ float As[MG_BK][MG_BM + 4];
    __shared__ float Ws[MG_BK][MG_BN + 4];
    __shared__ float Us[FIRST ? MG_BK : 1][MG_BN + 4];
    __shared__ int src_row[MG_BM];
    pdl_wait();
    pdl_launch_dependents();
    int expert, row0, row_end;
    if (!mg_find_tile(offsets, experts, blockIdx.y, expert, row0, row_end)) return;
    const int n0 = blockIdx.x * MG_BN;
    if (threadIdx.x < MG_BM) {
        const int r = row0 + threadIdx.x;
        // FIRST: the row of A is the pair's token; otherwise the pair's place in the grouped order
        src_row[threadIdx.x] = r < row_end ? (FIRST ? sorted[r] / top : r) : -1;
    }
    __syncthreads();
    const TA* We = W + (size_t)expert * w_expert_stride;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;      // 16 x 8 threads, each 4 rows x 4 columns
    float acc[4][4], acc_u[FIRST ? 4 : 1][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[i][j] = 0.f;
            if (FIRST) acc_u[i][j] = 0.f;
        }
    for (int k0 = 0; k0 < K; k0 += MG_BK) {
        for (int i = threadIdx.x; i < MG_BM * MG_BK; i += MG_THREADS) {
            const int r = i / MG_BK, k = i % MG_BK;
            const int src = src_row[r];
            As[k][r] = (src >= 0 && k0 + k < K) ? to_float(A[(size_t)src * lda + k0 + k]) : 0.f;
        }
        for (int i = threadIdx.x; i < MG_BN * MG_BK; i += MG_THREADS) {
            const int n = i / MG_BK, k = i % MG_BK;
            const bool in = n0 + n < N && k0 + k < K;
            Ws[k][n] = in ? to_float(We[(size_t)(n0 + n) * ldw + k0 + k]) : 0.f;
            if (FIRST) Us[k][n] = in ? to_float(We[(size_t)(N + n0 + n) * ldw + k0 + k]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < MG_BK; ++kk) {
            float a[4], w[4], u[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w[j] = Ws[kk][tx * 4 + j];
                if (FIRST) u[j] = Us[kk][tx * 4 + j];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
                    if (FIRST) acc_u[i][j] = fmaf(a[i], u[j], acc_u[i][j]);
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = row0 + ty * 4 + i;
        if (r >= row_end) continue;
        const size_t dst = FIRST ? (size_t)r : (size_t)sorted[r];     // hidden rows in grouped order; results by pair
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= N) continue;
            if (FIRST) C[dst * ldc + n] = from_float<TC>(glu_clamped(acc[i][j], acc_u[i][j], limit, alpha));
            else C[dst * ldc + n] = from_float<TC>(acc[i][j]);
        }
    }
}

// first != 0: A = tokens [*, K], W = [experts, 2 N, K] (gate rows, then up rows), C = hidden [pairs, N] in the
// grouped order, type of A. first == 0: A = hidden [pairs, K], W = [experts, N, K], C = float32 [pairs, N] by pair.
TTB_EXPORT int ttb_moe_group_gemm(const void* A, int lda, const void* W, long long w_expert_stride, int ldw, void* C, int ldc,
                                  int dtype, int first, const int* offsets, const int* sorted, int pairs, int experts,
                                  int top, int N, int K, float limit, float alpha, cudaStream_t stream) {
    if (pairs == 0 || N == 0) return TTB_OK;
    if (!A || !W || !C || !offsets || !sorted || K < 1) return TTB_ERR_ARGUMENT;
    dim3 grid((N + MG_BN - 1) / MG_BN, (pairs + MG_BM - 1) / MG_BM + experts);
    if (grid.y > 65535) return TTB_ERR_UNSUPPORTED;
#define MG_LAUNCH(TA, TC, FIRST)                                                                                     \
    ttb_launch(moe_group_gemm_kernel<TA, TC, FIRST>, grid, MG_THREADS, 0, stream, (const TA*)A, lda, (const TA*)W,   \
               w_expert_stride, ldw, (TC*)C, ldc, offsets, sorted, experts, top, N, K, limit, alpha)
    if (dtype == TTB_DTYPE_BF16) {
        if (first) MG_LAUNCH(__nv_bfloat16, __nv_bfloat16, true); else MG_LAUNCH(__nv_bfloat16, float, false);
    } else if (dtype == TTB_DTYPE_F32) {
        if (first) MG_LAUNCH(float, float, true); else MG_LAUNCH(float, float, false);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
#undef MG_LAUNCH
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the weighted sum per token
template <typename TS>
__global__ void moe_combine_kernel(const float* __restrict__ pair_out, const float* __restrict__ weight, int top,
                                   const TS* __restrict__ shared_out, const float* __restrict__ shared_gate,
                                   float* __restrict__ out, int width) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const float sg = shared_out != nullptr ? shared_gate[t] : 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
        float s = 0.f;
        for (int j = 0; j < top; ++j) s = fmaf(weight[(size_t)t * top + j], pair_out[((size_t)t * top + j) * width + c], s);
        if (shared_out != nullptr) s = fmaf(sg, to_float(shared_out[(size_t)t * width + c]), s);
        out[(size_t)t * width + c] = s;
    }
}

TTB_EXPORT int ttb_moe_combine(const float* pair_out, const float* weight, int top, const void* shared_out, int shared_dtype,
                               const float* shared_gate, float* out, int tokens, int width, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!pair_out || !weight || !out || (shared_out && !shared_gate)) return TTB_ERR_ARGUMENT;
    if (shared_out && shared_dtype == TTB_DTYPE_BF16)
        ttb_launch(moe_combine_kernel<__nv_bfloat16>, tokens, 256, 0, stream, pair_out, weight, top,
                   (const __nv_bfloat16*)shared_out, shared_gate, out, width);
    else
        ttb_launch(moe_combine_kernel<float>, tokens, 256, 0, stream, pair_out, weight, top, (const float*)shared_out,
                   shared_gate, out, width);
    return ttb_launch_status();
}

// ---------------------------------------------------------------- the activation on a dense product
template <typename T>
__global__ void glu_clamped_kernel(const T* __restrict__ gate_up, T* __restrict__ out, int rows, int inter, float limit,
                                   float alpha) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t total = (size_t)rows * inter;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / inter, c = i % inter;
        out[i] = from_float<T>(glu_clamped(to_float(gate_up[r * 2 * inter + c]), to_float(gate_up[r * 2 * inter + inter + c]),
                                           limit, alpha));
    }
}

TTB_EXPORT int ttb_glu_clamped(const void* gate_up, void* out, int dtype, int rows, int inter, float limit, float alpha,
                               cudaStream_t stream) {
    if (rows == 0 || inter == 0) return TTB_OK;
    if (!gate_up || !out) return TTB_ERR_ARGUMENT;
    const size_t total = (size_t)rows * inter;
    const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(glu_clamped_kernel<__nv_bfloat16>, blocks, 256, 0, stream, (const __nv_bfloat16*)gate_up, (__nv_bfloat16*)out,
                   rows, inter, limit, alpha);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(glu_clamped_kernel<float>, blocks, 256, 0, stream, (const float*)gate_up, (float*)out, rows, inter, limit, alpha);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
