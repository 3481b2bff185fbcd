// A router that scores all experts and may choose from the best groups only.
//
//   z = W_r h (float32);  s = softmax(z) over all experts
//   experts form `groups` equal groups of neighbours; a group's score is its largest s; the `keep` groups with the
//   largest scores stay (the lower index among equals), the others' experts cannot be chosen
//   the `top` largest s among the rest are chosen (the lower index among equals)
//   weight_j = s_j / (sum of the chosen s + floor)
//
// Rows whose scores are not numbers (padded rows of a captured step) get scores of zero and choose the first experts.
// RG_TOKENS tokens a block (eight in prompt portions, one in decode steps) share one pass over W_r; a warp per logit row, then a warp per token selects. Every logit is
// summed in the same order whatever else the batch holds (a lane takes four neighbouring columns at a time where the width
// allows 16-byte loads, in prompt portions and in decode steps alike).
#include "common.cuh"

#define RG_MAX_EXPERTS 1024

template <typename T, int RG_TOKENS>
__global__ void __launch_bounds__(512)
route_grouped_kernel(const T* __restrict__ x, int ldx, const float* __restrict__ w_router, int width, int experts, int top,
                     int groups, int keep, float floor_, int* __restrict__ choice, float* __restrict__ weight, int tokens) {
    extern __shared__ __align__(16) float rg_smem[];
    const int wpad = (width + 3) & ~3;
    float* h = rg_smem;                                   // [RG_TOKENS, wpad]
    float* z = h + RG_TOKENS * wpad;                      // [RG_TOKENS, experts]: logits, then scores
    int* open = reinterpret_cast<int*>(z + RG_TOKENS * experts);     // [RG_TOKENS, experts]: 1 while an expert may be chosen
    float* gbest = reinterpret_cast<float*>(open + RG_TOKENS * experts);     // [RG_TOKENS, groups]
    if (RG_TOKENS == 1) {      // a handful of tokens: the router's matrix on its way into L2 while the norm in front finishes
        const char* w = reinterpret_cast<const char*>(w_router);
        const size_t bytes = (size_t)experts * width * sizeof(float);
        for (size_t off = (size_t)(blockIdx.x * blockDim.x + threadIdx.x) * 128; off < bytes; off += (size_t)gridDim.x * blockDim.x * 128)
            prefetch_l2(w + off);
    }
    pdl_wait();
    pdl_launch_dependents();
    const int t0 = blockIdx.x * RG_TOKENS, nt = min(RG_TOKENS, tokens - t0);
    for (int i = 0; i < RG_TOKENS; ++i)
        for (int c = threadIdx.x; c < wpad; c += blockDim.x)
            h[i * wpad + c] = (i < nt && c < width) ? to_float(x[(size_t)(t0 + i) * ldx + c]) : 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const bool vec = (width & 3) == 0 && (reinterpret_cast<uintptr_t>(w_router) & 15) == 0;
    for (int e = warp; e < experts; e += nwarps) {
        const float* w = w_router + (size_t)e * width;
        float s[RG_TOKENS];
#pragma unroll
        for (int i = 0; i < RG_TOKENS; ++i) s[i] = 0.f;
        if (vec) {          // a lane's loads are independent of one another: they are in flight together
#pragma unroll 4
            for (int c = lane * 4; c < width; c += 128) {
                const float4 a = *reinterpret_cast<const float4*>(w + c);
#pragma unroll
                for (int i = 0; i < RG_TOKENS; ++i) {
                    const float4 x4 = *reinterpret_cast<const float4*>(h + i * wpad + c);
                    s[i] = fmaf(a.x, x4.x, s[i]); s[i] = fmaf(a.y, x4.y, s[i]); s[i] = fmaf(a.z, x4.z, s[i]); s[i] = fmaf(a.w, x4.w, s[i]);
                }
            }
        } else {
            for (int c = lane; c < width; c += 32) {
                const float a = w[c];
#pragma unroll
                for (int i = 0; i < RG_TOKENS; ++i) s[i] = fmaf(h[i * wpad + c], a, s[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < RG_TOKENS; ++i) {
            const float r = warp_sum(s[i]);
            if (lane == 0) z[i * experts + e] = r;
        }
    }
    __syncthreads();
    const int per_group = experts / groups;
    for (int i = warp; i < nt; i += nwarps) {
        float* zt = z + i * experts;
        int* op = open + i * experts;
        float* gb = gbest + i * groups;
        // softmax over all experts
        float top_z = -INFINITY;
        for (int e = lane; e < experts; e += 32) top_z = fmaxf(top_z, zt[e]);
        top_z = warp_max(top_z);
        float total = 0.f;
        for (int e = lane; e < experts; e += 32) total += expf(zt[e] - top_z);
        total = warp_sum(total);
        for (int e = lane; e < experts; e += 32) {
            const float sv = expf(zt[e] - top_z) / total;
            zt[e] = sv == sv ? sv : 0.f;          // a row that is not a number (a padded row on nobody's state) still chooses valid experts
        }
        __syncwarp();
        // the groups' scores; the best `keep` of them stay open
        for (int g = lane; g < groups; g += 32) {
            float best = -INFINITY;
            for (int e = g * per_group; e < (g + 1) * per_group; ++e) best = fmaxf(best, zt[e]);
            gb[g] = best;
        }
        for (int e = lane; e < experts; e += 32) op[e] = 0;
        __syncwarp();
        for (int j = 0; j < keep; ++j) {
            float best_s = -INFINITY;
            int best = 0x7fffffff;
            for (int g = lane; g < groups; g += 32) {
                const float v = gb[g];
                if (v >= 0.f && (best == 0x7fffffff || v > best_s)) { best = g; best_s = v; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float os = __shfl_xor_sync(0xffffffffu, best_s, o);
                const int og = __shfl_xor_sync(0xffffffffu, best, o);
                if (og != 0x7fffffff && (best == 0x7fffffff || os > best_s || (os == best_s && og < best))) { best = og; best_s = os; }
            }
            if (best != 0x7fffffff) {
                if (lane == 0) gb[best] = -1.f;                 // taken (scores are never negative)
                for (int e = best * per_group + lane; e < (best + 1) * per_group; e += 32) op[e] = 1;
            }
            __syncwarp();
        }
        // the `top` largest scores among the open experts
        float denom = 0.f;
        const int t = t0 + i;
        for (int j = 0; j < top; ++j) {
            float best_s = -INFINITY;
            int best = 0x7fffffff;
            for (int e = lane; e < experts; e += 32) {
                if (!op[e]) continue;
                const float v = zt[e];
                if (best == 0x7fffffff || v > best_s) { best = e; best_s = v; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float os = __shfl_xor_sync(0xffffffffu, best_s, o);
                const int oe = __shfl_xor_sync(0xffffffffu, best, o);
                if (oe != 0x7fffffff && (best == 0x7fffffff || os > best_s || (os == best_s && oe < best))) { best = oe; best_s = os; }
            }
            if (best == 0x7fffffff) best = 0;                   // cannot happen: keep * per_group >= top; never index with it
            if (lane == 0) {
                op[best] = 0;
                choice[(size_t)t * top + j] = best;
                weight[(size_t)t * top + j] = best_s;          // divided by the sum below
            }
            denom += best_s;
            __syncwarp();
        }
        for (int j = lane; j < top; j += 32) weight[(size_t)t * top + j] /= (denom + floor_);
    }
}

TTB_EXPORT int ttb_route_grouped(const void* x, int dtype, int ldx, const float* w_router, int tokens, int width, int experts,
                                 int top, int groups, int keep, float floor_, int* choice, float* weight, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!x || !w_router || !choice || !weight) return TTB_ERR_ARGUMENT;
    if (experts < 1 || experts > RG_MAX_EXPERTS || top < 1 || top > experts || groups < 1 || experts % groups || keep < 1 ||
        keep > groups || keep * (experts / groups) < top)
        return TTB_ERR_UNSUPPORTED;
    const int per_block = tokens > 64 ? 8 : 1;
    const size_t smem = ((size_t)per_block * (((width + 3) & ~3) + 2 * experts + groups)) * sizeof(float);
    if (smem > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    const int warps = experts < 4 ? 4 : (experts > 16 ? 16 : experts);
#define RG_LAUNCH(T, N)                                                                                               \
    do {                                                                                                              \
        static TtbOncePerDevice once;                                                                                 \
        if (smem > 48 * 1024 && once.pending()) {                                                                     \
            cudaFuncSetAttribute(route_grouped_kernel<T, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
            once.mark();                                                                                              \
        }                                                                                                             \
        ttb_launch(route_grouped_kernel<T, N>, (tokens + N - 1) / N, warps * 32, smem, stream, (const T*)x, ldx,      \
                   w_router, width, experts, top, groups, keep, floor_, choice, weight, tokens);                      \
    } while (0)
    if (dtype == TTB_DTYPE_BF16) { if (per_block == 8) RG_LAUNCH(__nv_bfloat16, 8); else RG_LAUNCH(__nv_bfloat16, 1); }
    else if (dtype == TTB_DTYPE_F32) { if (per_block == 8) RG_LAUNCH(float, 8); else RG_LAUNCH(float, 1); }
    else return TTB_ERR_UNSUPPORTED;
#undef RG_LAUNCH
    return ttb_launch_status();
}
