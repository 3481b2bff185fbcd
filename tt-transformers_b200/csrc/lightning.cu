// Linear attention with a fixed decay per head and a float32 matrix state per request.
//
//   q = silu(q'), k = silu(k'), v = silu(v')  (the projections' outputs, of the compute type)
//   S_t = decay_h S_(t-1) + k_t v_t^T   [dim, vdim];   o_t = S_t^T q_t
//
// lightning_scan: a warp owns LS_COLS columns of one head's state of one segment and walks the segment's tokens in
// order: lane l holds rows l, l + 32, ... of its columns in registers, so a token costs dim / 32 x LS_COLS multiply-adds
// per lane and LS_COLS warp sums. The state comes from the request's slot and goes back there after the last token
// (write_state 0: it is only read). Activations, products and the state are float32.
#include "common.cuh"

#define LS_COLS 8
#define LS_WARPS 4

__device__ __forceinline__ float ls_silu(float z) { return z / (1.f + expf(-z)); }

template <typename T, int NI>
__global__ void __launch_bounds__(LS_WARPS * 32)
lightning_scan_kernel(const T* __restrict__ proj, int ld, const int* __restrict__ cu_seqlens, const int* __restrict__ seg_slot,
                      float* __restrict__ state, const float* __restrict__ decay, float* __restrict__ out, int heads, int dim,
                      int vdim, int write_state) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int seg = blockIdx.z, head = blockIdx.y;
    const int c0 = (blockIdx.x * LS_WARPS + warp) * LS_COLS;
    if (c0 >= vdim) return;
    const int t_begin = cu_seqlens[seg], t_end = cu_seqlens[seg + 1];
    if (t_begin >= t_end) return;
    float* S = state + (((size_t)seg_slot[seg] * heads + head) * dim) * vdim;
    const float lambda = decay[head];
    float s[NI][LS_COLS];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
        const int d = lane + 32 * i;
#pragma unroll
        for (int c = 0; c < LS_COLS; ++c) s[i][c] = (d < dim && c0 + c < vdim) ? S[(size_t)d * vdim + c0 + c] : 0.f;
    }
    const int q_off = head * dim, k_off = heads * dim + head * dim, v_off = 2 * heads * dim + head * vdim + c0;
    for (int t = t_begin; t < t_end; ++t) {
        const T* row = proj + (size_t)t * ld;
        float q[NI], k[NI], v[LS_COLS];
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            const int d = lane + 32 * i;
            q[i] = d < dim ? ls_silu(to_float(row[q_off + d])) : 0.f;
            k[i] = d < dim ? ls_silu(to_float(row[k_off + d])) : 0.f;
        }
#pragma unroll
        for (int c = 0; c < LS_COLS; ++c) v[c] = c0 + c < vdim ? ls_silu(to_float(row[v_off + c])) : 0.f;
        float o[LS_COLS];
#pragma unroll
        for (int c = 0; c < LS_COLS; ++c) o[c] = 0.f;
#pragma unroll
        for (int i = 0; i < NI; ++i)
#pragma unroll
            for (int c = 0; c < LS_COLS; ++c) {
                s[i][c] = fmaf(lambda, s[i][c], k[i] * v[c]);
                o[c] = fmaf(s[i][c], q[i], o[c]);
            }
#pragma unroll
        for (int c = 0; c < LS_COLS; ++c) o[c] = warp_sum(o[c]);
        if (lane < LS_COLS && c0 + lane < vdim) {
            float mine = 0.f;
#pragma unroll
            for (int c = 0; c < LS_COLS; ++c)
                if (lane == c) mine = o[c];
            out[((size_t)t * heads + head) * vdim + c0 + lane] = mine;
        }
    }
    if (write_state) {
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            const int d = lane + 32 * i;
#pragma unroll
            for (int c = 0; c < LS_COLS; ++c)
                if (d < dim && c0 + c < vdim) S[(size_t)d * vdim + c0 + c] = s[i][c];
        }
    }
}

// proj [tokens, ld]: q [heads, dim] | k [heads, dim] | v [heads, vdim] | anything; state float32 [slots, heads, dim, vdim];
// out float32 [tokens, heads, vdim].
TTB_EXPORT int ttb_lightning_scan(const void* proj, int dtype, int ld, const int* cu_seqlens, const int* seg_slot, float* state,
                                  const float* decay, float* out, int segments, int heads, int dim, int vdim, int write_state,
                                  cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!proj || !cu_seqlens || !seg_slot || !state || !decay || !out) return TTB_ERR_ARGUMENT;
    if (dim < 1 || dim > 256 || vdim < 1 || heads < 1 || heads > 65535 || segments > 65535) return TTB_ERR_UNSUPPORTED;
    dim3 grid((vdim + LS_WARPS * LS_COLS - 1) / (LS_WARPS * LS_COLS), heads, segments);
    const int ni = (dim + 31) / 32;
#define LS_LAUNCH(T, NI)                                                                                              \
    ttb_launch(lightning_scan_kernel<T, NI>, grid, LS_WARPS * 32, 0, stream, (const T*)proj, ld, cu_seqlens, seg_slot, state, \
               decay, out, heads, dim, vdim, write_state)
#define LS_PICK(T)                                                                                                    \
    do {                                                                                                              \
        if (ni <= 1) LS_LAUNCH(T, 1); else if (ni <= 2) LS_LAUNCH(T, 2); else if (ni <= 4) LS_LAUNCH(T, 4); else LS_LAUNCH(T, 8); \
    } while (0)
    if (dtype == TTB_DTYPE_BF16) LS_PICK(__nv_bfloat16);
    else if (dtype == TTB_DTYPE_F32) LS_PICK(float);
    else return TTB_ERR_UNSUPPORTED;
#undef LS_PICK
#undef LS_LAUNCH
    return ttb_launch_status();
}
