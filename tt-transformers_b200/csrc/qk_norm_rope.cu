// Per-head RMS norm of queries and keys, rotation by position, and the write of keys and values into cache pages,
// for attention whose keys and values may differ in size.
//
// qkv [tokens, heads * dim | kv_heads * dim | kv_heads * vdim] of the compute type. One warp per (token, head unit),
// four of them a block:
//   query head:  q = rms(q) * w_q (optional), rotated, written back in place
//   key head:    k = rms(k) * w_k (optional), rotated, written back in place and into its page row
//   value head:  copied into its page row
// The norm is over `dim` with eps inside the root and one weight vector shared by all heads; the rotation pairs
// element i with i + rotary_dim / 2 for i < rotary_dim / 2 (angle = position * inv_freq[i], sincosf on float32) and
// leaves the other elements alone. Pages: keys [pages, kv_heads, page_size, dim], values [.., vdim].
#include "common.cuh"

#define QN_THREADS 128

template <typename T>
__global__ void __launch_bounds__(QN_THREADS)
qk_norm_rope_write_kernel(T* __restrict__ qkv, int ld, const int* __restrict__ positions, const int* __restrict__ seg_of_token,
                          const float* __restrict__ q_weight, const float* __restrict__ k_weight, float eps,
                          const float* __restrict__ inv_freq, int rotary_dim, int heads, int kv_heads, int dim, int vdim,
                          T* __restrict__ key_pages, T* __restrict__ value_pages, const int* __restrict__ block_table,
                          int table_width, int page_size, int num_pages, int write_kv, int* __restrict__ status) {
    extern __shared__ float qn_rows[];         // [warps][dim]
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x, unit = blockIdx.y * (QN_THREADS / 32) + warp;
    if (unit >= heads + 2 * kv_heads) return;
    float* qn_row = qn_rows + warp * dim;
    const int pos = positions[t];
    const bool is_q = unit < heads, is_k = !is_q && unit < heads + kv_heads;
    const int g = is_q ? unit : (is_k ? unit - heads : unit - heads - kv_heads);
    T* dst_page = nullptr;
    if (!is_q) {
        if (!write_kv) {
            if (!is_k) return;
        } else {
            const int page_index = pos / page_size;
            int page = -1;
            if (page_index >= table_width) {
                if (lane == 0) atomicExch(status, 0x1000000 + t);
            } else {
                page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
                if ((unsigned)page >= (unsigned)num_pages) {
                    if (lane == 0) atomicExch(status, 0x2000000 + t);
                    page = -1;
                }
            }
            if (page >= 0) {
                const size_t row = ((size_t)page * kv_heads + g) * page_size + pos % page_size;
                dst_page = is_k ? key_pages + row * dim : value_pages + row * vdim;
            }
        }
    }
    if (!is_q && !is_k) {                       // a value head: a copy
        const T* src = qkv + (size_t)t * ld + (size_t)(heads + kv_heads) * dim + (size_t)g * vdim;
        if (dst_page != nullptr)
            for (int d = lane; d < vdim; d += 32) dst_page[d] = src[d];
        return;
    }
    T* row = qkv + (size_t)t * ld + (size_t)(is_q ? g : heads + g) * dim;
    const float* weight = is_q ? q_weight : k_weight;
    float sumsq = 0.f;
    for (int d = lane; d < dim; d += 32) {
        const float v = to_float(row[d]);
        qn_row[d] = v;
        sumsq += v * v;
    }
    if (weight != nullptr) {
        sumsq = warp_sum(sumsq);
        const float scale = 1.f / sqrtf(sumsq / (float)dim + eps);
        for (int d = lane; d < dim; d += 32) qn_row[d] = qn_row[d] * scale * weight[d];
    }
    __syncwarp();
    const int half = rotary_dim / 2;
    for (int d = lane; d < dim; d += 32) {
        float v = qn_row[d];
        if (d < rotary_dim) {
            const int i = d < half ? d : d - half;
            float sn, cs;
            sincosf((float)pos * inv_freq[i], &sn, &cs);
            v = d < half ? qn_row[d] * cs - qn_row[d + half] * sn : qn_row[d] * cs + qn_row[d - half] * sn;
        }
        const T rounded = from_float<T>(v);
        row[d] = rounded;
        if (dst_page != nullptr) dst_page[d] = rounded;
    }
}

TTB_EXPORT int ttb_qk_norm_rope_write(void* qkv, int dtype, int ld, const int* positions, const int* seg_of_token,
                                      const float* q_weight, const float* k_weight, float eps, const float* inv_freq,
                                      int rotary_dim, int tokens, int heads, int kv_heads, int dim, int vdim, void* key_pages,
                                      void* value_pages, const int* block_table, int table_width, int page_size, int num_pages,
                                      int write_kv, int* status, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!qkv || !positions || !seg_of_token || !status) return TTB_ERR_ARGUMENT;
    if (write_kv && (!key_pages || !value_pages || !block_table || page_size < 1)) return TTB_ERR_ARGUMENT;
    if (rotary_dim < 0 || (rotary_dim & 1) || rotary_dim > dim || (rotary_dim > 0 && !inv_freq)) return TTB_ERR_ARGUMENT;
    if (dim < 1 || vdim < 1 || heads + 2 * kv_heads > 65535) return TTB_ERR_UNSUPPORTED;
    dim3 grid(tokens, (heads + 2 * kv_heads + QN_THREADS / 32 - 1) / (QN_THREADS / 32));
    const size_t smem = (size_t)(QN_THREADS / 32) * dim * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(qk_norm_rope_write_kernel<__nv_bfloat16>, grid, QN_THREADS, smem, stream, (__nv_bfloat16*)qkv, ld, positions,
                   seg_of_token, q_weight, k_weight, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, (__nv_bfloat16*)key_pages,
                   (__nv_bfloat16*)value_pages, block_table, table_width, page_size, num_pages, write_kv, status);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(qk_norm_rope_write_kernel<float>, grid, QN_THREADS, smem, stream, (float*)qkv, ld, positions, seg_of_token,
                   q_weight, k_weight, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, (float*)key_pages, (float*)value_pages,
                   block_table, table_width, page_size, num_pages, write_kv, status);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
