// A gated linear recurrence per channel behind a short causal convolution, with its state per request.
//
// causal_conv: u[t, c] = b_c[c] + sum_j w[c, j] * x(t - taps + 1 + j, c), x(s, c) = round(x'[s, c] + b_x[c]) for tokens of
//   this step and the request's kept inputs (tail [slots, taps - 1, channels], oldest first; zeros at a request's start)
//   for positions before it. One thread per (RC_CONV_TOKENS tokens, channel) with the inputs it needs in registers;
//   nothing is written but u, so that every block sees the tail as the step before left it.
// gated_recurrence: one thread per (segment, channel) walks the segment's tokens in order:
//   a = exp(-rate[c] * sigmoid(gr + br));  S = a S + sqrt(1 - a^2) * sigmoid(gi + bi) * u;  out = S * gelu_tanh(y' + b_y)
//   with the gates' float32 pre-activations [tokens, blocks, 2 s] (decay rows, then input rows, per block). At the end
//   it stores S and the convolution's new tail (the last taps - 1 inputs of what the request has seen).
//   Long segments are cut into parts of part_len tokens that run side by side (blockIdx.z): the recurrence is linear in
//   S, so part p first (phase 1) walks its tokens from S = 0 and leaves (A_p, B_p) = (product of its a, its end state)
//   in scratch memory; then (phase 2) every part folds the parts before it into its start state, S = A_q S + B_q from
//   the request's kept state on, and walks its tokens again, this time writing out. Phase 0: one part, no scratch.
// Gates, decays, the state and the recurrence are float32.
#include "common.cuh"

#define RC_THREADS 128
#define RC_MAX_TAPS 16
#define RC_GROUP 8
#define RC_CONV_TOKENS 8

__device__ __forceinline__ float rc_gelu_tanh(float z) {
    return 0.5f * z * (1.f + tanhf(0.7978845608028654f * (z + 0.044715f * z * z * z)));
}

template <typename T>
__global__ void __launch_bounds__(RC_THREADS)
causal_conv_kernel(const T* __restrict__ x, int ldx, const float* __restrict__ bias_x, const float* __restrict__ w,
                   const float* __restrict__ bias_c, const int* __restrict__ seg_of_token, const int* __restrict__ cu_seqlens,
                   const int* __restrict__ seg_slot, const T* __restrict__ tail, T* __restrict__ u, int channels, int taps,
                   int tokens) {
    pdl_wait();
    pdl_launch_dependents();
    const int c = blockIdx.x * RC_THREADS + threadIdx.x;
    if (c >= channels) return;
    const int first = blockIdx.y * RC_CONV_TOKENS, last = min(first + RC_CONV_TOKENS, tokens);
    const float bx = bias_x[c], bc = bias_c[c];
    const float* w_row = w + (size_t)c * taps;
    // the tokens of one group may lie in several segments, so every tap checks its own segment's start; a segment's
    // start, end and slot are looked up again only when the group walks into the next segment; inputs that
    // neighbouring tokens share come from the first-level cache
    int seg = seg_of_token[first];
    int start = cu_seqlens[seg], end = cu_seqlens[seg + 1];
    const T* kept = tail + (size_t)seg_slot[seg] * (taps > 1 ? taps - 1 : 1) * channels;
    for (int t = first; t < last; ++t) {
        if (t >= end) {
            seg = seg_of_token[t];
            start = cu_seqlens[seg];
            end = cu_seqlens[seg + 1];
            kept = tail + (size_t)seg_slot[seg] * (taps > 1 ? taps - 1 : 1) * channels;
        }
        float acc = bc;
        for (int j = 0; j < taps; ++j) {
            const int s = t - (taps - 1) + j;                  // flat index of the input this tap reads
            float v;
            if (s >= start) v = to_float(from_float<T>(to_float(x[(size_t)s * ldx + c]) + bx));
            else v = to_float(kept[(size_t)((taps - 1) + (s - start)) * channels + c]);
            acc = fmaf(w_row[j], v, acc);
        }
        u[(size_t)t * channels + c] = from_float<T>(acc);
    }
}

template <typename T>
__global__ void __launch_bounds__(RC_THREADS)
gated_recurrence_kernel(const T* __restrict__ u, const float* __restrict__ gates, long long gate_ld_token,
                        long long gate_ld_block, const float* __restrict__ gate_bias,
                        const float* __restrict__ rate, const T* __restrict__ yx, int ldyx, const float* __restrict__ bias_yx,
                        const int* __restrict__ cu_seqlens, const int* __restrict__ seg_slot, float* __restrict__ state,
                        T* __restrict__ tail, T* __restrict__ out, int channels, int block_size, int taps, int write_state,
                        float* __restrict__ scratch, int part_len, int phase) {
    pdl_wait();
    pdl_launch_dependents();
    const int seg = blockIdx.y, c = blockIdx.x * RC_THREADS + threadIdx.x, part = blockIdx.z, parts = gridDim.z;
    if (c >= channels) return;
    const int seg_begin = cu_seqlens[seg], seg_end = cu_seqlens[seg + 1];
    const int t_begin = phase == 0 ? seg_begin : seg_begin + part * part_len;
    const int t_end = phase == 0 ? seg_end : min(seg_end, t_begin + part_len);
    if (t_begin >= t_end) return;
    const int slot = seg_slot[seg];
    const int b = c / block_size, i = c % block_size;
    const size_t g_r = (size_t)b * 2 * block_size + i, g_i = g_r + block_size;     // within a token's 2 * channels gates
    const float br = gate_bias[g_r], bi = gate_bias[g_i], k = rate[c], by = bias_yx[c];
    const float* gate_r = gates + (size_t)b * gate_ld_block + i;                   // the product may be strided by token and block
    const float* gate_i = gate_r + block_size;
    float S = 0.f, A = 1.f;
    if (phase == 0) S = state[(size_t)slot * channels + c];
    if (phase == 2) {
        // the state as phase 1 found it (the part that ends the segment overwrites the slot while others still start)
        S = scratch[(((size_t)seg * (parts + 1) + parts) * channels + c) * 2];
        for (int q = 0; q < part; ++q) {
            const float* ab = scratch + (((size_t)seg * (parts + 1) + q) * channels + c) * 2;
            S = fmaf(ab[0], S, ab[1]);
        }
    }
    // RC_GROUP tokens at a time: their loads are independent of the recurrence and in flight together
    for (int t0 = t_begin; t0 < t_end; t0 += RC_GROUP) {
        float gr[RC_GROUP], gi[RC_GROUP], uu[RC_GROUP], yy[RC_GROUP];
#pragma unroll
        for (int k2 = 0; k2 < RC_GROUP; ++k2) {
            const int t = min(t0 + k2, t_end - 1);
            gr[k2] = gate_r[(size_t)t * gate_ld_token];
            gi[k2] = gate_i[(size_t)t * gate_ld_token];
            uu[k2] = to_float(u[(size_t)t * channels + c]);
            yy[k2] = phase == 1 ? 0.f : to_float(yx[(size_t)t * ldyx + c]);
        }
#pragma unroll
        for (int k2 = 0; k2 < RC_GROUP; ++k2) {
            const int t = t0 + k2;
            if (t >= t_end) break;
            const float r = 1.f / (1.f + expf(-(gr[k2] + br))), in = 1.f / (1.f + expf(-(gi[k2] + bi)));
            const float a = expf(-k * r);
            const float mult = sqrtf(fmaxf(1.f - a * a, 0.f));
            S = fmaf(a, S, mult * (in * uu[k2]));
            if (phase == 1) {
                A *= a;
            } else {
                out[(size_t)t * channels + c] = from_float<T>(S * rc_gelu_tanh(yy[k2] + by));
            }
        }
    }
    if (phase == 1) {
        float* ab = scratch + (((size_t)seg * (parts + 1) + part) * channels + c) * 2;
        ab[0] = A;
        ab[1] = S;
        if (part == 0) scratch[(((size_t)seg * (parts + 1) + parts) * channels + c) * 2] = state[(size_t)slot * channels + c];
        return;
    }
    if (!write_state || t_end != seg_end) return;            // the part that holds the segment's last token keeps the state
    state[(size_t)slot * channels + c] = S;
    if (taps > 1) {
        // the kept inputs followed by this step's: the last taps - 1 of them stay
        const int keep = taps - 1, len = seg_end - seg_begin;
        const int t_begin = seg_begin;
        const float bx = bias_yx[channels + c];
        T* kept = tail + (size_t)slot * keep * channels;
        T fresh[RC_MAX_TAPS];
        for (int j = 0; j < keep; ++j) {
            const int at = len + j;                            // index in (kept ++ new)
            fresh[j] = at < keep ? kept[(size_t)at * channels + c]
                                 : from_float<T>(to_float(yx[(size_t)(t_begin + at - keep) * ldyx + channels + c]) + bx);
        }
        for (int j = 0; j < keep; ++j) kept[(size_t)j * channels + c] = fresh[j];
    }
}

// x: the convolution's input before its bias, [tokens, ldx] (a slice of a wider product); u: [tokens, channels].
TTB_EXPORT int ttb_causal_conv(const void* x, int dtype, int ldx, const float* bias_x, const float* w, const float* bias_c,
                               const int* seg_of_token, const int* cu_seqlens, const int* seg_slot, const void* tail, void* u,
                               int tokens, int channels, int taps, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!x || !bias_x || !w || !bias_c || !seg_of_token || !cu_seqlens || !seg_slot || !tail || !u) return TTB_ERR_ARGUMENT;
    if (taps < 1 || taps > RC_MAX_TAPS || channels < 1 || tokens > 65535 * RC_CONV_TOKENS) return TTB_ERR_UNSUPPORTED;
    dim3 grid((channels + RC_THREADS - 1) / RC_THREADS, (tokens + RC_CONV_TOKENS - 1) / RC_CONV_TOKENS);
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(causal_conv_kernel<__nv_bfloat16>, grid, RC_THREADS, 0, stream, (const __nv_bfloat16*)x, ldx, bias_x, w, bias_c,
                   seg_of_token, cu_seqlens, seg_slot, (const __nv_bfloat16*)tail, (__nv_bfloat16*)u, channels, taps, tokens);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(causal_conv_kernel<float>, grid, RC_THREADS, 0, stream, (const float*)x, ldx, bias_x, w, bias_c, seg_of_token,
                   cu_seqlens, seg_slot, (const float*)tail, (float*)u, channels, taps, tokens);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// yx [tokens, ldyx]: the gate branch's product in columns 0 .. channels-1, the convolution's input in the next `channels`;
// bias_yx [2 channels] likewise. gates float32 [tokens, blocks, 2 s] (per block: decay rows, input rows) with element
// strides gate_ld_token and gate_ld_block.
TTB_EXPORT int ttb_gated_recurrence(const void* u, int dtype, const float* gates, long long gate_ld_token, long long gate_ld_block,
                                    const float* gate_bias, const float* rate,
                                    const void* yx, int ldyx, const float* bias_yx, const int* cu_seqlens, const int* seg_slot,
                                    float* state, void* tail, void* out, int segments, int channels, int blocks, int taps,
                                    int write_state, float* scratch, int parts, int part_len, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!u || !gates || !gate_bias || !rate || !yx || !bias_yx || !cu_seqlens || !seg_slot || !state || !tail || !out)
        return TTB_ERR_ARGUMENT;
    if (taps < 1 || taps > RC_MAX_TAPS || blocks < 1 || channels % blocks || segments > 65535) return TTB_ERR_UNSUPPORTED;
    if (parts < 1 || parts > 65535 || (parts > 1 && (!scratch || part_len < 1))) return TTB_ERR_ARGUMENT;
    dim3 grid((channels + RC_THREADS - 1) / RC_THREADS, segments, parts);
    // parts > 1: scratch holds segments * (parts + 1) * channels * 2 floats; two launches
    for (int phase = parts > 1 ? 1 : 0; phase <= (parts > 1 ? 2 : 0); ++phase) {
        if (dtype == TTB_DTYPE_BF16)
            ttb_launch(gated_recurrence_kernel<__nv_bfloat16>, grid, RC_THREADS, 0, stream, (const __nv_bfloat16*)u, gates, gate_ld_token,
                       gate_ld_block, gate_bias, rate, (const __nv_bfloat16*)yx, ldyx, bias_yx, cu_seqlens, seg_slot, state,
                       (__nv_bfloat16*)tail, (__nv_bfloat16*)out, channels, channels / blocks, taps, write_state, scratch, part_len, phase);
        else if (dtype == TTB_DTYPE_F32)
            ttb_launch(gated_recurrence_kernel<float>, grid, RC_THREADS, 0, stream, (const float*)u, gates, gate_ld_token, gate_ld_block,
                       gate_bias, rate, (const float*)yx, ldyx, bias_yx, cu_seqlens, seg_slot, state, (float*)tail, (float*)out,
                       channels, channels / blocks, taps, write_state, scratch, part_len, phase);
        else return TTB_ERR_UNSUPPORTED;
    }
    return ttb_launch_status();
}

// ---------------------------------------------------------------- a decoded token: convolution, gates and recurrence in one kernel
// Every segment holds one token. A block owns one block of channels of one segment: its threads compute the
// convolution's output u for their channels (rounded to the compute type, as the kernels above hand it on) into shared
// memory and shift the kept inputs, its warps then sum the 2 s gate rows of the block's matrix against u in float32, and
// its threads walk the recurrence one step and write S * gelu_tanh(y).
#define RT_THREADS 256

template <typename T>
__global__ void __launch_bounds__(RT_THREADS)
recurrent_token_kernel(const T* __restrict__ yx, int ldyx, const float* __restrict__ bias_yx, const float* __restrict__ conv_w,
                       const float* __restrict__ conv_b, const T* __restrict__ w_gates, const float* __restrict__ gate_bias,
                       const float* __restrict__ rate, const int* __restrict__ cu_seqlens, const int* __restrict__ seg_slot,
                       float* __restrict__ state, T* __restrict__ tail, T* __restrict__ out, int channels, int block_size, int taps,
                       int write_state) {
    extern __shared__ float rt_smem[];
    float* u_s = rt_smem;                     // [block_size]
    float* g_s = rt_smem + block_size;        // [2 block_size]
    const int seg = blockIdx.y, b = blockIdx.x;
    const T* w_block = w_gates + (size_t)b * 2 * block_size * block_size;
    for (size_t off = (size_t)threadIdx.x * 128; off < (size_t)2 * block_size * block_size * sizeof(T); off += (size_t)RT_THREADS * 128)
        prefetch_l2(reinterpret_cast<const char*>(w_block) + off);      // weights: nobody writes them
    pdl_wait();
    pdl_launch_dependents();
    const int t = cu_seqlens[seg];
    if (cu_seqlens[seg + 1] <= t) return;
    const int slot = seg_slot[seg];
    const int keep = taps - 1;
    for (int i = threadIdx.x; i < block_size; i += RT_THREADS) {
        const int c = b * block_size + i;
        const float fresh = to_float(from_float<T>(to_float(yx[(size_t)t * ldyx + channels + c]) + bias_yx[channels + c]));
        T* kept = tail + (size_t)slot * (keep > 0 ? keep : 1) * channels;
        float window[RC_MAX_TAPS];
        for (int j = 0; j < keep; ++j) window[j] = to_float(kept[(size_t)j * channels + c]);
        float acc = conv_b[c];
        for (int j = 0; j < keep; ++j) acc = fmaf(conv_w[(size_t)c * taps + j], window[j], acc);
        acc = fmaf(conv_w[(size_t)c * taps + keep], fresh, acc);
        u_s[i] = to_float(from_float<T>(acc));
        if (write_state) {
            for (int j = 0; j + 1 < keep; ++j) kept[(size_t)j * channels + c] = from_float<T>(window[j + 1]);
            if (keep > 0) kept[(size_t)(keep - 1) * channels + c] = from_float<T>(fresh);
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = warp; o < 2 * block_size; o += RT_THREADS / 32) {
        const T* row = w_block + (size_t)o * block_size;
        float sum = 0.f;
        for (int k = lane; k < block_size; k += 32) sum = fmaf(to_float(row[k]), u_s[k], sum);
        sum = warp_sum(sum);
        if (lane == 0) g_s[o] = sum;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < block_size; i += RT_THREADS) {
        const int c = b * block_size + i;
        const float gr = g_s[i] + gate_bias[(size_t)b * 2 * block_size + i];
        const float gi = g_s[block_size + i] + gate_bias[(size_t)b * 2 * block_size + block_size + i];
        const float r = 1.f / (1.f + expf(-gr)), in = 1.f / (1.f + expf(-gi));
        const float a = expf(-rate[c] * r);
        const float S = fmaf(a, state[(size_t)slot * channels + c], sqrtf(fmaxf(1.f - a * a, 0.f)) * (in * u_s[i]));
        out[(size_t)t * channels + c] = from_float<T>(S * rc_gelu_tanh(to_float(yx[(size_t)t * ldyx + c]) + bias_yx[c]));
        if (write_state) state[(size_t)slot * channels + c] = S;
    }
}

// yx [tokens, ldyx] as for ttb_gated_recurrence; w_gates [blocks, 2 s, s] of the compute type; every segment holds one token.
TTB_EXPORT int ttb_recurrent_token(const void* yx, int dtype, int ldyx, const float* bias_yx, const float* conv_w, const float* conv_b,
                                   const void* w_gates, const float* gate_bias, const float* rate, const int* cu_seqlens,
                                   const int* seg_slot, float* state, void* tail, void* out, int segments, int channels, int blocks,
                                   int taps, int write_state, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!yx || !bias_yx || !conv_w || !conv_b || !w_gates || !gate_bias || !rate || !cu_seqlens || !seg_slot || !state || !tail || !out)
        return TTB_ERR_ARGUMENT;
    if (taps < 1 || taps > RC_MAX_TAPS || blocks < 1 || channels % blocks || segments > 65535 || blocks > 65535) return TTB_ERR_UNSUPPORTED;
    const int s = channels / blocks;
    const size_t smem = (size_t)3 * s * sizeof(float);
    if (smem > 48 * 1024) return TTB_ERR_UNSUPPORTED;
    dim3 grid(blocks, segments);
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(recurrent_token_kernel<__nv_bfloat16>, grid, RT_THREADS, smem, stream, (const __nv_bfloat16*)yx, ldyx, bias_yx, conv_w,
                   conv_b, (const __nv_bfloat16*)w_gates, gate_bias, rate, cu_seqlens, seg_slot, state, (__nv_bfloat16*)tail,
                   (__nv_bfloat16*)out, channels, s, taps, write_state);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(recurrent_token_kernel<float>, grid, RT_THREADS, smem, stream, (const float*)yx, ldyx, bias_yx, conv_w, conv_b,
                   (const float*)w_gates, gate_bias, rate, cu_seqlens, seg_slot, state, (float*)tail, (float*)out, channels, s, taps,
                   write_state);
    else return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
