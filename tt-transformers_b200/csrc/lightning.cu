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
    if (dim < 1 || dim > 512 || vdim < 1 || heads < 1 || heads > 65535 || segments > 65535) return TTB_ERR_UNSUPPORTED;
    dim3 grid((vdim + LS_WARPS * LS_COLS - 1) / (LS_WARPS * LS_COLS), heads, segments);
    const int ni = (dim + 31) / 32;
#define LS_LAUNCH(T, NI)                                                                                              \
    ttb_launch(lightning_scan_kernel<T, NI>, grid, LS_WARPS * 32, 0, stream, (const T*)proj, ld, cu_seqlens, seg_slot, state, \
               decay, out, heads, dim, vdim, write_state)
#define LS_PICK(T)                                                                                                    \
    do {                                                                                                              \
        if (ni <= 1) LS_LAUNCH(T, 1); else if (ni <= 2) LS_LAUNCH(T, 2); else if (ni <= 4) LS_LAUNCH(T, 4); else if (ni <= 8) LS_LAUNCH(T, 8); else LS_LAUNCH(T, 16); \
    } while (0)
    if (dtype == TTB_DTYPE_BF16) LS_PICK(__nv_bfloat16);
    else if (dtype == TTB_DTYPE_F32) LS_PICK(float);
    else return TTB_ERR_UNSUPPORTED;
#undef LS_PICK
#undef LS_LAUNCH
    return ttb_launch_status();
}

// ---------------------------------------------------------------- prompt portions: the same recurrence, chunk by chunk
// For a chunk of C tokens that starts from the state S0 (L = decay):
//   o_i   = L^(i+1) S0^T q_i + sum_(j<=i) L^(i-j) (q_i . k_j) v_j
//   S_new = L^C S0 + sum_j L^(C-1-j) k_j v_j^T
// which is four small matrix products per chunk on the tensor cores (bfloat16 operands, float32 sums):
// A = Q K^T, Q S0, A' V and K^T V'. q, k and v are the activations rounded to bfloat16, as they leave the projection.
// Everything that carries a decay or the state is float32 and enters its product as a sum of two bfloat16 numbers
// (v = hi + lo with hi = bf16(v), lo = bf16(v - hi): sixteen bits of mantissa, 2^-17 relative), each half with a
// product of its own: A' = A * L^(i-j), V' = V * L^(C-1-j) and S0. The state itself stays float32 in shared memory
// for the whole segment. A block owns LC_VS columns of one head's state of one segment and walks its chunks in order.
// Long segments are cut into parts of part_len tokens (a multiple of the chunk) that run side by side (blockIdx.x):
// the recurrence is linear in S, so in phase 1 every part walks its chunks from S = 0, keys and values only, and leaves
// its end state in scratch memory; a small kernel turns the end states into start states, part by part
// (S_start[0] = the request's kept state, S_start[p + 1] = decay^part_len S_start[p] + S_end[p]); in phase 2 every part
// walks its chunks again from its start state, now with the queries. Phase 0: one part, no scratch.
#include <mma.h>
using namespace nvcuda;

#define LC_C 64
#define LC_VS 32
#define LC_THREADS 256
#define LC_BATCH 8

struct LcLayout {
    int ldq, ldv, lda_f, lda_h, lds_f, lds_h, ldo;
    size_t q, k, v, vh, vl, af, ah, al, sf, sh, sl, of, pw, total;
};

static __host__ __device__ inline LcLayout lc_layout(int dim) {
    LcLayout L;
    L.ldq = dim + 8; L.ldv = LC_VS + 8; L.lda_f = LC_C + 4; L.lda_h = LC_C + 8; L.lds_f = LC_VS + 4; L.lds_h = LC_VS + 8;
    L.ldo = LC_VS + 4;
    size_t at = 0;
    L.q = at; at += (size_t)LC_C * L.ldq * 2;
    L.k = at; at += (size_t)LC_C * L.ldq * 2;
    L.v = at; at += (size_t)LC_C * L.ldv * 2;
    L.vh = at; at += (size_t)LC_C * L.ldv * 2;
    L.vl = at; at += (size_t)LC_C * L.ldv * 2;
    L.af = at; at += (size_t)LC_C * L.lda_f * 4;
    L.ah = at; at += (size_t)LC_C * L.lda_h * 2;
    L.al = at; at += (size_t)LC_C * L.lda_h * 2;
    L.sf = at; at += (size_t)dim * L.lds_f * 4;
    L.sh = at; at += (size_t)dim * L.lds_h * 2;
    L.sl = at; at += (size_t)dim * L.lds_h * 2;
    L.of = at; at += (size_t)LC_C * L.ldo * 4;
    L.pw = at; at += (size_t)(LC_C + 4) * 4;
    L.total = at;
    return L;
}

// silu for values that are rounded to bfloat16 next: the fast exponential and division (two units in the last place
// of float32 each) are far below that rounding
__device__ __forceinline__ float lc_silu(float z) { return __fdividef(z, 1.f + __expf(-z)); }

__device__ __forceinline__ void lc_split(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

__global__ void __launch_bounds__(LC_THREADS)
lightning_chunk_kernel(const __nv_bfloat16* __restrict__ proj, int ld, const int* __restrict__ cu_seqlens,
                       const int* __restrict__ seg_slot, float* __restrict__ state, const float* __restrict__ decay,
                       float* __restrict__ out, int heads, int dim, int vdim, int write_state, float* __restrict__ scratch,
                       int part_len, int parts, int phase) {
    extern __shared__ __align__(128) unsigned char lc_smem[];
    const LcLayout L = lc_layout(dim);
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.q);
    __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.k);
    __nv_bfloat16* Vs = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.v);
    __nv_bfloat16* Vh = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.vh);
    __nv_bfloat16* Vl = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.vl);
    float* Af = reinterpret_cast<float*>(lc_smem + L.af);
    __nv_bfloat16* Ah = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.ah);
    __nv_bfloat16* Al = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.al);
    float* Sf = reinterpret_cast<float*>(lc_smem + L.sf);
    __nv_bfloat16* Sh = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.sh);
    __nv_bfloat16* Sl = reinterpret_cast<__nv_bfloat16*>(lc_smem + L.sl);
    float* Of = reinterpret_cast<float*>(lc_smem + L.of);
    float* pw = reinterpret_cast<float*>(lc_smem + L.pw);           // pw[x] = decay^x, x = 0 .. LC_C

    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5;
    const int seg = blockIdx.z, head = blockIdx.y, part = blockIdx.x % parts, c0 = (blockIdx.x / parts) * LC_VS;
    const int seg_begin = cu_seqlens[seg], seg_end = cu_seqlens[seg + 1];
    const int t_begin = seg_begin + part * part_len;
    const int t_end = phase == 0 ? seg_end : min(seg_end, t_begin + part_len);
    if (t_begin >= t_end) return;
    float* S = state + (((size_t)seg_slot[seg] * heads + head) * dim) * vdim;
    // scratch: [segment, head, part 0 .. parts (the last one: the state the request came with), dim, vdim]
    float* parts_S = scratch + ((size_t)seg * heads + head) * (parts + 1) * dim * vdim;
    const float lambda = decay[head];
    for (int x = tid; x <= LC_C; x += LC_THREADS) pw[x] = x == 0 ? 1.f : powf(lambda, (float)x);
    const int lane = tid & 31;
    for (int d = warp; d < dim; d += LC_THREADS / 32) {
        float v = 0.f;
        if (c0 + lane < vdim) {
            const size_t at = (size_t)d * vdim + c0 + lane;
            if (phase == 0) v = S[at];
            else if (phase == 2) v = parts_S[(size_t)part * dim * vdim + at];      // the part's start state (lightning_prefix_kernel)
        }
        Sf[d * L.lds_f + lane] = v;
    }
    const int q_off = head * dim, k_off = heads * dim + head * dim, v_off = 2 * heads * dim + head * vdim + c0;
    const int d_tiles = dim / 16;
    __syncthreads();

    for (int chunk0 = t_begin; chunk0 < t_end; chunk0 += LC_C) {
        const int n = min(LC_C, t_end - chunk0);
        // ---- the chunk's activations, rounded to bfloat16; rows past the chunk's end are zero; the state in two halves
        // sixteen bytes (eight values) a load, all loads of a batch in flight before the first is used: a row's q and k
        // are 2 * dim / 8 such units, a row's LC_VS values four, one unit a thread
        {
            const int vi = tid >> 2, vj = tid & 3;
            uint4 v_raw = make_uint4(0u, 0u, 0u, 0u);
            if (vi < n && c0 + vj * 8 < vdim) v_raw = *reinterpret_cast<const uint4*>(proj + (size_t)(chunk0 + vi) * ld + v_off + vj * 8);
            const int q_units = dim >> 3, row_units = dim >> 2, total = LC_C * row_units;
            const int row_shift = (row_units & (row_units - 1)) == 0 ? __ffs(row_units) - 1 : -1;      // a shift where it can be
            for (int base = 0; base < total; base += LC_THREADS * LC_BATCH) {
                uint4 raw[LC_BATCH];
#pragma unroll
                for (int r = 0; r < LC_BATCH; ++r) {
                    const int u = base + r * LC_THREADS + tid;
                    raw[r] = make_uint4(0u, 0u, 0u, 0u);
                    if (u < total) {
                        const int i = row_shift >= 0 ? u >> row_shift : u / row_units, j = u - i * row_units;
                        const bool is_q = j < q_units;
                        if (i < n && !(is_q && phase == 1))
                            raw[r] = *reinterpret_cast<const uint4*>(proj + (size_t)(chunk0 + i) * ld +
                                                                     (is_q ? q_off + j * 8 : k_off + (j - q_units) * 8));
                    }
                }
#pragma unroll
                for (int r = 0; r < LC_BATCH; ++r) {
                    const int u = base + r * LC_THREADS + tid;
                    if (u >= total) continue;
                    const int i = row_shift >= 0 ? u >> row_shift : u / row_units, j = u - i * row_units;
                    const bool is_q = j < q_units;
                    if (is_q && phase == 1) continue;               // phase 1 walks keys and values only
                    float f[8];
                    const uint32_t w[4] = {raw[r].x, raw[r].y, raw[r].z, raw[r].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        f[2 * e] = lc_silu(__uint_as_float(w[e] << 16));
                        f[2 * e + 1] = lc_silu(__uint_as_float(w[e] & 0xffff0000u));
                    }
                    store8((is_q ? Qs : Ks) + i * L.ldq + (is_q ? j : j - q_units) * 8, f);
                }
            }
            const uint32_t w[4] = {v_raw.x, v_raw.y, v_raw.z, v_raw.w};
            const float share = vi < n ? pw[n - 1 - vi] : 0.f;       // the value's share of the new state: v_j * decay^(n - 1 - j)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float raw_v = __uint_as_float((e & 1) ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
                const __nv_bfloat16 vb = __float2bfloat16_rn(lc_silu(raw_v));
                const int c = vj * 8 + e;
                Vs[vi * L.ldv + c] = vb;
                lc_split(__bfloat162float(vb) * share, Vh[vi * L.ldv + c], Vl[vi * L.ldv + c]);
            }
        }
        for (int d = warp; phase != 1 && d < dim; d += LC_THREADS / 32)
            lc_split(Sf[d * L.lds_f + lane], Sh[d * L.lds_h + lane], Sl[d * L.lds_h + lane]);
        __syncthreads();
        // ---- S = decay^n S + K^T V' (it reads the old state, whose two halves Q S0 below reads from their own copies;
        //      the warps take its tiles from the last warp down, the query products from the first warp up)
        const float shrink = pw[n];
        for (int tile = LC_THREADS / 32 - 1 - warp; tile < d_tiles * (LC_VS / 16); tile += LC_THREADS / 32) {
            const int ti = tile / (LC_VS / 16), tj = tile % (LC_VS / 16);
            wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
            wmma::load_matrix_sync(acc, Sf + ti * 16 * L.lds_f + tj * 16, L.lds_f, wmma::mem_row_major);
#pragma unroll
            for (int e = 0; e < acc.num_elements; ++e) acc.x[e] *= shrink;
            for (int kk = 0; kk < LC_C / 16; ++kk) {
                wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::col_major> a;     // K^T: element (d, j) = K[j][d]
                wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> b;
                wmma::load_matrix_sync(a, Ks + kk * 16 * L.ldq + ti * 16, L.ldq);
                wmma::load_matrix_sync(b, Vh + kk * 16 * L.ldv + tj * 16, L.ldv);
                wmma::mma_sync(acc, a, b, acc);
                wmma::load_matrix_sync(b, Vl + kk * 16 * L.ldv + tj * 16, L.ldv);
                wmma::mma_sync(acc, a, b, acc);
            }
            wmma::store_matrix_sync(Sf + ti * 16 * L.lds_f + tj * 16, acc, L.lds_f, wmma::mem_row_major);
        }
        if (phase != 1) {
        // ---- A = Q K^T (the tiles on and below the diagonal) and Q S0
        for (int tile = warp; tile < (LC_C / 16) * (LC_C / 16); tile += LC_THREADS / 32) {
            const int ti = tile / (LC_C / 16), tj = tile % (LC_C / 16);
            wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
            wmma::fill_fragment(acc, 0.f);
            if (tj <= ti) {
                for (int kk = 0; kk < d_tiles; ++kk) {
                    wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> a;
                    wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::col_major> b;
                    wmma::load_matrix_sync(a, Qs + ti * 16 * L.ldq + kk * 16, L.ldq);
                    wmma::load_matrix_sync(b, Ks + tj * 16 * L.ldq + kk * 16, L.ldq);
                    wmma::mma_sync(acc, a, b, acc);
                }
            }
            wmma::store_matrix_sync(Af + ti * 16 * L.lda_f + tj * 16, acc, L.lda_f, wmma::mem_row_major);
        }
        for (int tile = warp; tile < (LC_C / 16) * (LC_VS / 16); tile += LC_THREADS / 32) {
            const int ti = tile / (LC_VS / 16), tj = tile % (LC_VS / 16);
            wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
            wmma::fill_fragment(acc, 0.f);
            for (int kk = 0; kk < d_tiles; ++kk) {
                wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> a;
                wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> b;
                wmma::load_matrix_sync(a, Qs + ti * 16 * L.ldq + kk * 16, L.ldq);
                wmma::load_matrix_sync(b, Sh + kk * 16 * L.lds_h + tj * 16, L.lds_h);
                wmma::mma_sync(acc, a, b, acc);
                wmma::load_matrix_sync(b, Sl + kk * 16 * L.lds_h + tj * 16, L.lds_h);
                wmma::mma_sync(acc, a, b, acc);
            }
            wmma::store_matrix_sync(Of + ti * 16 * L.ldo + tj * 16, acc, L.ldo, wmma::mem_row_major);
        }
        __syncthreads();
        // ---- decays, in float32: A'[i, j] = A[i, j] * decay^(i - j) for j <= i, in two halves; (Q S0)[i, :] *= decay^(i + 1)
        for (int i = warp; i < LC_C; i += LC_THREADS / 32) {
#pragma unroll
            for (int j = lane; j < LC_C; j += 32)
                lc_split(j <= i ? Af[i * L.lda_f + j] * pw[i - j] : 0.f, Ah[i * L.lda_h + j], Al[i * L.lda_h + j]);
            Of[i * L.ldo + lane] *= pw[i + 1];
        }
        __syncthreads();
        }
        // ---- O += A' V
        for (int tile = warp; phase != 1 && tile < (LC_C / 16) * (LC_VS / 16); tile += LC_THREADS / 32) {
            const int ti = tile / (LC_VS / 16), tj = tile % (LC_VS / 16);
            wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc;
            wmma::load_matrix_sync(acc, Of + ti * 16 * L.ldo + tj * 16, L.ldo, wmma::mem_row_major);
            for (int kk = 0; kk <= ti; ++kk) {                   // A' is zero above the diagonal
                wmma::fragment<wmma::matrix_a, 16, 16, 16, __nv_bfloat16, wmma::row_major> a;
                wmma::fragment<wmma::matrix_b, 16, 16, 16, __nv_bfloat16, wmma::row_major> b;
                wmma::load_matrix_sync(b, Vs + kk * 16 * L.ldv + tj * 16, L.ldv);
                wmma::load_matrix_sync(a, Ah + ti * 16 * L.lda_h + kk * 16, L.lda_h);
                wmma::mma_sync(acc, a, b, acc);
                wmma::load_matrix_sync(a, Al + ti * 16 * L.lda_h + kk * 16, L.lda_h);
                wmma::mma_sync(acc, a, b, acc);
            }
            wmma::store_matrix_sync(Of + ti * 16 * L.ldo + tj * 16, acc, L.ldo, wmma::mem_row_major);
        }
        __syncthreads();
        for (int i = warp; phase != 1 && i < n; i += LC_THREADS / 32)
            if (c0 + lane < vdim) out[((size_t)(chunk0 + i) * heads + head) * vdim + c0 + lane] = Of[i * L.ldo + lane];
    }
    if (phase == 1) {                            // the part's end state from a start of zero
        for (int d = warp; d < dim; d += LC_THREADS / 32)
            if (c0 + lane < vdim) parts_S[(size_t)part * dim * vdim + (size_t)d * vdim + c0 + lane] = Sf[d * L.lds_f + lane];
        return;
    }
    if (write_state && t_end == seg_end) {
        for (int d = warp; d < dim; d += LC_THREADS / 32)
            if (c0 + lane < vdim) S[(size_t)d * vdim + c0 + lane] = Sf[d * L.lds_f + lane];
    }
}

// Between the two phases: scratch[seg, head, p] holds part p's end state from a start of zero and becomes part p's start
// state: start[0] = the state the request came with, start[p + 1] = decay^part_len * start[p] + end[p]. One thread per
// element of a head's state walks the parts in order.
__global__ void lightning_prefix_kernel(float* __restrict__ scratch, const float* __restrict__ state, const int* __restrict__ seg_slot,
                                        const int* __restrict__ cu_seqlens, const float* __restrict__ decay, int heads,
                                        int elements, int parts, int part_len) {
    pdl_wait();
    pdl_launch_dependents();
    const int e = blockIdx.x * blockDim.x + threadIdx.x, head = blockIdx.y, seg = blockIdx.z;
    if (e >= elements) return;
    const int len = cu_seqlens[seg + 1] - cu_seqlens[seg];
    const int used = (len + part_len - 1) / part_len;           // parts that hold tokens
    float* mine = scratch + ((size_t)seg * heads + head) * (parts + 1) * elements + e;
    const float shrink = powf(decay[head], (float)part_len);
    float start = state[((size_t)seg_slot[seg] * heads + head) * elements + e];
    for (int p = 0; p < used; ++p) {
        const float end = mine[(size_t)p * elements];
        mine[(size_t)p * elements] = start;
        start = fmaf(shrink, start, end);
    }
}

// The chunked form: bfloat16 projections, dim a multiple of 16 up to 256, vdim a multiple of 8, rows of 16-byte alignment. Same arguments as ttb_lightning_scan.
TTB_EXPORT int ttb_lightning_chunks_supports(int dim, int vdim) {
    return dim >= 16 && dim <= 256 && (dim & 15) == 0 && vdim >= 8 && (vdim & 7) == 0 && lc_layout(dim).total <= 200 * 1024;
}

// parts > 1: scratch holds segments * heads * (parts + 1) * dim * vdim floats, part_len is a multiple of the chunk (64).
TTB_EXPORT int ttb_lightning_chunks(const void* proj, int ld, const int* cu_seqlens, const int* seg_slot, float* state,
                                    const float* decay, float* out, int segments, int heads, int dim, int vdim, int write_state,
                                    float* scratch, int parts, int part_len, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!proj || !cu_seqlens || !seg_slot || !state || !decay || !out) return TTB_ERR_ARGUMENT;
    if (!ttb_lightning_chunks_supports(dim, vdim) || heads < 1 || heads > 65535 || segments > 65535) return TTB_ERR_UNSUPPORTED;
    if ((ld & 7) || !aligned16(proj)) return TTB_ERR_UNSUPPORTED;          // sixteen-byte loads of eight values
    const LcLayout L = lc_layout(dim);
    static TtbOncePerDevice once;
    if (once.pending()) {
        cudaError_t e = cudaFuncSetAttribute(lightning_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return (int)e;
        once.mark();
    }
    if (L.total > 200 * 1024) return TTB_ERR_UNSUPPORTED;
    if (parts < 1 || (parts > 1 && (!scratch || part_len < LC_C || part_len % LC_C))) return TTB_ERR_ARGUMENT;
    dim3 grid(((vdim + LC_VS - 1) / LC_VS) * parts, heads, segments);
    for (int phase = parts > 1 ? 1 : 0; phase <= (parts > 1 ? 2 : 0); ++phase) {
        ttb_launch(lightning_chunk_kernel, grid, LC_THREADS, L.total, stream, (const __nv_bfloat16*)proj, ld, cu_seqlens, seg_slot,
                   state, decay, out, heads, dim, vdim, write_state, scratch, part_len, parts, phase);
        if (phase == 1)
            ttb_launch(lightning_prefix_kernel, dim3((dim * vdim + 255) / 256, heads, segments), 256, 0, stream, scratch,
                       (const float*)state, seg_slot, cu_seqlens, decay, heads, dim * vdim, parts, part_len);
    }
    return ttb_launch_status();
}
