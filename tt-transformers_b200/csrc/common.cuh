// Shared device helpers: element types, vector loads, reductions, error codes.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#define TTB_OK 0
#define TTB_ERR_UNSUPPORTED (-2)   // a size or option this kernel does not take
#define TTB_ERR_ARGUMENT (-3)      // a null pointer or a contradiction between arguments

#define TTB_DTYPE_F32 0
#define TTB_DTYPE_BF16 1

#define TTB_EXPORT extern "C" __attribute__((visibility("default")))

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels of one step run back to back on one stream. Launched with the attribute below, a kernel
// may become resident while its predecessor is still running: everything before pdl_wait() (index
// arithmetic, prefetching weights, which no kernel of the step writes) overlaps the predecessor's
// tail; pdl_wait() returns once the predecessor has completed and its writes are visible. Every
// kernel launched this way calls pdl_launch_dependents() first and pdl_wait() before it reads or
// writes anything another kernel of the step touches. TTB200_PDL=0 in the environment turns the
// attribute off (the two device calls are then no-ops).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

static inline int ttb_pdl_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char* e = getenv("TTB200_PDL");
        enabled = (e && e[0] == '0') ? 0 : 1;
    }
    return enabled;
}

template <typename... KArgs, typename... Args>
static inline void ttb_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ttb_pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);   // errors surface in ttb_launch_status()
}

static inline int ttb_launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TTB_OK : (int)e;
}

// A kernel's attributes (its shared-memory limit, its cluster size) belong to a device: a launcher sets them
// before its first launch on each device it is used on.
#define TTB_MAX_DEVICES 64
struct TtbOncePerDevice {
    bool done[TTB_MAX_DEVICES] = {};
    bool pending() const {
        int d = 0;
        return cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= TTB_MAX_DEVICES || !done[d];
    }
    void mark() {
        int d = 0;
        if (cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < TTB_MAX_DEVICES) done[d] = true;
    }
};

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum / max over all threads; `scratch` holds 32 floats. Every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = (lane < nwarps) ? scratch[lane] : 0.f;
    r = warp_sum(r);
    return r;
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = (lane < nwarps) ? scratch[lane] : -INFINITY;
    r = warp_max(r);
    return r;
}

// Eight consecutive elements as floats. The 16-byte (bf16) or 2x16-byte (f32) path needs
// an address aligned to that size; callers check alignment before choosing it.
__device__ __forceinline__ void load8(const float* p, float (&out)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&out)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = raw;
}

// Ask L2 for the 128-byte line that holds p (weights that no kernel writes may be asked for before pdl_wait()).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }
