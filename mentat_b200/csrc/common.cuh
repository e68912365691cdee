// Shared device helpers of libmentat_b200 (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/mentat_b200.h"

#include <atomic>

namespace mentat {
// kernels this library has launched (host counter, all devices and streams)
inline std::atomic<long long> g_kernel_launches{0};
}  // namespace mentat

// follows every kernel launch: counts it and turns a launch error into a status
#define MENTAT_CHECK_LAUNCH()                                                 \
    do {                                                                      \
        mentat::g_kernel_launches.fetch_add(1, std::memory_order_relaxed);    \
        if (cudaPeekAtLastError() != cudaSuccess) {                           \
            (void)cudaGetLastError();                                         \
            return MENTAT_ERR_CUDA;                                           \
        }                                                                     \
    } while (0)

namespace mentat {

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while its predecessor on the stream still runs;
// griddep_wait() returns once that predecessor has completed and its writes
// are visible (at once for an ordinary launch), and griddep_launch() lets the
// next such kernel on the stream be scheduled.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether kernels go out with programmatic stream serialization (MENTAT_PDL=0
// launches them one after another instead), and a launch with or without it.
static inline bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MENTAT_PDL");
        v = (e && *e) ? (atoi(e) != 0) : 1;
    }
    return v != 0;
}
template <typename... KArgs, typename... Args>
static cudaError_t launch(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// device timeline of one call (trace builds only): nanosecond stamps, first and
// last over the CTAs of a kernel
#ifdef MENTAT_TC_TRACE
static __device__ unsigned long long g_timeline[32];
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
static __device__ unsigned long long g_cta_end[2][256];  // per CTA of the wide (0) and narrow (1) kernel
#define TL_CTA_END(w) do { if (threadIdx.x == 0 && blockIdx.x < 256) mentat::g_cta_end[(w)][blockIdx.x] = mentat::gtime(); } while (0)
#define TL_FIRST(k) do { if (threadIdx.x == 0) atomicMin(&mentat::g_timeline[(k)], mentat::gtime()); } while (0)
#define TL_LAST(k) do { if (threadIdx.x == 0) atomicMax(&mentat::g_timeline[(k)], mentat::gtime()); } while (0)
#else
#define TL_FIRST(k) do { } while (0)
#define TL_LAST(k) do { } while (0)
#define TL_CTA_END(w) do { } while (0)
#endif

// ---------------------------------------------------------------------------
// sm_100 packed f32x2 arithmetic (one instruction for two IEEE round-to-nearest
// operations, the same bits as two scalar ones) and the three-input max
// ---------------------------------------------------------------------------
#define MENTAT_F32X2_BINARY(name, op)                                                                      \
    __device__ __forceinline__ float2 name(float2 a, float2 b) {                                          \
        float2 d;                                                                                         \
        asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t" op \
            " rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"                                                \
            : "=f"(d.x), "=f"(d.y)                                                                        \
            : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));                                                    \
        return d;                                                                                         \
    }
MENTAT_F32X2_BINARY(fadd2, "add.rn.f32x2")
MENTAT_F32X2_BINARY(fsub2, "sub.rn.f32x2")
MENTAT_F32X2_BINARY(fmul2, "mul.rn.f32x2")
#undef MENTAT_F32X2_BINARY
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    static constexpr int code = MENTAT_F32;
    __device__ __forceinline__ static float to_f(float x) { return x; }
    __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int code = MENTAT_BF16;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
    static constexpr int code = MENTAT_F16;
    __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
    __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

__host__ __device__ inline int dtype_bytes(int dtype) { return dtype == MENTAT_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// cache indexing
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t seq_index(const mentat_kv_cache& c, int layer, int slot) {
    return (int64_t)layer * c.max_seqs + slot;
}
__device__ __forceinline__ int32_t* table_row(const mentat_kv_cache& c, int layer, int slot) {
    return c.tables + ((int64_t)layer * c.max_seqs + slot) * c.max_blocks_per_seq;
}
// element offset of the (layer, block, slot-in-block) row; a row is Hkv*D elements
__device__ __forceinline__ int64_t pool_row(const mentat_kv_cache& c, int layer, int block, int s) {
    return (((int64_t)layer * c.num_blocks + block) * c.block_size + s) * (int64_t)c.num_kv_heads *
           c.head_dim;
}

// first device error wins; later ones are dropped
__device__ __forceinline__ void set_error(const mentat_kv_cache& c, int code, int64_t arg) {
    unsigned long long* e = reinterpret_cast<unsigned long long*>(c.ctrl + MENTAT_CTRL_ERROR);
    if (atomicCAS(e, 0ull, (unsigned long long)code) == 0ull) c.ctrl[MENTAT_CTRL_ERRARG] = arg;
}
__device__ __forceinline__ bool has_error(const mentat_kv_cache& c) {
    return *((volatile int64_t*)(c.ctrl + MENTAT_CTRL_ERROR)) != 0;
}

// ---------------------------------------------------------------------------
// block-wide exclusive scan of ints (blockDim.x a multiple of 32, <= 1024)
// ---------------------------------------------------------------------------
// 64-bit variant (several small counters packed in one word)
__device__ __forceinline__ long long block_exclusive_scan64(long long v, long long* total, long long* smem32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    long long x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem32[warp] = x;
    __syncthreads();
    if (warp == 0) {
        long long w = lane < nwarps ? smem32[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            long long y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        smem32[lane] = w;
    }
    __syncthreads();
    long long base = warp ? smem32[warp - 1] : 0;
    *total = smem32[nwarps - 1];
    __syncthreads();
    return base + x - v;
}

__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* smem32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem32[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? smem32[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        smem32[lane] = w;
    }
    __syncthreads();
    int base = warp ? smem32[warp - 1] : 0;
    *total = smem32[nwarps - 1];
    __syncthreads();
    return base + x - v;
}

// copy `n` bytes with a whole block; 16-byte vectors when everything is aligned
__device__ __forceinline__ void block_copy_bytes(void* dst, const void* src, int64_t n) {
    if ((((uintptr_t)dst | (uintptr_t)src | (uintptr_t)n) & 15) == 0) {
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        for (int64_t i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = s[i];
        return;
    }
    const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
    uint8_t* d = reinterpret_cast<uint8_t*>(dst);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

}  // namespace mentat
