// Fused logits -> entropy -> gate -> decision kernel, one cluster of CTAs per leaf.
//
// Replaces, per leaf, compute_entropy (core/generator_utils.py:196-202),
// apply_repetition_penalty (:205-230), the log_softmax / argmax / topk of
// MentatGenerator._do_extend / _do_branch (core/generator.py:283-310) and the
// EMA / threshold / decision arithmetic of _step_leaf (:342-369) with
// adaptive_threshold (generator_utils.py:247-253) and _soft_explore_factor
// (generator.py:319-331).
//
// The reduced-precision rounding chain of the reference's CPU path is
// reproduced element by element (R = round to the logits dtype):
//   xt = R(x / T);  m = max xt;  S = sum exp(xt - m)         (float)
//   p  = R(exp(xt - m) / S);     L = R(log(R(S)))
//   lp = R((xt - m) - L);        H = -R(sum R(p * lp))       (NaN terms -> 0)
// The penalised logits z (R(x / pen) for x > 0, R(x * pen) otherwise, over
// the leaf's generated tokens) go through the same log_softmax; extend takes
// the lowest index among the maximal log-probs, branch the top K ordered by
// value then index.  The decision is evaluated in double precision with the
// reference's operation order and no fused multiply-adds.

#include <cooperative_groups.h>

#include "common.cuh"

namespace mentat {

constexpr int GATE_THREADS = 512;
constexpr int GATE_WARPS = GATE_THREADS / 32;

template <typename T> __device__ __forceinline__ float rnd(float x) { return Elem<T>::to_f(Elem<T>::from_f(x)); }
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }
// bf16 round-to-nearest-even on the bit pattern (integer pipe; finite values and
// infinities; the callers never pass NaN)
template <> __device__ __forceinline__ float rnd<__nv_bfloat16>(float x) {
    uint32_t u = __float_as_uint(x);
    u += 0x7fffu + ((u >> 16) & 1u);
    return __uint_as_float(u & 0xffff0000u);
}

// Correctly rounded a / b from rb = RN(1 / b) (Markstein's division, as in
// P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 1990): q = RN(a rb) is within an ulp
// of a / b, r = a - q b is exact with a fused multiply-add, and RN(q + r rb) is
// the correctly rounded quotient, the same bits as IEEE division.  Quotients
// near the underflow threshold (and a = 0) take the IEEE division itself.
__device__ __forceinline__ float div_rn(float a, float b, float rb) {
    const float q = __fmul_rn(a, rb);
    if (!(fabsf(q) >= 0x1p-124f)) return __fdiv_rn(a, b);
    const float r = __fmaf_rn(-q, b, a);
    return __fmaf_rn(r, rb, q);
}

// Kahan's compensated sum in single precision (no reassociation: every step
// is an explicit round-to-nearest operation); value() is the pair as a double
struct KSum {
    float s = 0.f, c = 0.f;
    __device__ __forceinline__ void add(float x) {
        const float y = __fsub_rn(x, c);
        const float t = __fadd_rn(s, y);
        c = __fsub_rn(__fsub_rn(t, s), y);
        s = t;
    }
    __device__ __forceinline__ double value() const { return (double)s - (double)c; }
};

// 64-bit key ordering by value, then by lower index
__device__ __forceinline__ uint64_t topkey(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)u << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ float key_val(uint64_t k) {
    uint32_t u = (uint32_t)(k >> 32);
    u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    return __uint_as_float(u);
}
__device__ __forceinline__ int key_idx(uint64_t k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// Each leaf runs on a cluster of GATE_CLUSTER CTAs, each over a contiguous
// slice of the vocabulary, in three passes over the slice (16-byte loads when
// the row is aligned; the row stays in L2 after the first pass):
//   A  maxima of xt and z;
//   B  S = sum exp(xt - m), the penalised S, and the float-accurate entropy's sums;
//   C  the rounded entropies and the top-K of the penalised log-probs.
// After each pass the slices' values are exchanged through distributed shared
// memory and combined in rank order, so every CTA derives the same statistics;
// rank 0 combines the pass-C values and writes the leaf's record.
constexpr int GATE_CLUSTER = 8;
constexpr int GATE_VEC = 8;  // slice starts are multiples of 8 elements (16-byte aligned)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_maxf(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// K rounds of max extraction over the lanes' descending lists (entries past a
// lane's list read as 0, the smallest key); lane 0 receives the merged list.
template <typename Get>
__device__ __forceinline__ void warp_topk_merge(int K, Get get, uint64_t* dst) {
    const int lane = threadIdx.x & 31;
    int head = 0;
    for (int k = 0; k < K; ++k) {
        const uint64_t mine = get(head);
        const uint64_t w = warp_max_u64(mine);
        if (w == mine && w != 0ull) ++head;
        if (lane == 0) dst[k] = w;
    }
}

// element u (a compile-time index after unrolling) of a 16-byte vector of T, as float
template <typename T> __device__ __forceinline__ float vget(const uint4& r, int u);
template <> __device__ __forceinline__ float vget<float>(const uint4& r, int u) { return __uint_as_float((&r.x)[u]); }
template <> __device__ __forceinline__ float vget<__nv_bfloat16>(const uint4& r, int u) {
    const uint32_t w = (&r.x)[u >> 1];
    return __uint_as_float((u & 1) ? (w & 0xffff0000u) : (w << 16));
}
template <> __device__ __forceinline__ float vget<__half>(const uint4& r, int u) {
    const uint32_t w = (&r.x)[u >> 1];
    return __half2float(__ushort_as_half((unsigned short)((u & 1) ? (w >> 16) : (w & 0xffffu))));
}
// element u of a 16-byte vector of T set to v (v is representable in T)
template <typename T> __device__ __forceinline__ void vset(uint4& r, int u, float v);
template <> __device__ __forceinline__ void vset<float>(uint4& r, int u, float v) { (&r.x)[u] = __float_as_uint(v); }
template <> __device__ __forceinline__ void vset<__nv_bfloat16>(uint4& r, int u, float v) {
    const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    uint32_t& w = (&r.x)[u >> 1];
    w = (u & 1) ? ((w & 0xffffu) | (b << 16)) : ((w & 0xffff0000u) | b);
}
template <> __device__ __forceinline__ void vset<__half>(uint4& r, int u, float v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(v));
    uint32_t& w = (&r.x)[u >> 1];
    w = (u & 1) ? ((w & 0xffffu) | (b << 16)) : ((w & 0xffff0000u) | b);
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// online (max, sum exp, sum exp * shift) of the float-accurate entropy: the
// state (m, S, A) stands for S = sum e^(y - m), A = sum e^(y - m) (y - m)
struct AccEnt {
    float m = -INFINITY, S = 0.f, A = 0.f;
    __device__ __forceinline__ void add(float y) {
        if (y > m) {
            if (m != -INFINITY) {
                const float f = expf(m - y);
                A = (A + S * (m - y)) * f;
                S *= f;
            }
            m = y;
        }
        const float d = y - m;
        const float e = expf(d);
        S += e;
        A += e * d;
    }
    __device__ __forceinline__ void merge(float m2, float S2, float A2) {
        if (m2 == -INFINITY) return;
        if (m == -INFINITY) { m = m2; S = S2; A = A2; return; }
        const float mn = fmaxf(m, m2);
        const float f1 = expf(m - mn), f2 = expf(m2 - mn);
        A = (A + S * (m - mn)) * f1 + (A2 + S2 * (m2 - mn)) * f2;
        S = S * f1 + S2 * f2;
        m = mn;
    }
    __device__ __forceinline__ void warp_merge() {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            const float S2 = __shfl_xor_sync(0xffffffffu, S, o);
            const float A2 = __shfl_xor_sync(0xffffffffu, A, o);
            merge(m2, S2, A2);
        }
    }
};

// e^d for d <= 0 with IEEE single-precision multiplies and adds only (no fused
// multiply-add, no hardware approximation), so that the numpy restatement in
// the oracle produces the same bits.  Cody and Waite's argument reduction
// (W. J. Cody, W. Waite, "Software Manual for the Elementary Functions", 1980):
// d = k ln2 + r with k = rint(d / ln2), ln2 split into a 15-bit head (k ln2_hi
// is exact) and a tail; then the degree-7 Taylor polynomial of e^r on
// |r| <= ln2/2 by Horner's rule, and the exact scaling by 2^k (k rounded to the
// nearest integer, ties to even, by the 1.5 * 2^23 addition).  Inputs below
// -87 (results near the single-precision underflow) give 0.
__device__ __forceinline__ float exp_cw(float d) {
    if (!(d >= -87.0f)) return 0.0f;
    // k = rint(d log2(e)): adding 1.5 * 2^23 rounds to an integer (ties to even)
    // and leaves it in the low bits of the sum
    const float kb = __fadd_rn(__fmul_rn(d, 0x1.715476p+0f), 12582912.0f);
    const float k = __fsub_rn(kb, 12582912.0f);
    const int ki = __float_as_int(kb) - 0x4b400000;
    const float r = __fsub_rn(__fsub_rn(d, __fmul_rn(k, 0x1.62e4p-1f)),  // ln2 head
                              __fmul_rn(k, 0x1.7f7d1cp-20f));            // ln2 tail
    float p = 0x1.a01a02p-13f;                                           // 1/7!
    p = __fadd_rn(__fmul_rn(p, r), 0x1.6c16c2p-10f);                     // 1/6!
    p = __fadd_rn(__fmul_rn(p, r), 0x1.111112p-7f);                      // 1/5!
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-5f);                      // 1/4!
    p = __fadd_rn(__fmul_rn(p, r), 0x1.555556p-3f);                      // 1/3!
    p = __fadd_rn(__fmul_rn(p, r), 0.5f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    return __fmul_rn(p, __int_as_float((ki + 127) << 23));                // k >= -126
}

// exp_cw of two values with packed f32x2 operations: each lane takes exactly the
// scalar function's operations (IEEE round-to-nearest, no fused multiply-add), so
// each result has the scalar one's bits
__device__ __forceinline__ float2 exp_cw2(float2 d) {
    const float2 kb = fadd2(fmul2(d, f2(0x1.715476p+0f)), f2(12582912.0f));
    const float2 k = fsub2(kb, f2(12582912.0f));
    const int kx = __float_as_int(kb.x) - 0x4b400000, ky = __float_as_int(kb.y) - 0x4b400000;
    const float2 r = fsub2(fsub2(d, fmul2(k, f2(0x1.62e4p-1f))), fmul2(k, f2(0x1.7f7d1cp-20f)));
    float2 p = f2(0x1.a01a02p-13f);
    p = fadd2(fmul2(p, r), f2(0x1.6c16c2p-10f));
    p = fadd2(fmul2(p, r), f2(0x1.111112p-7f));
    p = fadd2(fmul2(p, r), f2(0x1.555556p-5f));
    p = fadd2(fmul2(p, r), f2(0x1.555556p-3f));
    p = fadd2(fmul2(p, r), f2(0.5f));
    p = fadd2(fmul2(p, r), f2(1.0f));
    p = fadd2(fmul2(p, r), f2(1.0f));
    // lanes below -87 (whose k may be out of range) are replaced by 0 below
    const float2 e = fmul2(p, make_float2(__uint_as_float((uint32_t)(kx + 127) << 23),
                                          __uint_as_float((uint32_t)(ky + 127) << 23)));
    return make_float2(d.x >= -87.0f ? e.x : 0.0f, d.y >= -87.0f ? e.y : 0.0f);
}

// KSum over two chains at once (packed f32x2); value() adds both chains in double
struct KSum2 {
    float2 s = make_float2(0.f, 0.f), c = make_float2(0.f, 0.f);
    __device__ __forceinline__ void add(float2 x) {
        const float2 y = fsub2(x, c);
        const float2 t = fadd2(s, y);
        c = fsub2(fsub2(t, s), y);
        s = t;
    }
    __device__ __forceinline__ double value() const {
        return ((double)s.x - (double)c.x) + ((double)s.y - (double)c.y);
    }
};

// div_rn of two numerators by one divisor (packed f32x2); a lane whose quotient is
// near the underflow threshold takes the IEEE division, as div_rn does
__device__ __forceinline__ float2 div_rn2(float2 a, float b, float rb) {
    const float2 q = fmul2(a, f2(rb));
    const float2 r = ffma2(make_float2(-q.x, -q.y), f2(b), a);
    float2 d = ffma2(r, f2(rb), q);
    if (!(fabsf(q.x) >= 0x1p-124f)) d.x = __fdiv_rn(a.x, b);
    if (!(fabsf(q.y) >= 0x1p-124f)) d.y = __fdiv_rn(a.y, b);
    return d;
}

// Inserts `cur` into the descending list best[0..K); returns the new best[K - 1].
// Out of line, so that the list lives in local memory and the hot loop keeps
// only the threshold in registers.
__device__ __noinline__ uint64_t topk_insert(uint64_t* best, int K, uint64_t cur) {
    for (int k = 0; k < K; ++k) {
        if (cur > best[k]) {
            const uint64_t t = best[k];
            best[k] = cur;
            cur = t;
        }
    }
    return best[K - 1];
}

// Dynamic shared memory of a gate CTA: the slice's repetition-penalty bitmap,
// then (when `cache` is set) the slice's xt and z values in the logits dtype,
// which passes B and C read instead of the logits.
template <typename T>
__host__ __device__ inline int gate_slice(int V) {
    return ((V + GATE_CLUSTER - 1) / GATE_CLUSTER + GATE_VEC - 1) / GATE_VEC * GATE_VEC;
}
__host__ __device__ inline int gate_bitmap_bytes(int per) { return ((per + 31) / 32 * 4 + 15) / 16 * 16; }

template <typename T>
__global__ void __launch_bounds__(GATE_THREADS, sizeof(T) == 4 ? 1 : 2)  // fp32 needs > 64 registers
k_gate(const T* __restrict__ logits, int V, int64_t ld, const int32_t* __restrict__ hist_ptr,
       const int32_t* __restrict__ hist_ids, const double* __restrict__ ema_old, mentat_gate_params P,
       mentat_gate_out* __restrict__ out, int cache) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) uint8_t gate_smem[];
    __shared__ float s_red[2][GATE_WARPS], s_acc[3][GATE_WARPS];
    __shared__ double s_redd[2][GATE_WARPS];
    __shared__ uint64_t s_keys[GATE_WARPS][MENTAT_GATE_MAXK];
    __shared__ float s_xa[5];                        // this CTA's values of pass A
    __shared__ double s_xb[2], s_xc[2];              // ... of passes B and C
    __shared__ uint64_t s_xk[MENTAT_GATE_MAXK];      // this CTA's top-K
    __shared__ float s_glob[5];
    __shared__ double s_globd[2];
    const int C = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int leaf = blockIdx.x / C, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = gate_slice<T>(V);
    const int v0 = min(V, rank * per), v1 = min(V, v0 + per);
    const int nwords = (per + 31) >> 5;
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(gate_smem);
    T* xt_s = reinterpret_cast<T*>(gate_smem + gate_bitmap_bytes(per));  // [per]
    T* z_s = xt_s + per;                                                // [per]
    const T* x = logits + (int64_t)leaf * ld;
    const float Tf = (float)P.temperature, pf = (float)P.penalty;
    const float rT = __frcp_rn(Tf), rP = __frcp_rn(pf);  // correctly rounded reciprocals for div_rn
    const bool want_pen = (P.flags & MENTAT_GATE_SKIP_PEN_ENTROPY) == 0;
    const bool use_t = P.temperature != 1.0;
    const int K = P.K;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(v0 * sizeof(T))) & 15) == 0;
    constexpr int VW = 16 / sizeof(T);  // elements per 16-byte load

    for (int w = tid; w < nwords; w += GATE_THREADS) bitmap[w] = 0u;
    __syncthreads();
    for (int h = hist_ptr[leaf] + tid; h < hist_ptr[leaf + 1]; h += GATE_THREADS) {
        const int id = hist_ids[h];
        if (id >= v0 && id < v1) atomicOr(&bitmap[(id - v0) >> 5], 1u << ((id - v0) & 31));
    }
    __syncthreads();
    // f(i, xt_i, z_i, y_i) for every element of the slice, from the logits:
    // y = x / T, xt = R(y), z = the penalised logit
    auto from_logits = [&](auto&& f) {
        auto elem = [&](int i, float xv, uint32_t hit) {
            const float y = use_t ? div_rn(xv, Tf, rT) : xv;
            const float xt = use_t ? rnd<T>(y) : xv;
            float z = xv;
            if (hit) z = xv > 0.f ? rnd<T>(div_rn(xv, pf, rP)) : rnd<T>(__fmul_rn(xv, pf));
            f(i, xt, z, y);
        };
        int tail = v0;
        if (vec) {
            for (int j = v0 + tid * VW; j + VW <= v1; j += GATE_THREADS * VW) {
                const uint4 e = *reinterpret_cast<const uint4*>(x + j);
                const uint32_t bits = bitmap[(j - v0) >> 5] >> ((j - v0) & 31);
#pragma unroll
                for (int u = 0; u < VW; ++u) elem(j + u, vget<T>(e, u), (bits >> u) & 1u);
            }
            tail = v0 + (v1 - v0) / VW * VW;
        }
        for (int i = tail + tid; i < v1; i += GATE_THREADS)
            elem(i, Elem<T>::to_f(x[i]), (bitmap[(i - v0) >> 5] >> ((i - v0) & 31)) & 1u);
    };
    // g(i, xt_i, z_i) for every element of the slice: from the shared-memory
    // copy when the slice is cached, else recomputed from the logits
    auto for_slice = [&](auto&& g) {
        if (cache) {
            const int n = v1 - v0;
            for (int j = tid * VW; j + VW <= n; j += GATE_THREADS * VW) {
                const uint4 a = *reinterpret_cast<const uint4*>(xt_s + j);
                const uint4 b = *reinterpret_cast<const uint4*>(z_s + j);
#pragma unroll
                for (int u = 0; u < VW; ++u) g(v0 + j + u, vget<T>(a, u), vget<T>(b, u));
            }
            for (int i = n / VW * VW + tid; i < n; i += GATE_THREADS)
                g(v0 + i, Elem<T>::to_f(xt_s[i]), Elem<T>::to_f(z_s[i]));
        } else {
            from_logits([&](int i, float xt, float z, float) { g(i, xt, z); });
        }
    };

    // g2(i, (xt_i, xt_i+1), (z_i, z_i+1)) for pairs of the cached slice, g1 for single
    // elements (the slice's tail, or every element when the slice is not cached)
    auto for_slice2 = [&](auto&& g2, auto&& g1) {
        if (cache) {
            const int n = v1 - v0;
            for (int j = tid * VW; j + VW <= n; j += GATE_THREADS * VW) {
                const uint4 a = *reinterpret_cast<const uint4*>(xt_s + j);
                const uint4 b = *reinterpret_cast<const uint4*>(z_s + j);
#pragma unroll
                for (int u = 0; u < VW; u += 2)
                    g2(v0 + j + u, make_float2(vget<T>(a, u), vget<T>(a, u + 1)),
                       make_float2(vget<T>(b, u), vget<T>(b, u + 1)));
            }
            for (int i = n / VW * VW + tid; i < n; i += GATE_THREADS)
                g1(v0 + i, Elem<T>::to_f(xt_s[i]), Elem<T>::to_f(z_s[i]));
        } else {
            from_logits([&](int i, float xt, float z, float) { g1(i, xt, z); });
        }
    };

    // pass A: maxima of xt and z, the float-accurate entropy's online sums, and
    // the slice copy (16-byte stores when the logits were read 16 bytes at a time)
    float mt = -INFINITY, mz = -INFINITY;
    AccEnt acc;
    auto take = [&](float xt, float z, float y) {
        mt = fmaxf(mt, xt);
        mz = fmaxf(mz, z);
        acc.add(y);
    };
    if (vec && cache) {
        for (int j = v0 + tid * VW; j + VW <= v1; j += GATE_THREADS * VW) {
            const uint4 e = *reinterpret_cast<const uint4*>(x + j);
            uint4 a = e, b = e;
            const uint32_t bits = bitmap[(j - v0) >> 5] >> ((j - v0) & 31);
#pragma unroll
            for (int u = 0; u < VW; ++u) {
                const float xv = vget<T>(e, u);
                const float y = use_t ? div_rn(xv, Tf, rT) : xv;
                const float xt = use_t ? rnd<T>(y) : xv;
                float z = xv;
                if ((bits >> u) & 1u) z = xv > 0.f ? rnd<T>(div_rn(xv, pf, rP)) : rnd<T>(__fmul_rn(xv, pf));
                take(xt, z, y);
                if (use_t) vset<T>(a, u, xt);
                if ((bits >> u) & 1u) vset<T>(b, u, z);
            }
            *reinterpret_cast<uint4*>(xt_s + (j - v0)) = a;
            *reinterpret_cast<uint4*>(z_s + (j - v0)) = b;
        }
        const int tail = v0 + (v1 - v0) / VW * VW;
        for (int i = tail + tid; i < v1; i += GATE_THREADS) {
            const float xv = Elem<T>::to_f(x[i]);
            const float y = use_t ? div_rn(xv, Tf, rT) : xv;
            const float xt = use_t ? rnd<T>(y) : xv;
            float z = xv;
            if ((bitmap[(i - v0) >> 5] >> ((i - v0) & 31)) & 1u) z = xv > 0.f ? rnd<T>(div_rn(xv, pf, rP)) : rnd<T>(__fmul_rn(xv, pf));
            take(xt, z, y);
            xt_s[i - v0] = Elem<T>::from_f(xt);
            z_s[i - v0] = Elem<T>::from_f(z);
        }
    } else {
        from_logits([&](int i, float xt, float z, float y) {
            take(xt, z, y);
            if (cache) {
                xt_s[i - v0] = Elem<T>::from_f(xt);
                z_s[i - v0] = Elem<T>::from_f(z);
            }
        });
    }
    __syncthreads();  // the slice copy is read by other threads in passes B and C
    mt = warp_maxf(mt);
    mz = warp_maxf(mz);
    acc.warp_merge();
    if (lane == 0) { s_red[0][warp] = mt; s_red[1][warp] = mz; }
    if (lane == 0) { s_acc[0][warp] = acc.m; s_acc[1][warp] = acc.S; s_acc[2][warp] = acc.A; }
    __syncthreads();
    if (warp == 0) {
        const float a = warp_maxf(lane < GATE_WARPS ? s_red[0][lane] : -INFINITY);
        const float b = warp_maxf(lane < GATE_WARPS ? s_red[1][lane] : -INFINITY);
        AccEnt t;
        if (lane < GATE_WARPS) t.merge(s_acc[0][lane], s_acc[1][lane], s_acc[2][lane]);
        t.warp_merge();
        if (lane == 0) { s_xa[0] = a; s_xa[1] = b; s_xa[2] = t.m; s_xa[3] = t.S; s_xa[4] = t.A; }
    }
    cluster.sync();
    if (warp == 0) {
        float a = -INFINITY, b = -INFINITY;
        AccEnt t;
        if (lane < C) {
            const float* r = cluster.map_shared_rank(s_xa, lane);
            a = r[0];
            b = r[1];
            t.merge(r[2], r[3], r[4]);
        }
        a = warp_maxf(a);
        b = warp_maxf(b);
        t.warp_merge();
        if (lane == 0) { s_glob[0] = a; s_glob[1] = b; s_glob[2] = t.S; s_glob[3] = t.A; }
    }
    __syncthreads();
    mt = s_glob[0];
    mz = s_glob[1];

    // pass B: S = sum exp(xt - mt) and the penalised one, accumulated in double
    // and rounded to float once: the float sum of the reference, exactly rounded
    // (pairs in packed f32x2 arithmetic: the same bits per element, half the instructions)
    KSum kt, kz;
    KSum2 kt2, kz2;
    for_slice2(
        [&](int, float2 xt, float2 z) {
            kt2.add(exp_cw2(fsub2(xt, f2(mt))));
            kz2.add(exp_cw2(fsub2(z, f2(mz))));
        },
        [&](int, float xt, float z) {
            kt.add(exp_cw(__fsub_rn(xt, mt)));
            kz.add(exp_cw(__fsub_rn(z, mz)));
        });
    double St = warp_sum_d(kt.value() + kt2.value());
    double Sz = warp_sum_d(kz.value() + kz2.value());
    if (lane == 0) { s_redd[0][warp] = St; s_redd[1][warp] = Sz; }
    __syncthreads();
    if (warp == 0) {
        const double a = warp_sum_d(lane < GATE_WARPS ? s_redd[0][lane] : 0.0);
        const double b = warp_sum_d(lane < GATE_WARPS ? s_redd[1][lane] : 0.0);
        if (lane == 0) { s_xb[0] = a; s_xb[1] = b; }
    }
    cluster.sync();
    if (warp == 0) {
        double a = 0.0, b = 0.0;
        if (lane < C) {
            const double* r = cluster.map_shared_rank(s_xb, lane);
            a = r[0];
            b = r[1];
        }
        a = warp_sum_d(a);
        b = warp_sum_d(b);
        if (lane == 0) { s_globd[0] = a; s_globd[1] = b; }
    }
    __syncthreads();
    const float Stf = (float)s_globd[0], Szf = (float)s_globd[1];
    const float rSt = __frcp_rn(Stf), rSz = __frcp_rn(Szf);
    // log in double, rounded once to float: the correctly rounded value
    // log-softmax = (x - m) - L.  torch's CPU kernels take L = R(log(R(S))) (the
    // default); with MENTAT_GATE_FLOAT_LOGSUM, L = log(S) in float, as its CUDA
    // kernels do.  The logs are correctly rounded (double, rounded once).
    const bool float_logsum = (P.flags & MENTAT_GATE_FLOAT_LOGSUM) != 0;
    const float Lt = float_logsum ? (float)log((double)Stf) : rnd<T>((float)log((double)rnd<T>(Stf)));
    const float Lz = float_logsum ? (float)log((double)Szf) : rnd<T>((float)log((double)rnd<T>(Szf)));

    // pass C: rounded entropies (terms summed in double) and the top-K of the
    // penalised log-probs
    KSum hs, hz;
    KSum2 hs2, hz2;
    uint64_t best[MENTAT_GATE_MAXK];
#pragma unroll
    for (int k = 0; k < MENTAT_GATE_MAXK; ++k) best[k] = 0ull;
    uint64_t kth = 0ull;  // best[K - 1], the smallest key kept
    // a NaN term counts as 0 (nan_to_num); in the pair form it is added as 0
    auto term2 = [&](float2 pl) {
        return make_float2(pl.x == pl.x ? rnd<T>(pl.x) : 0.f, pl.y == pl.y ? rnd<T>(pl.y) : 0.f);
    };
    auto pass_c2 = [&](int i, float2 xt, float2 z) {
        {
            const float2 dt = fsub2(xt, f2(mt));
            const float2 q = div_rn2(exp_cw2(dt), Stf, rSt);
            const float2 l = fsub2(dt, f2(Lt));
            hs2.add(term2(fmul2(make_float2(rnd<T>(q.x), rnd<T>(q.y)), make_float2(rnd<T>(l.x), rnd<T>(l.y)))));
        }
        const float2 dz = fsub2(z, f2(mz));
        const float2 l = fsub2(dz, f2(Lz));
        const float lpz0 = rnd<T>(l.x), lpz1 = rnd<T>(l.y);
        if (want_pen) {
            const float2 q = div_rn2(exp_cw2(dz), Szf, rSz);
            hz2.add(term2(fmul2(make_float2(rnd<T>(q.x), rnd<T>(q.y)), make_float2(lpz0, lpz1))));
        }
        uint64_t cur = topkey(lpz0, i);
        if (cur > kth) kth = topk_insert(best, K, cur);  // rare once the list has filled
        cur = topkey(lpz1, i + 1);
        if (cur > kth) kth = topk_insert(best, K, cur);
    };
    for_slice2(pass_c2, [&](int i, float xt, float z) {
        {
            const float dt = __fsub_rn(xt, mt);
            const float p = rnd<T>(div_rn(exp_cw(dt), Stf, rSt));
            const float lp = rnd<T>(__fsub_rn(dt, Lt));
            const float pl = __fmul_rn(p, lp);
            if (pl == pl) hs.add(rnd<T>(pl));  // nan_to_num: NaN terms count as 0
        }
        const float dz = __fsub_rn(z, mz);
        const float lpz = rnd<T>(__fsub_rn(dz, Lz));
        if (want_pen) {
            const float p = rnd<T>(div_rn(exp_cw(dz), Szf, rSz));
            const float pl = __fmul_rn(p, lpz);
            if (pl == pl) hz.add(rnd<T>(pl));
        }
        const uint64_t cur = topkey(lpz, i);
        if (cur > kth) kth = topk_insert(best, K, cur);  // rare once the list has filled
    });
    const double Hs = warp_sum_d(hs.value() + hs2.value());
    const double Hz = warp_sum_d(hz.value() + hz2.value());
    if (lane == 0) { s_redd[0][warp] = Hs; s_redd[1][warp] = Hz; }
    warp_topk_merge(K, [&](int head) {
        uint64_t v = 0ull;
#pragma unroll
        for (int j = 0; j < MENTAT_GATE_MAXK; ++j)
            if (j == head) v = best[j];
        return v;
    }, s_keys[warp]);
    __syncthreads();
    if (warp == 0) {
        const double a = warp_sum_d(lane < GATE_WARPS ? s_redd[0][lane] : 0.0);
        const double b = warp_sum_d(lane < GATE_WARPS ? s_redd[1][lane] : 0.0);
        warp_topk_merge(K, [&](int head) {
            return lane < GATE_WARPS && head < K ? s_keys[lane][head] : 0ull;
        }, s_xk);
        if (lane == 0) { s_xc[0] = a; s_xc[1] = b; }
    }
    cluster.sync();
    if (rank == 0 && warp == 0) {  // the leaf's sums, top-K and decision
        double a = 0.0, b = 0.0;
        const uint64_t* rk = nullptr;
        if (lane < C) {
            const double* r = cluster.map_shared_rank(s_xc, lane);
            a = r[0];
            b = r[1];
            rk = cluster.map_shared_rank(s_xk, lane);
        }
        a = warp_sum_d(a);
        b = warp_sum_d(b);
        warp_topk_merge(K, [&](int head) { return lane < C && head < K ? rk[head] : 0ull; }, s_keys[0]);
        __syncwarp();
        if (lane == 0) {
            const uint64_t* res = s_keys[0];
            mentat_gate_out o;
            const double H = -(double)rnd<T>((float)a);
            o.entropy = H;
            o.pen_entropy = want_pen ? -(double)rnd<T>((float)b) : 0.0;
            o.entropy_acc = (double)logf(s_glob[2]) - (double)s_glob[3] / (double)s_glob[2];
            const double eo = ema_old[leaf];
            double ema;
            if (eo != eo) ema = H;
            else ema = __dadd_rn(__dmul_rn(P.alpha, H), __dmul_rn(__dsub_rn(1.0, P.alpha), eo));
            const double util = __ddiv_rn((double)P.num_active, (double)(P.M > 1 ? P.M : 1));
            const double dyn = __dmul_rn(P.mult, __dadd_rn(1.0, __dmul_rn(__dmul_rn(2.0, util), util)));
            double warm = 1.0;
            if (P.step < P.window) {
                const double t = __ddiv_rn((double)P.step, (double)(P.window > 1 ? P.window : 1));
                warm = __dadd_rn(P.initial, __dmul_rn(__dsub_rn(1.0, P.initial), t));
            }
            const double tau = __dmul_rn(__dmul_rn(ema, dyn), warm);
            o.ema = ema;
            o.tau = tau;
            o.branch = (H > tau) && (P.M - P.num_active >= K) ? 1 : 0;
            o.argmax = key_idx(res[0]);
            o.argmax_lp = key_val(res[0]);
#pragma unroll
            for (int k = 0; k < MENTAT_GATE_MAXK; ++k) {
                o.topk_ids[k] = k < K ? key_idx(res[k]) : -1;
                o.topk_lps[k] = k < K ? key_val(res[k]) : 0.f;
            }
            o.pad[0] = o.pad[1] = o.pad[2] = 0;
            out[leaf] = o;
        }
    }
    cluster.sync();  // every CTA's shared memory stays alive until rank 0 has read it
}

// shared memory a CTA may hold: the whole slice cache when it fits
constexpr int GATE_SMEM_MAX = 200 * 1024;

template <typename T>
static int launch_gate(const void* logits, int n, int V, int64_t ld, const int32_t* hp, const int32_t* hi,
                       const double* ema, const mentat_gate_params& P, mentat_gate_out* out, cudaStream_t s) {
    const int per = gate_slice<T>(V);
    const size_t bm = (size_t)gate_bitmap_bytes(per);
    const size_t cached = bm + (size_t)2 * per * sizeof(T);
    const int cache = cached <= (size_t)GATE_SMEM_MAX ? 1 : 0;
    const size_t smem = cache ? cached : bm;  // V <= 2^20 keeps the bitmap alone within 16 KB
    // the dynamic shared-memory limit is a per-device attribute
    static bool attr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MENTAT_ERR_CUDA;
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(k_gate<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, GATE_SMEM_MAX) !=
            cudaSuccess)
            return MENTAT_ERR_CUDA;
        attr[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n * GATE_CLUSTER);
    cfg.blockDim = dim3(GATE_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = GATE_CLUSTER;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_gate<T>, reinterpret_cast<const T*>(logits), V, ld, hp, hi, ema, P, out,
                           cache) != cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

}  // namespace mentat

using namespace mentat;

extern "C" int mentat_gate_step(const void* logits, int32_t dtype, int32_t n, int32_t V, int64_t ld,
                                const int32_t* hist_ptr, const int32_t* hist_ids, const double* ema_old,
                                const mentat_gate_params* P, mentat_gate_out* out, cudaStream_t s) {
    if (n < 0 || V <= 0 || V > (1 << 20) || !P || P->K < 1 || P->K > MENTAT_GATE_MAXK || P->K > V || ld < V ||
        P->temperature <= 0.0)
        return MENTAT_ERR_ARG;
    if (n == 0) return MENTAT_OK;
    if (!logits || !hist_ptr || !hist_ids || !ema_old || !out) return MENTAT_ERR_ARG;
    switch (dtype) {
        case MENTAT_BF16: return launch_gate<__nv_bfloat16>(logits, n, V, ld, hist_ptr, hist_ids, ema_old, *P, out, s);
        case MENTAT_F16: return launch_gate<__half>(logits, n, V, ld, hist_ptr, hist_ids, ema_old, *P, out, s);
        case MENTAT_F32: return launch_gate<float>(logits, n, V, ld, hist_ptr, hist_ids, ema_old, *P, out, s);
        default: return MENTAT_ERR_UNSUPPORTED;
    }
}
