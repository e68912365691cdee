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

template <typename T>
__global__ void __launch_bounds__(GATE_THREADS, sizeof(T) == 4 ? 1 : 2)  // fp32 needs > 64 registers
k_gate(const T* __restrict__ logits, int V, int64_t ld, const int32_t* __restrict__ hist_ptr,
       const int32_t* __restrict__ hist_ids, const double* __restrict__ ema_old, mentat_gate_params P,
       mentat_gate_out* __restrict__ out) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ uint32_t bitmap[];
    __shared__ float s_red[4][GATE_WARPS];
    __shared__ uint64_t s_keys[GATE_WARPS][MENTAT_GATE_MAXK];
    __shared__ float s_xa[2], s_xb[4], s_xc[2];      // this CTA's values of passes A, B, C
    __shared__ uint64_t s_xk[MENTAT_GATE_MAXK];      // this CTA's top-K
    __shared__ float s_glob[6];
    const int C = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int leaf = blockIdx.x / C, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = ((V + C - 1) / C + GATE_VEC - 1) / GATE_VEC * GATE_VEC;
    const int v0 = min(V, rank * per), v1 = min(V, v0 + per);
    const int nwords = (per + 31) >> 5;
    const T* x = logits + (int64_t)leaf * ld;
    const float Tf = (float)P.temperature, pf = (float)P.penalty;
    const bool use_t = P.temperature != 1.0;
    const int K = P.K;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(v0 * sizeof(T))) & 15) == 0;

    for (int w = tid; w < nwords; w += GATE_THREADS) bitmap[w] = 0u;
    __syncthreads();
    for (int h = hist_ptr[leaf] + tid; h < hist_ptr[leaf + 1]; h += GATE_THREADS) {
        const int id = hist_ids[h];
        if (id >= v0 && id < v1) atomicOr(&bitmap[(id - v0) >> 5], 1u << ((id - v0) & 31));
    }
    __syncthreads();
    // f(i, x_i, xt_i, z_i, y_i) for every element of the slice: vector steps, then the tail
    auto for_slice = [&](auto&& f) {
        auto elem = [&](int i, float xv, uint32_t hit) {
            const float y = use_t ? xv / Tf : xv;
            const float xt = use_t ? rnd<T>(y) : xv;
            float z = xv;
            if (hit) z = xv > 0.f ? rnd<T>(xv / pf) : rnd<T>(xv * pf);
            f(i, xt, z, y);
        };
        int tail = v0;
        if (vec) {
            constexpr int VW = 16 / sizeof(T);  // elements per 16-byte load
            for (int j = v0 + tid * VW; j + VW <= v1; j += GATE_THREADS * VW) {
                alignas(16) T e[VW];
                *reinterpret_cast<uint4*>(e) = *reinterpret_cast<const uint4*>(x + j);
                const uint32_t bits = bitmap[(j - v0) >> 5] >> ((j - v0) & 31);
#pragma unroll
                for (int u = 0; u < VW; ++u) elem(j + u, Elem<T>::to_f(e[u]), (bits >> u) & 1u);
            }
            tail = v0 + (v1 - v0) / VW * VW;
        }
        for (int i = tail + tid; i < v1; i += GATE_THREADS)
            elem(i, Elem<T>::to_f(x[i]), (bitmap[(i - v0) >> 5] >> ((i - v0) & 31)) & 1u);
    };

    // pass A: maxima
    float mt = -INFINITY, mz = -INFINITY;
    for_slice([&](int, float xt, float z, float) {
        mt = fmaxf(mt, xt);
        mz = fmaxf(mz, z);
    });
    mt = warp_maxf(mt);
    mz = warp_maxf(mz);
    if (lane == 0) { s_red[0][warp] = mt; s_red[1][warp] = mz; }
    __syncthreads();
    if (warp == 0) {
        const float a = warp_maxf(lane < GATE_WARPS ? s_red[0][lane] : -INFINITY);
        const float b = warp_maxf(lane < GATE_WARPS ? s_red[1][lane] : -INFINITY);
        if (lane == 0) { s_xa[0] = a; s_xa[1] = b; }
    }
    cluster.sync();
    if (warp == 0) {
        float a = -INFINITY, b = -INFINITY;
        if (lane < C) {
            const float* r = cluster.map_shared_rank(s_xa, lane);
            a = r[0];
            b = r[1];
        }
        a = warp_maxf(a);
        b = warp_maxf(b);
        if (lane == 0) { s_glob[0] = a; s_glob[1] = b; }
    }
    __syncthreads();
    mt = s_glob[0];
    mz = s_glob[1];

    // pass B: sums of exp about the maxima (the accurate entropy's shifted by mt)
    float St = 0.f, Sz = 0.f, Sa = 0.f, Aa = 0.f;
    for_slice([&](int, float xt, float z, float y) {
        St += expf(xt - mt);
        Sz += expf(z - mz);
        const float d = y - mt;
        const float ea = expf(d);
        Sa += ea;
        Aa += ea * d;
    });
    St = warp_sum(St);
    Sz = warp_sum(Sz);
    Sa = warp_sum(Sa);
    Aa = warp_sum(Aa);
    if (lane == 0) { s_red[0][warp] = St; s_red[1][warp] = Sz; s_red[2][warp] = Sa; s_red[3][warp] = Aa; }
    __syncthreads();
    if (warp == 0) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = warp_sum(lane < GATE_WARPS ? s_red[k][lane] : 0.f);
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 4; ++k) s_xb[k] = v[k];
        }
    }
    cluster.sync();
    if (warp == 0) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (lane < C) {
            const float* r = cluster.map_shared_rank(s_xb, lane);
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = r[k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = warp_sum(v[k]);
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 4; ++k) s_glob[2 + k] = v[k];
        }
    }
    __syncthreads();
    St = s_glob[2];
    Sz = s_glob[3];
    const float Lt = rnd<T>(logf(rnd<T>(St)));
    const float Lz = rnd<T>(logf(rnd<T>(Sz)));

    // pass C: rounded entropies and the top-K of the penalised log-probs
    float Hs = 0.f, Hz = 0.f;
    uint64_t best[MENTAT_GATE_MAXK];
#pragma unroll
    for (int k = 0; k < MENTAT_GATE_MAXK; ++k) best[k] = 0ull;
    uint64_t kth = 0ull;  // best[K - 1], the smallest key kept
    for_slice([&](int i, float xt, float z, float) {
        {
            const float p = rnd<T>(expf(xt - mt) / St);
            const float lp = rnd<T>((xt - mt) - Lt);
            float pl = rnd<T>(p * lp);
            if (pl != pl) pl = 0.f;
            Hs += pl;
        }
        const float lpz = rnd<T>((z - mz) - Lz);
        {
            const float p = rnd<T>(expf(z - mz) / Sz);
            float pl = rnd<T>(p * lpz);
            if (pl != pl) pl = 0.f;
            Hz += pl;
        }
        uint64_t cur = topkey(lpz, i);
        if (cur > kth) {
#pragma unroll
            for (int k = 0; k < MENTAT_GATE_MAXK; ++k) {
                if (k < K && cur > best[k]) {
                    const uint64_t t = best[k];
                    best[k] = cur;
                    cur = t;
                }
            }
#pragma unroll
            for (int k = 0; k < MENTAT_GATE_MAXK; ++k)
                if (k == K - 1) kth = best[k];
        }
    });
    Hs = warp_sum(Hs);
    Hz = warp_sum(Hz);
    if (lane == 0) { s_red[0][warp] = Hs; s_red[1][warp] = Hz; }
    warp_topk_merge(K, [&](int head) {
        uint64_t v = 0ull;
#pragma unroll
        for (int j = 0; j < MENTAT_GATE_MAXK; ++j)
            if (j == head) v = best[j];
        return v;
    }, s_keys[warp]);
    __syncthreads();
    if (warp == 0) {
        const float a = warp_sum(lane < GATE_WARPS ? s_red[0][lane] : 0.f);
        const float b = warp_sum(lane < GATE_WARPS ? s_red[1][lane] : 0.f);
        warp_topk_merge(K, [&](int head) {
            return lane < GATE_WARPS && head < K ? s_keys[lane][head] : 0ull;
        }, s_xk);
        if (lane == 0) { s_xc[0] = a; s_xc[1] = b; }
    }
    cluster.sync();
    if (rank == 0 && warp == 0) {  // the leaf's sums, top-K and decision
        float a = 0.f, b = 0.f;
        const uint64_t* rk = nullptr;
        if (lane < C) {
            const float* r = cluster.map_shared_rank(s_xc, lane);
            a = r[0];
            b = r[1];
            rk = cluster.map_shared_rank(s_xk, lane);
        }
        a = warp_sum(a);
        b = warp_sum(b);
        warp_topk_merge(K, [&](int head) { return lane < C && head < K ? rk[head] : 0ull; }, s_keys[0]);
        __syncwarp();
        if (lane == 0) {
            const uint64_t* res = s_keys[0];
            mentat_gate_out o;
            const double H = -(double)rnd<T>(a);
            o.entropy = H;
            o.pen_entropy = -(double)rnd<T>(b);
            o.entropy_acc = (double)logf(s_glob[4]) - (double)s_glob[5] / (double)s_glob[4];
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

template <typename T>
static int launch_gate(const void* logits, int n, int V, int64_t ld, const int32_t* hp, const int32_t* hi,
                       const double* ema, const mentat_gate_params& P, mentat_gate_out* out, cudaStream_t s) {
    const int per = ((V + GATE_CLUSTER - 1) / GATE_CLUSTER + GATE_VEC - 1) / GATE_VEC * GATE_VEC;
    const size_t smem = (size_t)((per + 31) / 32) * 4;
    // V <= 2^20 keeps the slice bitmap within 16 KB, under the default dynamic limit
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
    if (cudaLaunchKernelEx(&cfg, k_gate<T>, reinterpret_cast<const T*>(logits), V, ld, hp, hi, ema, P, out) !=
        cudaSuccess)
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
