// Fused logits -> entropy -> gate -> decision kernel, one CTA per leaf.
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

#include "common.cuh"

namespace mentat {

constexpr int GATE_THREADS = 1024;

template <typename T> __device__ __forceinline__ float rnd(float x) { return Elem<T>::to_f(Elem<T>::from_f(x)); }
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }

// online (max, sum exp) accumulator
struct MS {
    float m, s;
    __device__ __forceinline__ void add(float x) {
        if (x == -INFINITY) return;
        if (x > m) {
            s = (m == -INFINITY) ? 1.f : s * expf(m - x) + 1.f;
            m = x;
        } else {
            s += expf(x - m);
        }
    }
    __device__ __forceinline__ void merge(float om, float os) {
        if (om == -INFINITY) return;
        if (m == -INFINITY) { m = om; s = os; return; }
        if (om > m) { s = s * expf(m - om) + os; m = om; }
        else s += os * expf(om - m);
    }
};
// online (max, sum e, sum e * (y - max)) for the float-accurate entropy
struct MSA {
    float m, s, a;
    __device__ __forceinline__ void add(float y) {
        if (y == -INFINITY) return;
        if (m == -INFINITY) { m = y; s = 1.f; a = 0.f; return; }
        if (y > m) {
            const float sc = expf(m - y);
            a = (a + s * (m - y)) * sc;
            s = s * sc + 1.f;
            m = y;
        } else {
            const float e = expf(y - m);
            s += e;
            a += e * (y - m);
        }
    }
    __device__ __forceinline__ void merge(float om, float os, float oa) {
        if (om == -INFINITY) return;
        if (m == -INFINITY) { m = om; s = os; a = oa; return; }
        if (om > m) {
            const float sc = expf(m - om);
            a = (a + s * (m - om)) * sc + oa;
            s = s * sc + os;
            m = om;
        } else {
            const float sc = expf(om - m);
            a += (oa + os * (om - m)) * sc;
            s += os * sc;
        }
    }
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

template <typename T>
__global__ void __launch_bounds__(GATE_THREADS)
k_gate(const T* __restrict__ logits, int V, int64_t ld, const int32_t* __restrict__ hist_ptr,
       const int32_t* __restrict__ hist_ids, const double* __restrict__ ema_old, mentat_gate_params P,
       mentat_gate_out* __restrict__ out) {
    extern __shared__ uint32_t bitmap[];
    __shared__ float sh_f[3][32];
    __shared__ float sh_g[3][32];
    __shared__ float sh_a[32];
    __shared__ float sh_b[4];
    __shared__ uint64_t sh_keys[32][MENTAT_GATE_MAXK];
    const int leaf = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwords = (V + 31) >> 5;
    const T* x = logits + (int64_t)leaf * ld;
    const float Tf = (float)P.temperature, pf = (float)P.penalty;
    const bool use_t = P.temperature != 1.0;
    const int K = P.K;

    for (int w = tid; w < nwords; w += GATE_THREADS) bitmap[w] = 0u;
    __syncthreads();
    for (int h = hist_ptr[leaf] + tid; h < hist_ptr[leaf + 1]; h += GATE_THREADS) {
        const int id = hist_ids[h];
        if (id >= 0 && id < V) atomicOr(&bitmap[id >> 5], 1u << (id & 31));
    }
    __syncthreads();

    // pass 1: maxima and sums
    MS st{-INFINITY, 0.f}, sz{-INFINITY, 0.f};
    MSA acc{-INFINITY, 0.f, 0.f};
    for (int i = tid; i < V; i += GATE_THREADS) {
        const float xv = Elem<T>::to_f(x[i]);
        const float y = use_t ? xv / Tf : xv;
        st.add(use_t ? rnd<T>(y) : xv);
        acc.add(y);
        float z = xv;
        if ((bitmap[i >> 5] >> (i & 31)) & 1u) z = xv > 0.f ? rnd<T>(xv / pf) : rnd<T>(xv * pf);
        sz.add(z);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        float a = __shfl_xor_sync(0xffffffffu, st.m, o), b = __shfl_xor_sync(0xffffffffu, st.s, o);
        st.merge(a, b);
        a = __shfl_xor_sync(0xffffffffu, sz.m, o);
        b = __shfl_xor_sync(0xffffffffu, sz.s, o);
        sz.merge(a, b);
        a = __shfl_xor_sync(0xffffffffu, acc.m, o);
        b = __shfl_xor_sync(0xffffffffu, acc.s, o);
        float cc = __shfl_xor_sync(0xffffffffu, acc.a, o);
        acc.merge(a, b, cc);
    }
    if (lane == 0) {
        sh_f[0][warp] = st.m; sh_f[1][warp] = st.s; sh_f[2][warp] = sz.m;
        sh_g[0][warp] = sz.s; sh_g[1][warp] = acc.m; sh_g[2][warp] = acc.s;
        sh_a[warp] = acc.a;
    }
    __syncthreads();
    __shared__ float sh_acc[3];
    if (warp == 0) {
        MS a{sh_f[0][lane], sh_f[1][lane]}, b{sh_f[2][lane], sh_g[0][lane]};
        MSA cacc{sh_g[1][lane], sh_g[2][lane], sh_a[lane]};
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            float u = __shfl_xor_sync(0xffffffffu, a.m, o), v = __shfl_xor_sync(0xffffffffu, a.s, o);
            a.merge(u, v);
            u = __shfl_xor_sync(0xffffffffu, b.m, o);
            v = __shfl_xor_sync(0xffffffffu, b.s, o);
            b.merge(u, v);
            u = __shfl_xor_sync(0xffffffffu, cacc.m, o);
            v = __shfl_xor_sync(0xffffffffu, cacc.s, o);
            float w = __shfl_xor_sync(0xffffffffu, cacc.a, o);
            cacc.merge(u, v, w);
        }
        if (lane == 0) {
            sh_b[0] = a.m; sh_b[1] = a.s; sh_b[2] = b.m; sh_b[3] = b.s;
            sh_acc[0] = cacc.m; sh_acc[1] = cacc.s; sh_acc[2] = cacc.a;
        }
    }
    __syncthreads();
    const float mt = sh_b[0], St = sh_b[1], mz = sh_b[2], Sz = sh_b[3];
    const float Lt = rnd<T>(logf(rnd<T>(St)));
    const float Lz = rnd<T>(logf(rnd<T>(Sz)));

    // pass 2: rounded entropies and top-K of the penalised log-probs
    float Hs = 0.f, Hz = 0.f;
    uint64_t best[MENTAT_GATE_MAXK];
#pragma unroll
    for (int k = 0; k < MENTAT_GATE_MAXK; ++k) best[k] = 0ull;
    for (int i = tid; i < V; i += GATE_THREADS) {
        const float xv = Elem<T>::to_f(x[i]);
        const float xt = use_t ? rnd<T>(xv / Tf) : xv;
        {
            const float p = rnd<T>(expf(xt - mt) / St);
            const float lp = rnd<T>((xt - mt) - Lt);
            float pl = rnd<T>(p * lp);
            if (pl != pl) pl = 0.f;
            Hs += pl;
        }
        float z = xv;
        if ((bitmap[i >> 5] >> (i & 31)) & 1u) z = xv > 0.f ? rnd<T>(xv / pf) : rnd<T>(xv * pf);
        const float lpz = rnd<T>((z - mz) - Lz);
        {
            const float p = rnd<T>(expf(z - mz) / Sz);
            float pl = rnd<T>(p * lpz);
            if (pl != pl) pl = 0.f;
            Hz += pl;
        }
        uint64_t cur = topkey(lpz, i);
#pragma unroll
        for (int k = 0; k < MENTAT_GATE_MAXK; ++k) {
            if (k < K && cur > best[k]) {
                const uint64_t t = best[k];
                best[k] = cur;
                cur = t;
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        Hs += __shfl_xor_sync(0xffffffffu, Hs, o);
        Hz += __shfl_xor_sync(0xffffffffu, Hz, o);
    }
    if (lane == 0) {
        sh_f[1][warp] = Hs;
        sh_f[2][warp] = Hz;
    }
    {  // warp top-K: K rounds of max extraction over the lanes' sorted lists
        int head = 0;
        for (int k = 0; k < K; ++k) {
            uint64_t mine = 0ull;
#pragma unroll
            for (int j = 0; j < MENTAT_GATE_MAXK; ++j)
                if (j == head) mine = best[j];
            const uint64_t w = warp_max_u64(mine);
            if (w == mine && w != 0ull) ++head;
            if (lane == 0) sh_keys[warp][k] = w;
        }
    }
    __syncthreads();
    if (warp == 0) {
        float a = sh_f[1][lane], b = sh_f[2][lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, o);
            b += __shfl_xor_sync(0xffffffffu, b, o);
        }
        int head = 0;
        uint64_t res[MENTAT_GATE_MAXK];
#pragma unroll
        for (int k = 0; k < MENTAT_GATE_MAXK; ++k) res[k] = 0ull;
        for (int k = 0; k < K; ++k) {
            const uint64_t mine = head < K ? sh_keys[lane][head] : 0ull;
            const uint64_t w = warp_max_u64(mine);
            if (w == mine && w != 0ull) ++head;
#pragma unroll
            for (int j = 0; j < MENTAT_GATE_MAXK; ++j)
                if (j == k) res[j] = w;
        }
        if (lane == 0) {
            mentat_gate_out o;
            const double H = -(double)rnd<T>(a);
            o.entropy = H;
            o.pen_entropy = -(double)rnd<T>(b);
            o.entropy_acc = (double)logf(sh_acc[1]) - (double)sh_acc[2] / (double)sh_acc[1];
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
}

template <typename T>
static int launch_gate(const void* logits, int n, int V, int64_t ld, const int32_t* hp, const int32_t* hi,
                       const double* ema, const mentat_gate_params& P, mentat_gate_out* out, cudaStream_t s) {
    const size_t smem = (size_t)((V + 31) / 32) * 4;
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(k_gate<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        attr_set = true;
    }
    k_gate<T><<<n, GATE_THREADS, smem, s>>>(reinterpret_cast<const T*>(logits), V, ld, hp, hi, ema, P, out);
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
