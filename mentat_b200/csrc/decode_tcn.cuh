// Narrow tensor-core decode units: <= 32 query rows (a branch's own tokens, or
// a prefix shared by few rows).  Included by decode_attention.cu after
// decode_tc.cuh (shares its PTX wrappers and tensor maps).
//
// The contraction is transposed so that the 128 tokens of a tile, not the few
// query rows, fill the MMA's M dimension:
//   S^T[128 tok x 32 rows]   = K_tile[128 tok x D] . Q^T          (8 MMAs, N=32)
//   O^T[D x 32 rows]        += V_tile^T[D x 128 tok] . P^T         (8 MMAs, N=32,
//                                                                  V read MN-major)
// Thread t of the four softmax warps owns token t (TMEM lane t) and holds its
// 32 row scores.  Row statistics are lazy: a row's reference max is set on the
// first tile and raised only when a block-wide vote finds a score above it by
// more than 2^8 (then O^T's column and the running sums are rescaled); the
// per-row sums stay in registers, one partial per thread, and are reduced once
// per unit with a 31-shuffle transpose-reduce.
// Roles: warps 0-3 softmax, warp 4 lane 0 MMA issue, warps 5 and 7 TMA issue
// of K and of V (lanes 0-7, one 16-token block each), each through a stage ring
// of its own (a K stage is free once its Q K^T has run, a V stage once its P V
// has), warp 6 claims units and stages their Q rows into one of two unit slots
// while the current unit runs.
// Every mbarrier wait is bounded (TC_WAIT_CYCLES); on timeout the CTA records
// HDR_TC_ABORT, drains its copies in flight and frees its TMEM.

#pragma once

namespace mentat {

#ifdef MENTAT_TC_TRACE
#define TCN_TRACE(k) do { if (blockIdx.x == 0 && (threadIdx.x == 128 || threadIdx.x == 0) && g_trace_on && (k) < 2048) g_tc_trace[(k) + (threadIdx.x ? 0 : 2048)] = clock64(); } while (0)
#else
#define TCN_TRACE(k) do { } while (0)
#endif

constexpr int TCN_ROWS = 32;                        // query rows (MMA N)
constexpr int TCN_TILE = 128;                       // tokens per tile (MMA M)
#ifndef MENTAT_TCN_KST
#define MENTAT_TCN_KST 3
#endif
#ifndef MENTAT_TCN_VST
#define MENTAT_TCN_VST 3
#endif
constexpr int TCN_KST = MENTAT_TCN_KST;              // K stages (freed after Q K^T)
constexpr int TCN_VST = MENTAT_TCN_VST;              // V stages (freed after P V)
static_assert(TCN_KST >= 2 && TCN_VST >= 2 && TCN_KST + TCN_VST <= 6, "six 32 KB stages fit beside Q and P");
constexpr int TCN_THREADS = 8 * 32;  // 4 softmax, MMA, K TMA, scheduler, V TMA
constexpr int TCN_Q_BYTES = 2 * TCN_ROWS * 128;      // [half][32 rows][128 B]
constexpr int TCN_KV_STAGE = 2 * TCN_TILE * 128;     // [half][128 tok][128 B] = 32 KB
constexpr int TCN_P_BYTES = TCN_TILE * TCN_ROWS * 2;  // [128 tok][32 rows] bf16, 64-byte swizzle = 8 KB
constexpr int TCN_OFF_Q = 0;
constexpr int TCN_OFF_K = TCN_OFF_Q + 2 * TCN_Q_BYTES;    // two unit slots
constexpr int TCN_OFF_V = TCN_OFF_K + TCN_KST * TCN_KV_STAGE;
constexpr int TCN_OFF_P = TCN_OFF_V + TCN_VST * TCN_KV_STAGE;  // two buffers
constexpr int TCN_OFF_BAR = TCN_OFF_P + 2 * TCN_P_BYTES;
constexpr int TCN_SMEM = TCN_OFF_BAR + 256 + 1024;
constexpr uint32_t TCN_TMEM_COLS = 128;             // O^T at 0, S^T[buf] at 32 + 32 * buf

// lane l ends with op over the 32 lanes of a[l]; a[] is clobbered
template <bool MAX>
__device__ __forceinline__ float transpose_reduce32(float (&a)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int k = 0; k < o; ++k) {
            const float send = up ? a[k] : a[k + o];
            const float keep = up ? a[k + o] : a[k];
            const float recv = __shfl_xor_sync(0xffffffffu, send, o);
            a[k] = MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    return a[0];
}

// named barrier `id` over `count` threads with an OR of `flag`
__device__ __forceinline__ int bar_sync_or_id(int id, int count, int flag) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %3, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(flag), "r"(count), "r"(id)
        : "memory");
    return (int)out;
}

template <typename T, int D>
__global__ void __launch_bounds__(TCN_THREADS, 1)
k_units_tcn(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
            mentat_kv_cache c, int layer, const int32_t* slots, const T* __restrict__ q, int64_t q_stride, int Hq,
            float scale_log2, DecodeWs ws, int max_parts) {
    static_assert(D == 128, "the narrow kernel is built for head_dim 128");
    constexpr int HALVES = D / 64;
    constexpr int FMT = Elem<T>::code == MENTAT_BF16 ? 1 : 0;
    constexpr uint32_t IDESC_QK = idesc_f16(FMT, 128, TCN_ROWS, 0, 0);  // A = K (K-major), B = Q (K-major)
    constexpr uint32_t IDESC_PV = idesc_f16(FMT, 128, TCN_ROWS, 1, 1);  // A = V^T (MN-major), B = P^T (MN-major)
    constexpr int QV = TCN_ROWS * (D / 8) / 32;  // 16-byte Q chunks per producer lane
    extern __shared__ uint8_t tcn_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tcn_smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ __align__(8) uint64_t s_probe_bar;
    __shared__ int s_unit[2][8];  // per unit slot: q_lo, q_hi, t0u, t1u, ord, head, valid, sequence slot
    __shared__ float s_mref[TCN_ROWS], s_fac[TCN_ROWS], s_red[4][TCN_ROWS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool softmax = warp < 4;
    const bool leader = warp == 4 && lane == 0;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_kfull0 = sbase + TCN_OFF_BAR;         // [NST] K tile landed
    const uint32_t bar_s0 = bar_kfull0 + 8 * TCN_KST;        // [2] S^T buffer written
    const uint32_t bar_pv0 = bar_s0 + 16;                    // [2] P V done, per P buffer
    const uint32_t bar_kempty0 = bar_pv0 + 16;               // [NST] K stage read by its Q K^T
    const uint32_t bar_ufull0 = bar_kempty0 + 8 * TCN_KST;   // [2] unit slot filled (producer)
    const uint32_t bar_uempty0 = bar_ufull0 + 16;            // [2] unit slot released (consumers)
    const uint32_t bar_vfull0 = bar_uempty0 + 16;            // [NST] V tile landed
    const uint32_t bar_vempty0 = bar_vfull0 + 8 * TCN_VST;   // [VST] V stage read by its P V
    const int Hkv = c.num_kv_heads, G = Hq / Hkv;

    for (int i = tid; i < TCN_OFF_BAR / 16; i += TCN_THREADS) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        for (int st = 0; st < TCN_KST; ++st) {
            mbar_init(bar_kfull0 + 8 * st, 1);
            mbar_init(bar_kempty0 + 8 * st, 1);
        }
        for (int st = 0; st < TCN_VST; ++st) {
            mbar_init(bar_vfull0 + 8 * st, 1);
            mbar_init(bar_vempty0 + 8 * st, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_s0 + 8 * b, 1);
            mbar_init(bar_pv0 + 8 * b, 1);
            mbar_init(bar_ufull0 + 8 * b, 1);
            mbar_init(bar_uempty0 + 8 * b, 1);
        }
        mbar_init(smem_u32(&s_probe_bar), 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_u32(&s_tmem), TCN_TMEM_COLS);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    // Launched after the wide kernel, which waited for the plan before it let
    // this one start: the plan is complete here.  This kernel does not wait for
    // the wide one until its end, so the two overlap on the SMs the wide kernel
    // leaves free.
    griddep_launch();
    if (tid == 0 && !wait_probe(smem_u32(&s_probe_bar))) s_abort = 1;
    __syncthreads();  // every role sees the probe's outcome before it claims or streams a unit
    TL_FIRST(6);

#ifdef MENTAT_TC_TRACE
    bool g_trace_on = true;
#endif
    uint32_t issued = 0;  // TMA warps: tiles whose copies have been issued
    const int nunits = ws.hdr[HDR_NTCN];
    const int64_t nwork = (int64_t)nunits * Hkv;

    if (warp == 6) {
        // Scheduler warp: claims units into the two unit slots, staging each
        // one's Q rows.  A slot is refilled as soon as the consumers release
        // it, so the next unit is ready a whole unit ahead.
        for (uint32_t k = 0;; ++k) {
            const int slot = k & 1;
            int ok = 1, w = 0;
            if (lane == 0) {
                if (k >= 2) ok = mbar_wait(bar_uempty0 + 8 * slot, ((k >> 1) - 1) & 1);
                if (ok) w = atomicAdd(&ws.hdr[HDR_TCN_NEXT], 1);
            }
            const bool valid = __shfl_sync(0xffffffffu, (ok && !s_abort && w < nwork) ? 1 : 0, 0) != 0;
            w = __shfl_sync(0xffffffffu, w, 0);
            int q_lo = 0, q_hi = 0, t0u = 0, t1u = 0, ord = 0, head = 0, seq_slot = 0;
            if (valid) {
                const int u = w / Hkv;
                head = w % Hkv;
                const int32_t* U = ws.units_tcn + (int64_t)u * UNIT_INTS;
                q_lo = U[0], q_hi = U[1], t0u = U[2], t1u = U[3], ord = U[4];
                seq_slot = slots[q_lo];
                const int R = (q_hi - q_lo + 1) * G;  // <= 32
                uint4 v[QV];
#pragma unroll
                for (int j = 0; j < QV; ++j) {
                    const int idx = lane + 32 * j, r = idx / (D / 8), ch = idx % (D / 8);
                    v[j] = make_uint4(0, 0, 0, 0);
                    if (r < R) {
                        const int seq = q_lo + r / G, g = r % G;
                        v[j] = *reinterpret_cast<const uint4*>(q + (int64_t)seq * q_stride + (int64_t)(head * G + g) * D + ch * 8);
                    }
                }
                uint8_t* qs = smem + TCN_OFF_Q + slot * TCN_Q_BYTES;
#pragma unroll
                for (int j = 0; j < QV; ++j) {
                    const int idx = lane + 32 * j, r = idx / (D / 8), ch = idx % (D / 8);
                    *reinterpret_cast<uint4*>(qs + (ch >> 3) * (TCN_ROWS * 128) + sw128_off(r, ch & 7)) = v[j];
                }
                fence_proxy_async();  // Q is read by the tensor cores
            }
            __syncwarp();
            if (lane == 0) {
                int* su = s_unit[slot];
                su[0] = q_lo, su[1] = q_hi, su[2] = t0u, su[3] = t1u, su[4] = ord, su[5] = head;
                su[6] = valid ? 1 : 0, su[7] = seq_slot;
                mbar_arrive(bar_ufull0 + 8 * slot);
            }
            if (!valid) break;
        }
    } else if (warp == 5 || warp == 7) {
        // TMA warps: warp 5 streams each published unit's K tiles and warp 7 its V
        // tiles, each through a stage ring of its own (a K stage is free again once
        // its Q K^T has run, a V stage once its P V has).  Lanes 0-7 read the tile's
        // block ids (one tile ahead) and each issues the copies of one block.
        const bool is_k = warp == 5;
        const CUtensorMap* map = is_k ? &tmap_k : &tmap_v;
        const uint32_t ring = sbase + (is_k ? TCN_OFF_K : TCN_OFF_V);
        const uint32_t full0 = is_k ? bar_kfull0 : bar_vfull0, empty0 = is_k ? bar_kempty0 : bar_vempty0;
        const uint32_t nst = is_k ? TCN_KST : TCN_VST;
        for (uint32_t k = 0;; ++k) {
            const int slot = k & 1;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(bar_ufull0 + 8 * slot, (k >> 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) s_abort = 1;
            if (__any_sync(0xffffffffu, !ok || !s_unit[slot][6] || s_abort)) break;  // warp-uniform
            const int t0u = s_unit[slot][2], t1u = s_unit[slot][3], head = s_unit[slot][5];
            const int32_t* tab = table_row(c, layer, s_unit[slot][7]);
            const int blk0 = t0u / 16, nblk = (t1u + 15) / 16 - blk0;
            const int ntiles = (nblk + 7) / 8;
            int next = (lane < 8 && lane < nblk) ? checked_block(c, tab[blk0 + lane]) : 0;
            for (int i = 0; i < ntiles; ++i) {
                const int blk = next;
                const int nb = min(8, nblk - 8 * i);
                if (i + 1 < ntiles)
                    next = (lane < 8 && 8 * (i + 1) + lane < nblk) ? checked_block(c, tab[blk0 + 8 * (i + 1) + lane]) : 0;
                const uint32_t gi = issued, stage = gi % nst;
                const uint32_t bar = full0 + 8 * stage;
                if (lane == 0) {
                    if (gi >= nst && !mbar_wait(empty0 + 8 * stage, ((gi / nst) - 1) & 1)) ok = 0;
                    if (ok) mbar_expect_tx(bar, (uint32_t)(nb * HALVES * 2048));
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    s_abort = 1;
                    break;
                }
                if (lane < nb) {
#pragma unroll
                    for (int h2 = 0; h2 < HALVES; ++h2) {
                        const uint32_t off = stage * TCN_KV_STAGE + h2 * (TCN_TILE * 128) + lane * 2048;
                        tma_load_3d(ring + off, map, bar, h2 * 64, head, blk * 16);
                    }
                }
                ++issued;
            }
            if (__any_sync(0xffffffffu, s_abort)) break;
        }
    } else {
        // Consumers: warps 0-3 softmax (thread = token = TMEM lane), warp 4
        // lane 0 issues the MMAs.
        uint32_t g0 = 0;  // tiles processed before the current unit
        for (uint32_t k = 0;; ++k) {
            const int slot = k & 1;
            const int got = mbar_wait(bar_ufull0 + 8 * slot, (k >> 1) & 1);
            // uniform decision across the 160 consumer threads
            if (bar_sync_or(160, !got || !s_unit[slot][6] || s_abort)) {
                if (!got) s_abort = 1;
                break;
            }
            TCN_TRACE(0);
#ifdef MENTAT_TC_TRACE
            if (blockIdx.x == 0 && tid == 0 && k < 64) g_tc_trace[3072 + 4 * k] = clock64();
#endif
            const int* su = s_unit[slot];
            const int q_lo = su[0], q_hi = su[1], t0u = su[2], t1u = su[3], ord = su[4], head = su[5];
            const int R = (q_hi - q_lo + 1) * G;
            const int blk0 = t0u / 16, nblk = (t1u + 15) / 16 - blk0;
            const int ntiles = (nblk + 7) / 8;
            const uint32_t qbase = sbase + TCN_OFF_Q + slot * TCN_Q_BYTES;
            if (tid < TCN_ROWS) s_mref[tid] = -INFINITY;  // warp 0; read by others only after the vote barriers

            auto issue_qk = [&](int i) {  // leader: S^T[(g0+i)%2] = K(i) Q^T
                const uint32_t g = g0 + i, stage = g % TCN_KST;
                if (!mbar_wait(bar_kfull0 + 8 * stage, (g / TCN_KST) & 1)) {
                    s_abort = 1;
                    return;
                }
                tc_fence_after();
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t ka = sbase + TCN_OFF_K + stage * TCN_KV_STAGE + (ks >> 2) * (TCN_TILE * 128) + (ks & 3) * 32;
                    const uint32_t qb = qbase + (ks >> 2) * (TCN_ROWS * 128) + (ks & 3) * 32;
                    umma_f16(tmem + 32 + 32 * (g & 1), sdesc_sw128(ka, 16, 1024), sdesc_sw128(qb, 16, 1024), IDESC_QK,
                             ks > 0);
                }
                umma_commit(bar_s0 + 8 * (g & 1));
                umma_commit(bar_kempty0 + 8 * stage);  // the K stage is free once this Q K^T has run
            };
            if (leader) issue_qk(0);
            // The softmax side only touches the first NR rows (R rounded up to 8).
            int aborted = 0;
            auto run_tiles = [&](auto nr_const) {
                constexpr int NR = decltype(nr_const)::value;
                float l_acc[NR];  // this thread's (token's) share of each row's sum
                float mref[NR];   // copy of s_mref
    #pragma unroll
                for (int r = 0; r < NR; ++r) {
                    l_acc[r] = 0.f;
                    mref[r] = -INFINITY;
                }
                for (int i = 0; i < ntiles && warp < 5; ++i) {
                    const uint32_t g = g0 + i;
                    TCN_TRACE(8 + 8 * i);
                    if (leader && !s_abort && i + 1 < ntiles) issue_qk(i + 1);
                    TCN_TRACE(9 + 8 * i);
                    if (softmax) {
                        if (!mbar_wait(bar_s0 + 8 * (g & 1), (g >> 1) & 1)) s_abort = 1;
                        tc_fence_after();
                        TCN_TRACE(10 + 8 * i);
#ifdef MENTAT_TC_TRACE
                        if (blockIdx.x == 0 && tid == 0 && i == 0 && k < 64) g_tc_trace[3072 + 4 * k + 1] = clock64();
#endif
                        float sv[NR];
                        tmem_ld_n<NR>(tmem + lane_off + 32 + 32 * (g & 1), sv);
                        const int t = (blk0 + 8 * i) * 16 + tid;  // this thread's token
                        const bool valid = t >= t0u && t < t1u;
                        int raise = 0;
    #pragma unroll
                        for (int r = 0; r < NR; ++r) {
                            sv[r] = valid ? sv[r] * scale_log2 : -INFINITY;
                            raise |= (r < R) && (sv[r] > mref[r] + 8.f);
                        }
                        // rare path: some row needs a (new) reference max
                        if (bar_sync_or_id(2, 128, raise)) {
                            float a[32];
    #pragma unroll
                            for (int r = 0; r < 32; ++r) a[r] = r < NR ? sv[r] : -INFINITY;
                            const float wmax = transpose_reduce32<true>(a);
                            s_red[warp][lane] = wmax;
                            bar_sync_id(2, 128);
                            if (warp == 0) {
                                const float tmax = fmaxf(fmaxf(s_red[0][lane], s_red[1][lane]), fmaxf(s_red[2][lane], s_red[3][lane]));
                                const float mo = s_mref[lane];
                                float f = 1.f;
                                if (lane < R && (mo == -INFINITY || tmax > mo + 8.f)) {
                                    f = mo == -INFINITY ? 0.f : ex2_approx(mo - tmax);
                                    s_mref[lane] = tmax;
                                }
                                s_fac[lane] = f;
                            }
                            bar_sync_id(2, 128);
                            bool any = false;
                            float fac[NR];
    #pragma unroll
                            for (int r = 0; r < NR; ++r) {
                                fac[r] = s_fac[r];
                                mref[r] = s_mref[r];
                                l_acc[r] *= fac[r];
                                any |= fac[r] != 1.f;
                            }
                            // O^T columns of raised rows, once P V(i-1) is done
                            if (i > 0 && any) {
                                const uint32_t gp = g - 1;
                                if (!mbar_wait(bar_pv0 + 8 * (gp & 1), (gp >> 1) & 1)) s_abort = 1;
                                tc_fence_after();
    #pragma unroll
                                for (int c8 = 0; c8 < NR; c8 += 8) {
                                    float ov[8];
                                    tmem_ld8(tmem + lane_off + c8, ov);
    #pragma unroll
                                    for (int r = 0; r < 8; ++r) ov[r] *= fac[c8 + r];
                                    tmem_st8(tmem + lane_off + c8, ov);
                                }
                            }
                        }
                        TCN_TRACE(11 + 8 * i);
                        // P^T row of this token: NR probabilities, rounded to T; rows >= R are 0
                        uint32_t pk[NR / 2];
    #pragma unroll
                        for (int j = 0; j < NR / 2; ++j) {
                            const float p0 = 2 * j < R ? ex2_approx(sv[2 * j] - mref[2 * j]) : 0.f;
                            const float p1 = 2 * j + 1 < R ? ex2_approx(sv[2 * j + 1] - mref[2 * j + 1]) : 0.f;
                            pk[j] = Pair<T>::pack(p0, p1);
                            l_acc[2 * j] += Pair<T>::lo(pk[j]);
                            l_acc[2 * j + 1] += Pair<T>::hi(pk[j]);
                        }
                        // P buffer (g%2) was last read by P V(i-2)
                        if (i >= 2) {
                            const uint32_t gp = g - 2;
                            if (!mbar_wait(bar_pv0 + 8 * (gp & 1), (gp >> 1) & 1)) s_abort = 1;
                        }
                        // MN-major, 64-byte swizzle: token row tid holds rows 0-31 in four 16-byte chunks
                        uint8_t* prow = smem + TCN_OFF_P + (g & 1) * TCN_P_BYTES + (tid >> 3) * 512 + (tid & 7) * 64;
                        const int sw = (tid & 7) >> 1;
    #pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            uint4 v = make_uint4(0, 0, 0, 0);
                            if (8 * c < NR) v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                            *reinterpret_cast<uint4*>(prow + ((c ^ sw) << 4)) = v;
                        }
                        TCN_TRACE(13 + 8 * i);
                    }
                    tc_fence_before();
                    fence_proxy_async();
                    aborted = bar_sync_or(160, s_abort);  // P(i) stored: softmax warps + issuer warp
                    TCN_TRACE(14 + 8 * i);
                    if (aborted) break;
                    if (leader) {  // O^T += V(i)^T P(i)^T
                        const uint32_t stage = g % TCN_VST;
                        if (!mbar_wait(bar_vfull0 + 8 * stage, (g / TCN_VST) & 1)) {
                            s_abort = 1;  // no P V: the softmax warps' next waits give up too
                        } else {
                            tc_fence_after();
                            for (int ks = 0; ks < TCN_TILE / 16; ++ks) {
                                const uint32_t va = sbase + TCN_OFF_V + stage * TCN_KV_STAGE + ks * 2048;
                                const uint32_t pb = sbase + TCN_OFF_P + (g & 1) * TCN_P_BYTES + ks * 1024;
                                umma_f16(tmem, sdesc_sw128(va, TCN_TILE * 128, 1024), sdesc(pb, TCN_P_BYTES, 512, 4),
                                         IDESC_PV, (i > 0 || ks > 0));
                            }
                            umma_commit(bar_pv0 + 8 * (g & 1));
                            umma_commit(bar_vempty0 + 8 * stage);
                        }
                    }
                    TCN_TRACE(15 + 8 * i);
                }
                if (bar_sync_or(160, aborted || s_abort)) {
                    aborted = 1;
                    return;
                }
                // row sums, then the partials (thread t = output element d of every row)
                if (softmax) {
                    float a[32];
    #pragma unroll
                    for (int r = 0; r < 32; ++r) a[r] = r < NR ? l_acc[r] : 0.f;
                    s_red[warp][lane] = transpose_reduce32<false>(a);
                    const uint32_t gl = g0 + ntiles - 1;
                    if (!mbar_wait(bar_pv0 + 8 * (gl & 1), (gl >> 1) & 1)) s_abort = 1;
                    tc_fence_after();
                    float ov[NR];
                    tmem_ld_n<NR>(tmem + lane_off, ov);  // row d = tid of O^T
                    if (tid < D) {
    #pragma unroll
                        for (int r = 0; r < NR; ++r) {
                            if (r < R) {
                                const int seq = q_lo + r / G, hq = head * G + r % G;
                                const int64_t pi = ((int64_t)seq * max_parts + ord) * Hq + hq;
                                ws.part_o[pi * D + tid] = ov[r];
                            }
                        }
                    }
                }
            };
            if (R <= 8) run_tiles(std::integral_constant<int, 8>{});
            else if (R <= 16) run_tiles(std::integral_constant<int, 16>{});
            else run_tiles(std::integral_constant<int, 32>{});
            if (aborted) {
                s_abort = 1;
                break;
            }
            // all four softmax warps' row sums are in s_red
            if (softmax) bar_sync_id(3, 128);
            if (tid < R) {
                const int seq = q_lo + tid / G, hq = head * G + tid % G;
                const int64_t pi = ((int64_t)seq * max_parts + ord) * Hq + hq;
                ws.part_ml[pi * 2] = s_mref[tid];
                ws.part_ml[pi * 2 + 1] = (s_red[0][tid] + s_red[1][tid]) + (s_red[2][tid] + s_red[3][tid]);
            }
            TCN_TRACE(4);
#ifdef MENTAT_TC_TRACE
            g_trace_on = false;
            if (blockIdx.x == 0 && tid == 0 && k < 64) {
                g_tc_trace[3072 + 4 * k + 2] = clock64();
                g_tc_trace[3072 + 4 * k + 3] = ntiles;
            }
#endif
            g0 += ntiles;
            // unit done: O^T, S^T and the slot's Q may be reused
            tc_fence_before();
            bar_sync_or(160, 0);
            tc_fence_after();
            if (tid == 0) mbar_arrive(bar_uempty0 + 8 * slot);
        }
    }
    __syncthreads();
    if (s_abort) {
        if (tid == 0) atomicExch(&ws.hdr[HDR_TC_ABORT], 1);
        if ((warp == 5 || warp == 7) && lane == 0) {  // every lane of a TMA warp counted the same tiles
            const uint32_t nst = warp == 5 ? TCN_KST : TCN_VST;
            for (uint32_t k = issued > nst ? issued - nst : 0; k < issued; ++k)
                (void)mbar_wait((warp == 5 ? bar_kfull0 : bar_vfull0) + 8 * (k % nst), (k / nst) & 1);
        }
        __syncthreads();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TCN_TMEM_COLS);
    TL_LAST(7);
    TL_CTA_END(1);
    griddep_wait();  // complete only after the wide kernel: the merge reads both kernels' partials
}

}  // namespace mentat
