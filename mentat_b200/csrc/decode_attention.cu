// Tree-aware paged GQA decode attention (replaces build_packed_kv + attn_decode
// of the reference: core/paged_kv_cache.py:289-368, adapters/attention_backend.py:192-228).
//
// Three stream-ordered launches:
//   1. k_plan    (1 CTA)  - reads the batch's block tables, finds the token
//      prefixes that adjacent sequences share (longest common block prefix),
//      builds the LCP-interval tree of the batch and cuts every node of it
//      (a token range shared by a contiguous run of sequences) into units of
//      <= CHUNK tokens x <= 16 query rows.  Each unit gets a partial-result
//      ordinal that is unique along every sequence's root-to-leaf path.
//   2. k_units   (persistent CTAs, dynamic unit queue) - one unit x one kv
//      head per work item: stream the unit's K/V tiles once, compute scores
//      for all its query rows (GQA group x sharing sequences), online
//      softmax in base 2, and write the unnormalised partial (m, l, o).
//   3. k_merge   - log-sum-exp merge of each (sequence, q head)'s partials.
// A shared prefix is therefore read once per unit instead of once per branch,
// and the packed KV of the reference is never materialised.

#include "common.cuh"

#ifdef MENTAT_TC_TRACE
__device__ long long g_plan_trace[16];
#define PLAN_TRACE(k) do { if (threadIdx.x == 0) g_plan_trace[(k)] = clock64(); } while (0)
#else
#define PLAN_TRACE(k) do { } while (0)
#endif

#include <climits>
#include <cstdlib>
#include <type_traits>

namespace mentat {

// cycles of the test hook's wait in every tensor-core unit CTA (0: off); set by
// mentat_decode_set_wait_probe
__device__ long long g_decode_wait_probe = 0;

constexpr int PLAN_HDR = 64;        // header ints, see HDR_*
constexpr int HDR_NSIMT = 0, HDR_SIMT_NEXT = 1, HDR_ERR = 2, HDR_NTC = 3, HDR_TC_NEXT = 4, HDR_TC_ABORT = 5,
              HDR_NTCN = 6, HDR_TCN_NEXT = 7;
// what the plan was made for, checked by a call that reuses it: n, max_parts,
// the GQA group, and the routing (tensor-core kernels on, narrow kernel on,
// row threshold)
constexpr int HDR_PLAN_N = 8, HDR_PLAN_PARTS = 9, HDR_PLAN_G = 10, HDR_PLAN_ROUTE = 11;
// wide tensor-core CTAs that take units in a decode call (the others leave their
// SMs to the narrow kernel at once), chosen by the plan
constexpr int HDR_TC_CTAS = 12;
constexpr int KIND_FFMA = 0, KIND_TC = 1, KIND_TCN = 2, NKINDS = 3;
constexpr int UNIT_INTS = 8;        // seq_lo, seq_hi, tok0, tok1, ordinal
constexpr int CHUNK = 256;          // tokens per FFMA unit
constexpr int CHUNK_TC = 2048;      // tokens per tensor-core unit
constexpr int MAX_ROWS = 16;        // query rows per unit on the FFMA path
constexpr int TC_MAX_ROWS = 256;    // query rows per unit on the wide tensor-core path (two M=128 tiles)
constexpr int TCN_MAX_ROWS = 32;    // query rows per unit on the narrow (transposed) tensor-core path
constexpr int PLAN_MAX_SEQS = 1024;  // sequences per launch (callers split larger batches)
// the plan's shared memory (dynamic, sized by n): 22 n + 2 ints, see k_plan
__host__ __device__ inline int plan_smem_bytes(int n) { return (22 * n + 2) * 4; }

struct DecodeWs {
    int32_t* hdr;
    int32_t* nparts;  // [n]
    int32_t* lcp;     // [n] first differing block of pair (i-1, i), filled by k_lcp
    int32_t* units;   // [n * max_parts][UNIT_INTS]  FFMA units
    int32_t* units_tc;  // [n * max_parts][UNIT_INTS]  wide tensor-core units
    int32_t* units_tcn; // [n * max_parts][UNIT_INTS]  narrow tensor-core units
    float* part_ml;   // [n][max_parts][Hq][2]
    float* part_o;    // [n][max_parts][Hq][D]
};

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline void ws_carve(void* base, int n, int hq, int d, int max_parts, DecodeWs* w,
                                         int64_t* total) {
    int64_t off = 0;
    char* b = reinterpret_cast<char*>(base);
    auto take = [&](int64_t bytes) {
        char* p = b ? b + off : nullptr;
        off = align_up(off + bytes, 256);
        return p;
    };
    w->hdr = reinterpret_cast<int32_t*>(take(PLAN_HDR * 4));
    w->nparts = reinterpret_cast<int32_t*>(take((int64_t)n * 4));
    w->lcp = reinterpret_cast<int32_t*>(take((int64_t)n * 4));
    w->units = reinterpret_cast<int32_t*>(take((int64_t)n * max_parts * UNIT_INTS * 4));
    w->units_tc = reinterpret_cast<int32_t*>(take((int64_t)n * max_parts * UNIT_INTS * 4));
    w->units_tcn = reinterpret_cast<int32_t*>(take((int64_t)n * max_parts * UNIT_INTS * 4));
    w->part_ml = reinterpret_cast<float*>(take((int64_t)n * max_parts * hq * 2 * 4));
    w->part_o = reinterpret_cast<float*>(take((int64_t)n * max_parts * hq * d * 4));
    *total = off;
}

// ---------------------------------------------------------------------------
// 0. first differing table entry of each adjacent pair: one block per pair
//    walks the two table rows LCP_CHUNK entries at a time and writes the first
//    differing block index (INT_MAX: none) to ws.lcp
// ---------------------------------------------------------------------------
constexpr int LCP_THREADS = 256;
constexpr int LCP_CHUNK = LCP_THREADS * 16;
__global__ void __launch_bounds__(LCP_THREADS) k_lcp(mentat_kv_cache c, int layer, const int32_t* slots, int n,
                                                     DecodeWs ws) {
    __shared__ int s_min[LCP_THREADS / 32];
    griddep_wait();  // tables and lengths may come from the previous launch on the stream
    griddep_launch();
    TL_FIRST(0);
    const int pair = blockIdx.x + 1;  // compares sequences pair-1 and pair
    if (pair >= n) return;
    int sa = slots[pair - 1], sb = slots[pair];
    if (sa < 0 || sa >= c.max_seqs) sa = 0;
    if (sb < 0 || sb >= c.max_seqs) sb = 0;
    if (sa == sb) return;  // the plan does not read this pair
    const int bs = c.block_size;
    const int la = c.ntok[seq_index(c, layer, sa)], lb = c.ntok[seq_index(c, layer, sb)];
    const int m = min((la + bs - 1) / bs, (lb + bs - 1) / bs);
    const int32_t* ta = table_row(c, layer, sa);
    const int32_t* tb = table_row(c, layer, sb);
    // 16-byte loads only when every row is 16-byte aligned, so a load never crosses a row end
    const bool vec = (c.max_blocks_per_seq & 3) == 0 && ((((uintptr_t)ta) | ((uintptr_t)tb)) & 15) == 0;
    int first = INT_MAX;
    // chunks in order; the first chunk with a difference holds the answer
    for (int j0 = 0; j0 < m && first == INT_MAX; j0 += LCP_CHUNK) {
        int f = INT_MAX;
        if (vec) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + (u * LCP_THREADS + threadIdx.x) * 4;
                if (j < m) {
                    const int4 a = *reinterpret_cast<const int4*>(ta + j);
                    const int4 b = *reinterpret_cast<const int4*>(tb + j);
                    if (a.x != b.x) f = min(f, j);
                    else if (a.y != b.y && j + 1 < m) f = min(f, j + 1);
                    else if (a.z != b.z && j + 2 < m) f = min(f, j + 2);
                    else if (a.w != b.w && j + 3 < m) f = min(f, j + 3);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int j = j0 + u * LCP_THREADS + threadIdx.x;
                if (j < m && ta[j] != tb[j]) f = min(f, j);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, o));
        if ((threadIdx.x & 31) == 0) s_min[threadIdx.x >> 5] = f;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < LCP_THREADS / 32; ++w) first = min(first, s_min[w]);
        __syncthreads();
    }
    if (threadIdx.x == 0) ws.lcp[pair] = first;
    TL_LAST(1);
}

// Plan parameters for one launch.  A segment (node of the LCP-interval tree or
// a sequence's own leaf range) with rows = width x G goes to
//   the narrow tensor-core kernel when narrow_ok and rows <= 32,
//   the wide tensor-core kernel when tc_ok and rows >= tc_min_rows,
//   the FFMA kernel otherwise.
struct PlanParams {
    int G;
    int tc_ok;        // dtype / head_dim / block size fit the wide tensor-core kernel
    int narrow_ok;    // ... and the narrow one
    int tc_min_rows;  // rows threshold for the tensor-core kernels
    int sms;          // SMs of the device
    int tc_ctas;      // wide tensor-core CTAs that take units (0: the plan chooses)
};

constexpr int LPT_BUCKETS = CHUNK_TC / 128;  // tensor-core units by 128-token tile count

__host__ __device__ inline int plan_route(const PlanParams& pp) {
    return pp.tc_ok | (pp.narrow_ok << 1) | (pp.tc_min_rows << 2);
}

__device__ __forceinline__ int seg_kind(const PlanParams& pp, int width) {
    const int rows = width * pp.G;
    if (!pp.tc_ok || rows < pp.tc_min_rows) return KIND_FFMA;
    if (pp.narrow_ok && rows <= TCN_MAX_ROWS) return KIND_TCN;
    return KIND_TC;
}
__device__ __forceinline__ int seg_chunk(int kind) { return kind == KIND_FFMA ? CHUNK : CHUNK_TC; }
__device__ __forceinline__ int seg_spu(const PlanParams& pp, int kind) {
    const int rows = kind == KIND_FFMA ? MAX_ROWS : (kind == KIND_TC ? TC_MAX_ROWS : TCN_MAX_ROWS);
    return max(1, rows / pp.G);
}

// Wide tensor-core CTAs for a decode call, evaluated by one warp.  The wide
// units are compute bound: about 1.55 us per 128-token tile and 128-row tile
// on one SM (B200, head_dim 128; in proportion to head_dim).  The narrow units
// stream at the HBM rate the pair of kernels reaches together, about 5.9 TB/s
// of K/V tiles on B200.  The call is then shortest when the wide kernel's
// compute spans the whole stream: lane k - 1 estimates the wide phase with k
// items per CTA in turn (w = ceil(items / k) CTAs, the phase lasting about
// max(cost / w, longest item)), and the most waves whose phase still ends
// within the time both queues' bytes take at that rate win.  When even one
// wave outlasts the bytes (wide work alone, or little narrow work), every SM
// the wide items can use takes one.
__device__ inline int tc_ctas_warp(int items, float wcost, float wmax, float wtiles, float ntiles, int sms,
                                   int head_dim, int lane) {
    if (items <= 0) return sms;
    const float a_w = 1.55f * head_dim * (1.f / 128.f);                  // us per tile and row tile
    const float tiles_per_us = 5.9e6f / (512.f * (float)head_dim);        // 128 tokens x K, V x 2 B
    const float t_bytes = (wtiles + ntiles) / tiles_per_us;
    const int k = lane + 1;
    const int w = min((items + k - 1) / k, sms);
    const float tw = a_w * fmaxf(__fdividef(wcost, (float)w), wmax);
    const unsigned fit = __ballot_sync(0xffffffffu, lane < 8 && tw <= 1.05f * t_bytes);
    const int best = fit ? __shfl_sync(0xffffffffu, w, 31 - __clz(fit)) : min(items, sms);
    return max(1, best);
}

__global__ void __launch_bounds__(1024)
k_plan(mentat_kv_cache c, int layer, const int32_t* slots, int n, PlanParams pp, DecodeWs ws, int max_parts) {
    // per-sequence, per-boundary and per-node arrays in dynamic shared memory
    // (plan_smem_bytes(n)); nodes and boundaries number at most n - 1
    extern __shared__ int plan_smem[];
    int* s_len = plan_smem;             // [n]
    int* s_slot = s_len + n;            // [n]
    int* s_h = s_slot + n;              // [n + 1] h[i] = LCP(i-1, i) in tokens, h[0] = h[n] = 0
    int* s_top = s_h + n + 1;           // [n + 1] deepest node covering i-1, i after boundary i
    int* s_nlo = s_top + n + 1;         // [n] node intervals, depths and parents
    int* s_nhi = s_nlo + n;
    int* s_ndep = s_nhi + n;
    int* s_npar = s_ndep + n;
    int* s_nid = s_npar + n;            // [n] node id of a representative boundary
    int* s_brep = s_nid + n;            // [n] per boundary
    int* s_blo = s_brep + n;
    int* s_bhi = s_blo + n;
    int* s_nbase = s_bhi + n;           // [n]
    int* s_nchunk = s_nbase + n;        // [n]
    int* s_seg_units = s_nchunk + n;    // [2n] internal nodes, then leaves
    int* s_seg_first = s_seg_units + 2 * n;  // [NKINDS][2n] first unit of each segment in its kind's queue
    __shared__ int smem32[32];
    __shared__ int s_bcnt[LPT_BUCKETS];
    __shared__ long long s_scan64[32];
    __shared__ unsigned s_ktot[NKINDS];  // saturating: each term is clamped to FIELD
    __shared__ int s_nnodes, s_err;
    __shared__ unsigned s_wcost, s_wmax, s_wtiles, s_ntiles;  // work of the tensor-core queues, see tc_ctas_warp
    const int tid = threadIdx.x;
    const int bs = c.block_size;
    // With the LCP kernel ahead of this one (n > 1), the slots and lengths were
    // final when that kernel passed its own wait, so they are read while it runs;
    // otherwise they may come from the previous launch and are read after the wait.
    if (n <= 1) griddep_wait();
    for (int i = tid; i < n; i += blockDim.x) {
        int slot = slots[i];
        if (slot < 0 || slot >= c.max_seqs) slot = 0;
        s_slot[i] = slot;
        s_len[i] = c.ntok[seq_index(c, layer, slot)];
    }
    if (n > 1) griddep_wait();  // the pair LCPs
    griddep_launch();
    TL_FIRST(2);
    PLAN_TRACE(0);
    if (tid == 0) {
        s_h[0] = 0;
        s_h[n] = 0;
        s_err = 0;
        s_wcost = s_wmax = s_wtiles = s_ntiles = 0;
    }
    __syncthreads();

    PLAN_TRACE(1);
    // LCP of adjacent sequences, in tokens, from k_lcp's first differing block
    for (int i = 1 + tid; i < n; i += blockDim.x) {
        const int la = s_len[i - 1], lb = s_len[i];
        const int m = min((la + bs - 1) / bs, (lb + bs - 1) / bs);
        const int first = s_slot[i - 1] == s_slot[i] ? m : min(m, ws.lcp[i]);
        s_h[i] = min(min(first * bs, la), lb);
    }
    __syncthreads();
    PLAN_TRACE(2);
    // LCP-interval tree, one thread per boundary b (between sequences b-1 and
    // b).  A boundary of depth d = h[b] > 0 belongs to the node of depth d
    // whose interval is the maximal run of boundaries with h >= d around b;
    // the node's representative is the run's leftmost boundary of depth
    // exactly d, and node ids number the representatives left to right (the
    // order in which a left-to-right stack walk would push them).
    {
        // one warp per boundary: search 32 boundaries per step with ballots
        const int warp = tid >> 5, lane = tid & 31;
        const int nwarps = blockDim.x >> 5;
        for (int b = 1 + warp; b < n; b += nwarps) {
            const int d = s_h[b];
            int rep = 0, lo = 0, hi = 0;
            if (d > 0) {
                rep = b;
                // nearest boundary j < b with h[j] < d (0 stands for "none"); the
                // leftmost boundary of depth d after it is the representative
                for (int base = b - 1;; base -= 32) {
                    const int j = base - lane;
                    const int hj = j >= 1 ? s_h[j] : 0;
                    const unsigned less = __ballot_sync(0xffffffffu, j < 1 || hj < d);
                    unsigned eq = __ballot_sync(0xffffffffu, j >= 1 && hj == d);
                    if (less) eq &= (1u << (__ffs(less) - 1)) - 1u;
                    if (eq) rep = base - (31 - __clz(eq));
                    if (less) {
                        lo = max(0, base - (__ffs(less) - 1));
                        break;
                    }
                }
                if (rep == b) {
                    hi = n - 1;
                    for (int base = b + 1; base <= n - 1; base += 32) {
                        const int k = base + lane;
                        const unsigned less = __ballot_sync(0xffffffffu, k > n - 1 || s_h[min(k, n)] < d);
                        if (less) {
                            hi = base + (__ffs(less) - 1) - 1;
                            break;
                        }
                    }
                }
            }
            if (lane == 0) {
                s_brep[b] = rep;
                s_blo[b] = lo;
                s_bhi[b] = hi;
            }
        }
        __syncthreads();
        const int bnd = tid + 1;
        const int rep = bnd < n ? s_brep[bnd] : 0;
        const int lo = bnd < n ? s_blo[bnd] : 0, hi = bnd < n ? s_bhi[bnd] : 0;
        int nnodes;
        const bool is_rep = rep != 0 && rep == bnd;
        const int id = block_exclusive_scan(is_rep ? 1 : 0, &nnodes, smem32);
        if (is_rep) {
            s_nid[bnd] = id;
            s_nlo[id] = lo;
            s_nhi[id] = hi;
            s_ndep[id] = s_h[bnd];
        }
        __syncthreads();
        // deepest node covering sequences b-1 and b
        if (bnd < n) s_top[bnd] = rep ? s_nid[rep] : -1;
        if (tid == 0) {
            s_top[0] = -1;
            s_top[n] = -1;
            s_nnodes = nnodes;
        }
        __syncthreads();
        // parent: the node of the deeper of the two boundaries bounding the interval
        for (int x = tid; x < nnodes; x += blockDim.x) {
            const int xl = s_nlo[x], xh = s_nhi[x];
            const int hl = xl >= 1 ? s_h[xl] : 0, hr = xh + 1 <= n - 1 ? s_h[xh + 1] : 0;
            s_npar[x] = (hl == 0 && hr == 0) ? -1 : (hl >= hr ? s_top[xl] : s_top[xh + 1]);
        }
        __syncthreads();
        for (int x = tid; x < nnodes; x += blockDim.x) {
            const int p = s_npar[x];
            const int pdep = p >= 0 ? s_ndep[p] : 0;
            const int ch = seg_chunk(seg_kind(pp, s_nhi[x] - s_nlo[x] + 1));
            s_nchunk[x] = (s_ndep[x] - pdep + ch - 1) / ch;
        }
        __syncthreads();
        // partial ordinals: a node's chunks follow those of all its ancestors
        for (int x = tid; x < nnodes; x += blockDim.x) {
            int base = 0;
            for (int p = s_npar[x]; p >= 0; p = s_npar[p]) base += s_nchunk[p];
            s_nbase[x] = base;
        }
        __syncthreads();
    }
    PLAN_TRACE(3);
    const int nn = s_nnodes;
    const int nseg = nn + n;
    const int leaf_kind = seg_kind(pp, 1);
    for (int s = tid; s < nseg; s += blockDim.x) {
        int cnt;
        if (s < nn) {
            const int width = s_nhi[s] - s_nlo[s] + 1;
            const int spu = seg_spu(pp, seg_kind(pp, width));
            cnt = s_nchunk[s] * ((width + spu - 1) / spu);
        } else {
            const int i = s - nn;
            const int a = s_top[i], b = s_top[i + 1];
            const int da = a >= 0 ? s_ndep[a] : 0, db = b >= 0 ? s_ndep[b] : 0;
            const int node = da >= db ? a : b;
            const int d0 = node >= 0 ? s_ndep[node] : 0;
            const int base = node >= 0 ? s_nbase[node] + s_nchunk[node] : 0;
            const int chunk = seg_chunk(leaf_kind);
            const int ch = (s_len[i] - d0 + chunk - 1) / chunk;
            cnt = ch;
            ws.nparts[i] = base + ch;
            if (base + ch > max_parts) atomicExch(&s_err, 1);
        }
        s_seg_units[s] = cnt;
    }
    __syncthreads();
    PLAN_TRACE(4);
    // exclusive scans of the unit counts per kernel kind, packed 21 bits per
    // kind into one 64-bit scan (a count that does not fit is a plan overflow)
    const int s0 = 2 * tid, s1 = 2 * tid + 1;
    auto kind_of = [&](int s) { return s < nn ? seg_kind(pp, s_nhi[s] - s_nlo[s] + 1) : leaf_kind; };
    constexpr long long FIELD = 1ll << 21;
    if (tid < NKINDS) s_ktot[tid] = 0;
    __syncthreads();
    {
        const int k0 = s0 < nseg ? kind_of(s0) : -1, k1 = s1 < nseg ? kind_of(s1) : -1;
        const unsigned c0 = k0 >= 0 ? (unsigned)min((long long)s_seg_units[s0], FIELD) : 0u;
        const unsigned c1 = k1 >= 0 ? (unsigned)min((long long)s_seg_units[s1], FIELD) : 0u;
#pragma unroll
        for (int kind = 0; kind < NKINDS; ++kind) {
            const unsigned r = __reduce_add_sync(0xffffffffu, (k0 == kind ? c0 : 0u) + (k1 == kind ? c1 : 0u));
            if ((tid & 31) == 0 && r) atomicAdd(&s_ktot[kind], r);
        }
    }
    __syncthreads();
    const bool fits = s_ktot[0] < FIELD && s_ktot[1] < FIELD && s_ktot[2] < FIELD;  // no field can carry
    if (!fits && tid == 0) s_err = 1;
    auto packed = [&](int s) -> long long {
        if (s >= nseg || !fits) return 0;
        return (long long)s_seg_units[s] << (21 * kind_of(s));
    };
    const long long p0 = packed(s0), p1 = packed(s1);
    long long ptot;
    const long long pe = block_exclusive_scan64(p0 + p1, &ptot, s_scan64);
    int totals[NKINDS];
#pragma unroll
    for (int kind = 0; kind < NKINDS; ++kind) {
        const int sh = 21 * kind;
        totals[kind] = (int)((ptot >> sh) & (FIELD - 1));
        const int e = (int)((pe >> sh) & (FIELD - 1));
        if (s0 < nseg) s_seg_first[kind * 2 * n + s0] = e;
        if (s1 < nseg) s_seg_first[kind * 2 * n + s1] = e + (int)((p0 >> sh) & (FIELD - 1));
    }
    if (tid == 0) {
        for (int kind = 0; kind < NKINDS; ++kind)
            if ((int64_t)totals[kind] > (int64_t)n * max_parts) s_err = 1;
        ws.hdr[HDR_NSIMT] = s_err ? 0 : totals[KIND_FFMA];
        ws.hdr[HDR_SIMT_NEXT] = 0;
        ws.hdr[HDR_ERR] = s_err;
        ws.hdr[HDR_NTC] = s_err ? 0 : totals[KIND_TC];
        ws.hdr[HDR_TC_NEXT] = 0;
        ws.hdr[HDR_NTCN] = s_err ? 0 : totals[KIND_TCN];
        ws.hdr[HDR_TCN_NEXT] = 0;
        ws.hdr[HDR_TC_ABORT] = 0;
        ws.hdr[HDR_PLAN_N] = n;
        ws.hdr[HDR_PLAN_PARTS] = max_parts;
        ws.hdr[HDR_PLAN_G] = pp.G;
        ws.hdr[HDR_PLAN_ROUTE] = plan_route(pp);
        if (s_err) set_error(c, MENTAT_DEV_PLAN_OVERFLOW, totals[0] + totals[1] + totals[2]);
    }
    __syncthreads();
    PLAN_TRACE(5);
    if (s_err) return;
    // Unit records, written longest first within each tensor-core queue (a
    // counting sort on the tile count) so that the last units a persistent
    // CTA claims are the short ones.  Queue order does not change the result:
    // every unit writes its own (sequence, ordinal, head) partial.
    auto make_unit = [&](int kind, int u, int* rec) {
        const int* first = s_seg_first + kind * 2 * n;
        int lo = 0, hi = nseg - 1;  // last segment whose first unit <= u (zero-count segments precede it)
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (first[mid] <= u) lo = mid; else hi = mid - 1;
        }
        const int s = lo, k = u - first[s];
        if (s < nn) {
            const int width = s_nhi[s] - s_nlo[s] + 1;
            const int sk = seg_kind(pp, width);
            const int spu = seg_spu(pp, sk), chunk = seg_chunk(sk);
            const int ngroups = (width + spu - 1) / spu;
            const int ch = k / ngroups, rg = k % ngroups;
            const int p = s_npar[s];
            const int pdep = p >= 0 ? s_ndep[p] : 0;
            rec[0] = s_nlo[s] + rg * spu;
            rec[1] = min(s_nhi[s], rec[0] + spu - 1);
            rec[2] = pdep + ch * chunk;
            rec[3] = min(s_ndep[s], rec[2] + chunk);
            rec[4] = s_nbase[s] + ch;
        } else {
            const int i = s - nn;
            const int a = s_top[i], b = s_top[i + 1];
            const int da = a >= 0 ? s_ndep[a] : 0, db = b >= 0 ? s_ndep[b] : 0;
            const int node = da >= db ? a : b;
            const int d0 = node >= 0 ? s_ndep[node] : 0;
            const int base = node >= 0 ? s_nbase[node] + s_nchunk[node] : 0;
            const int chunk = seg_chunk(leaf_kind);
            rec[0] = rec[1] = i;
            rec[2] = d0 + k * chunk;
            rec[3] = min(s_len[i], rec[2] + chunk);
            rec[4] = base + k;
        }
    };
    auto bucket_of = [](const int* rec) { return min(LPT_BUCKETS - 1, (rec[3] - rec[2] - 1) / 128); };
    for (int kind = 0; kind < NKINDS; ++kind) {
        const int total = totals[kind];
        if (total == 0) continue;  // uniform across the block
        int32_t* units = kind == KIND_FFMA ? ws.units : (kind == KIND_TC ? ws.units_tc : ws.units_tcn);
        const bool lpt = kind != KIND_FFMA;
        const bool one_pass = total <= (int)blockDim.x;  // each thread keeps its record between the passes
        int mine[5];
        if (one_pass && tid < total) make_unit(kind, tid, mine);
        if (lpt) {
            if (tid < LPT_BUCKETS) s_bcnt[tid] = 0;
            __syncthreads();
            for (int u = tid; u < total; u += blockDim.x) {
                int rec[5];
                if (one_pass) {
#pragma unroll
                    for (int f = 0; f < 5; ++f) rec[f] = mine[f];
                } else {
                    make_unit(kind, u, rec);
                }
                atomicAdd(&s_bcnt[bucket_of(rec)], 1);
            }
            __syncthreads();
            if (tid == 0) {
                int run = 0;
                for (int b = LPT_BUCKETS - 1; b >= 0; --b) {
                    const int cnt = s_bcnt[b];
                    s_bcnt[b] = run;  // cursor: first position of bucket b
                    run += cnt;
                }
            }
            __syncthreads();
        }
        for (int u = tid; u < total; u += blockDim.x) {
            int rec[5];
            if (one_pass) {
#pragma unroll
                for (int f = 0; f < 5; ++f) rec[f] = mine[f];
            } else {
                make_unit(kind, u, rec);
            }
            const int dst = lpt ? atomicAdd(&s_bcnt[bucket_of(rec)], 1) : u;
            int32_t* U = units + (int64_t)dst * UNIT_INTS;
            U[0] = rec[0]; U[1] = rec[1]; U[2] = rec[2]; U[3] = rec[3]; U[4] = rec[4];
            if (lpt) {  // 128-token tiles of 16-token blocks, as the tensor-core kernels cut them
                const unsigned nt = (unsigned)(((rec[3] + 15) / 16 - rec[2] / 16 + 7) / 8);
                const unsigned cw = kind == KIND_TC ? nt * (unsigned)(((rec[1] - rec[0] + 1) * pp.G + 127) / 128) : nt;
                const unsigned m = __activemask();
                const unsigned sum = __reduce_add_sync(m, cw), mx = __reduce_max_sync(m, cw);
                const unsigned tiles = kind == KIND_TC ? __reduce_add_sync(m, nt) : 0u;
                if ((tid & 31) == __ffs(m) - 1) {
                    atomicAdd(kind == KIND_TC ? &s_wcost : &s_ntiles, sum);
                    if (kind == KIND_TC) {
                        atomicMax(&s_wmax, mx);
                        atomicAdd(&s_wtiles, tiles);
                    }
                }
            }
        }
        __syncthreads();
    }
    if (tid < 32) {
        const int w = pp.tc_ctas > 0 ? pp.tc_ctas
                                     : tc_ctas_warp(totals[KIND_TC] * c.num_kv_heads, (float)s_wcost * c.num_kv_heads,
                                                    (float)s_wmax, (float)s_wtiles * c.num_kv_heads,
                                                    (float)s_ntiles * c.num_kv_heads, pp.sms, c.head_dim, tid);
        if (tid == 0) ws.hdr[HDR_TC_CTAS] = w;
    }
    __syncthreads();
    PLAN_TRACE(6);
    TL_LAST(3);
}

// ---------------------------------------------------------------------------
// 1b. a call that reuses the plan in the workspace (another layer of the same
//     decode step): check that the plan was made for this call's shape and
//     routing, and restart the unit queues.  On a mismatch no unit runs, the
//     merge zeroes the output and the call reports MENTAT_DEV_PLAN_OVERFLOW.
// ---------------------------------------------------------------------------
__global__ void k_plan_reuse(mentat_kv_cache c, int n, int max_parts, int route, int G, DecodeWs ws) {
    griddep_wait();  // the previous call's merge has read the header
    if (threadIdx.x == 0) {
        const bool same = ws.hdr[HDR_PLAN_N] == n && ws.hdr[HDR_PLAN_PARTS] == max_parts &&
                          ws.hdr[HDR_PLAN_G] == G && ws.hdr[HDR_PLAN_ROUTE] == route && ws.hdr[HDR_ERR] == 0;
        if (!same) {
            ws.hdr[HDR_ERR] = 1;
            ws.hdr[HDR_NSIMT] = ws.hdr[HDR_NTC] = ws.hdr[HDR_NTCN] = 0;
            set_error(c, MENTAT_DEV_PLAN_OVERFLOW, -1);
        }
        ws.hdr[HDR_SIMT_NEXT] = ws.hdr[HDR_TC_NEXT] = ws.hdr[HDR_TCN_NEXT] = 0;
        ws.hdr[HDR_TC_ABORT] = 0;
    }
    griddep_launch();
}

// ---------------------------------------------------------------------------
// 1c. the plan of a causal prefill: n new queries of one sequence, query i at
//     position pos0 + i (its tokens 0 .. pos0 + i are cached).  Queries are cut
//     into row groups of spu positions (the unit kernel's rows / G) and each
//     group's visible tokens [0, pos0 + last position + 1) into chunks of
//     prefill_chunk(pos0 + n) tokens; a unit is (group, chunk), with the chunk
//     number as its partial ordinal.  Groups are written last to first, so the
//     longest units come first in the queue.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
k_prefill_plan(mentat_kv_cache c, int n, int pos0, int G, int kind, int chunk, DecodeWs ws, int max_parts) {
    __shared__ int smem32[32];
    __shared__ int s_err;
    griddep_wait();
    griddep_launch();
    const int tid = threadIdx.x;
    const int spu = max(1, (kind == KIND_TC ? TC_MAX_ROWS : MAX_ROWS) / G);
    const int ngroups = (n + spu - 1) / spu;
    int32_t* units = kind == KIND_TC ? ws.units_tc : ws.units;
    if (tid == 0) s_err = 0;
    int carry = 0;
    for (int g0 = 0; g0 < ngroups; g0 += blockDim.x) {
        const int k = g0 + tid;
        const int g = ngroups - 1 - k;  // last group first
        int cnt = 0, a = 0, b = 0;
        if (k < ngroups) {
            a = g * spu;
            b = min(n, a + spu);
            cnt = (pos0 + b + chunk - 1) / chunk;
            if (cnt > max_parts) atomicExch(&s_err, 1);
        }
        int tot;
        const int base = carry + block_exclusive_scan(cnt, &tot, smem32);
        if (k < ngroups && base + cnt <= n * max_parts) {
            for (int ch = 0; ch < cnt && ch < max_parts; ++ch) {
                int32_t* U = units + (int64_t)(base + ch) * UNIT_INTS;
                U[0] = a;
                U[1] = b - 1;
                U[2] = ch * chunk;
                U[3] = min((ch + 1) * chunk, pos0 + b);
                U[4] = ch;
            }
        }
        carry += tot;
    }
    // every query's part count, one thread per query: its group's chunk count
    for (int i = tid; i < n; i += blockDim.x) {
        const int b = min(n, (i / spu + 1) * spu);
        ws.nparts[i] = min((pos0 + b + chunk - 1) / chunk, max_parts);
    }
    __syncthreads();
    if (tid == 0) {
        const bool err = s_err || carry > n * max_parts;
        ws.hdr[HDR_NSIMT] = (!err && kind == KIND_FFMA) ? carry : 0;
        ws.hdr[HDR_NTC] = (!err && kind == KIND_TC) ? carry : 0;
        ws.hdr[HDR_NTCN] = 0;
        ws.hdr[HDR_SIMT_NEXT] = ws.hdr[HDR_TC_NEXT] = ws.hdr[HDR_TCN_NEXT] = 0;
        ws.hdr[HDR_TC_ABORT] = 0;
        ws.hdr[HDR_ERR] = err ? 1 : 0;
        ws.hdr[HDR_PLAN_N] = -1;  // not a decode plan: a reuse is refused
        if (err) set_error(c, MENTAT_DEV_PLAN_OVERFLOW, carry);
    }
}

// ---------------------------------------------------------------------------
// 2. units (FFMA path: any dtype, <= 16 query rows per unit)
// ---------------------------------------------------------------------------
constexpr int TT = 32;  // tokens per tile
// 16 warps: one query row each in the score stage, and D / 512 of the tile's
// tokens per thread in the P V stage; a unit's tiles take a quarter of the time
// they took on 128 threads, which matters when a few long units set the call's
// time (config 1: 80 work items)
constexpr int UNIT_THREADS = 512;

template <typename T, int D>
__global__ void __launch_bounds__(UNIT_THREADS)
k_units(mentat_kv_cache c, int layer, const int32_t* slots, const T* __restrict__ q, int64_t q_stride, int Hq,
        float qscale, DecodeWs ws, int max_parts, int causal_pos0) {
    constexpr int TS = UNIT_THREADS / D;  // token splits in the PV stage
    constexpr int KP = D + 1;             // padded K row (conflict-free column reads)
    // K and V tiles, and after a unit's last tile the token splits' partial sums
    constexpr int KV_FLOATS = TT * KP + TT * D, RED_FLOATS = TS * MAX_ROWS * D;
    __shared__ float q_s[MAX_ROWS][D];
    __shared__ __align__(16) float kv_red[KV_FLOATS > RED_FLOATS ? KV_FLOATS : RED_FLOATS];
    float(*k_s)[KP] = reinterpret_cast<float(*)[KP]>(kv_red);
    float(*v_s)[D] = reinterpret_cast<float(*)[D]>(kv_red + TT * KP);
    float(*red_s)[MAX_ROWS][D] = reinterpret_cast<float(*)[MAX_ROWS][D]>(kv_red);
    __shared__ float p_s[MAX_ROWS][TT];
    __shared__ float m_s[MAX_ROWS], l_s[MAX_ROWS], a_s[MAX_ROWS];
    __shared__ int s_work;
    griddep_wait();  // the plan
    griddep_launch();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Hkv = c.num_kv_heads, G = Hq / Hkv, bs = c.block_size;
    const int nunits = ws.hdr[HDR_NSIMT];
    const int64_t nwork = (int64_t)nunits * Hkv;
    const T* kpool = reinterpret_cast<const T*>(c.k_pool);
    const T* vpool = reinterpret_cast<const T*>(c.v_pool);
    for (;;) {
        if (tid == 0) s_work = atomicAdd(&ws.hdr[HDR_SIMT_NEXT], 1);
        __syncthreads();
        const int w = s_work;
        __syncthreads();
        if (w >= nwork) break;
        const int u = w / Hkv, head = w % Hkv;
        const int32_t* U = ws.units + (int64_t)u * UNIT_INTS;
        const int q_lo = U[0], q_hi = U[1], t0u = U[2], t1u = U[3], ord = U[4];
        const int R = (q_hi - q_lo + 1) * G;
        // prefill (causal_pos0 >= 0): every row reads the one sequence in slots[0], and
        // the row of query i sees tokens up to causal_pos0 + i
        const int32_t* tab = table_row(c, layer, slots[causal_pos0 >= 0 ? 0 : q_lo]);
        for (int idx = tid; idx < R * D; idx += UNIT_THREADS) {
            const int r = idx / D, d = idx % D;
            const int seq = q_lo + r / G, g = r % G;
            q_s[r][d] = Elem<T>::to_f(q[(int64_t)seq * q_stride + (int64_t)(head * G + g) * D + d]) * qscale;
        }
        if (tid < MAX_ROWS) {
            m_s[tid] = -INFINITY;
            l_s[tid] = 0.f;
        }
        float acc[MAX_ROWS];
#pragma unroll
        for (int r = 0; r < MAX_ROWS; ++r) acc[r] = 0.f;
        const int d_own = tid % D, ts_own = tid / D;
        // K and V rows of a tile: 16-byte loads into registers, all of a thread's in
        // flight together; the next tile's are requested before this tile's scores
        constexpr int VEC = 16 / sizeof(T);  // elements per load
        constexpr int PER = (TT * D / VEC + UNIT_THREADS - 1) / UNIT_THREADS;
        uint4 kr[PER], vr[PER];
        auto load_tile = [&](int t0) {
            const int cnt = min(TT, t1u - t0);
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int idx = tid + k * UNIT_THREADS, j = idx / (D / VEC), d = (idx % (D / VEC)) * VEC;
                if (j < cnt) {
                    const int p = t0 + j;
                    const int blk = tab[p / bs];
                    if ((unsigned)blk < (unsigned)c.num_blocks) {
                        const int64_t off = pool_row(c, layer, blk, p % bs) + (int64_t)head * D + d;
                        kr[k] = *reinterpret_cast<const uint4*>(kpool + off);
                        vr[k] = *reinterpret_cast<const uint4*>(vpool + off);
                    } else {  // a corrupt table entry: recorded, and read as zeros
                        set_error(c, MENTAT_DEV_BAD_BLOCK, blk);
                        kr[k] = vr[k] = make_uint4(0, 0, 0, 0);
                    }
                }
            }
        };
        if (t0u < t1u) load_tile(t0u);
        for (int t0 = t0u; t0 < t1u; t0 += TT) {
            const int cnt = min(TT, t1u - t0);
            __syncthreads();  // the previous tile's K and V are read
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int idx = tid + k * UNIT_THREADS, j = idx / (D / VEC), d = (idx % (D / VEC)) * VEC;
                if (j < cnt) {
                    const T* ke = reinterpret_cast<const T*>(&kr[k]);
                    const T* ve = reinterpret_cast<const T*>(&vr[k]);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        k_s[j][d + e] = Elem<T>::to_f(ke[e]);
                        v_s[j][d + e] = Elem<T>::to_f(ve[e]);
                    }
                }
            }
            if (t0 + TT < t1u) load_tile(t0 + TT);
            __syncthreads();
            {  // scores: lane = token, warps stride the rows
                const int j = lane;
                for (int r = warp; r < R; r += UNIT_THREADS / 32) {
                    float s = -INFINITY;
                    const bool seen = j < cnt && (causal_pos0 < 0 || t0 + j <= causal_pos0 + q_lo + r / G);
                    if (seen) {  // four independent partial sums over the head dimension
                        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 8
                        for (int d = 0; d < D; d += 4) {
                            s0 = fmaf(q_s[r][d], k_s[j][d], s0);
                            s1 = fmaf(q_s[r][d + 1], k_s[j][d + 1], s1);
                            s2 = fmaf(q_s[r][d + 2], k_s[j][d + 2], s2);
                            s3 = fmaf(q_s[r][d + 3], k_s[j][d + 3], s3);
                        }
                        s = (s0 + s1) + (s2 + s3);
                    }
                    float mx = s;
#pragma unroll
                    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    const float m_old = m_s[r];
                    const float m_new = fmaxf(m_old, mx);
                    // a row with no token seen yet keeps m = -inf and gets p = 0
                    const float p = (seen && m_new != -INFINITY) ? exp2f(s - m_new) : 0.f;
                    float sum = p;
#pragma unroll
                    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                    p_s[r][j] = p;
                    __syncwarp();
                    if (lane == 0) {
                        const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_old - m_new);
                        a_s[r] = alpha;
                        l_s[r] = l_s[r] * alpha + sum;
                        m_s[r] = m_new;
                    }
                }
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < MAX_ROWS; ++r) {
                if (r < R) {
                    float a = acc[r] * a_s[r];
                    for (int j = ts_own; j < cnt; j += TS) a = fmaf(p_s[r][j], v_s[j][d_own], a);
                    acc[r] = a;
                }
            }
        }
        __syncthreads();
        if (TS > 1) {  // the tiles' K and V are no longer read: their space takes the partial sums
#pragma unroll
            for (int r = 0; r < MAX_ROWS; ++r)
                if (r < R) red_s[ts_own][r][d_own] = acc[r];
            __syncthreads();
        }
        if (ts_own == 0) {
#pragma unroll
            for (int r = 0; r < MAX_ROWS; ++r) {
                if (r < R) {
                    float a = acc[r];
#pragma unroll
                    for (int t = 1; t < TS; ++t) a += red_s[t][r][d_own];
                    const int seq = q_lo + r / G, hq = head * G + r % G;
                    const int64_t pi = ((int64_t)seq * max_parts + ord) * Hq + hq;
                    ws.part_o[pi * D + d_own] = a;
                    if (d_own == 0) {
                        ws.part_ml[pi * 2] = m_s[r];
                        ws.part_ml[pi * 2 + 1] = l_s[r];
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 3. merge: one warp per (sequence, q head), lane k over output dimensions
//    k D/32 .. k D/32 + D/32 - 1.  Lane p holds partial p's (m, l); a butterfly
//    of log-sum-exp combines gives every lane the total (M, L), and lane p's
//    weight 2^(m_p - M) reaches the others by shuffle.  The first 18 partial
//    rows and the first 64 partials' (m, l) are all requested before the part
//    count is read, so a warp waits for memory once; more rows are taken 18 at
//    a time.
// ---------------------------------------------------------------------------
constexpr int MERGE_WARPS = 4;  // warps per CTA

template <int VL> struct MergeVec;
template <> struct MergeVec<2> {
    using type = float2;
    static __device__ __forceinline__ float at(const float2& v, int k) { return k == 0 ? v.x : v.y; }
};
template <> struct MergeVec<4> {
    using type = float4;
    static __device__ __forceinline__ float at(const float4& v, int k) {
        return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
    }
};

template <typename T, int D>
__global__ void __launch_bounds__(32 * MERGE_WARPS) k_merge(mentat_kv_cache c, int n, int Hq, DecodeWs ws,
                                                         int max_parts, T* __restrict__ out, int64_t out_stride,
                                                         int skip_single) {
    constexpr int VL = D / 32;   // output elements per lane
    constexpr int B = 18;        // partial rows in flight per lane (config 4 has 17-18 partials)
    using MV = MergeVec<VL>;
    using VT = typename MV::type;
    griddep_wait();  // every unit kernel's partials
    griddep_launch();
    TL_FIRST(8);
    const int lane = threadIdx.x & 31;
    const int pair = blockIdx.x * MERGE_WARPS + (threadIdx.x >> 5);
    if (pair >= n * Hq) return;
    const int i = pair / Hq, hq = pair % Hq;
    const float* ml = ws.part_ml + ((int64_t)i * max_parts * Hq + hq) * 2;  // partial p at ml[p * Hq * 2]
    const int64_t pstride = (int64_t)Hq * 2;
    const VT* po = reinterpret_cast<const VT*>(ws.part_o + ((int64_t)i * max_parts * Hq + hq) * D) + lane;
    const int64_t ostride = (int64_t)Hq * D / VL;  // in VT
    // prefill: the unit kernel wrote the output of a query with one partial itself; its
    // part count is read before any partial row (the decode merge loads the rows first)
    if (skip_single && ws.hdr[HDR_TC_ABORT] == 0 && ws.hdr[HDR_ERR] == 0 && ws.nparts[i] == 1) return;
    // rows up to max_parts exist in the workspace; those past the count get weight 0
    VT v[B];
#pragma unroll
    for (int j = 0; j < B; ++j)
        if (j < max_parts) v[j] = po[j * ostride];
    const float2 ninf = make_float2(-INFINITY, 0.f);
    const float2 ml_lo = lane < max_parts ? *reinterpret_cast<const float2*>(ml + lane * pstride) : ninf;
    const float2 ml_hi = lane + 32 < max_parts ? *reinterpret_cast<const float2*>(ml + (lane + 32) * pstride) : ninf;
    // this lane's (m, l) of partial p = (a multiple of 32) + lane
    auto ml_of = [&](int p) -> float2 {
        return p < 32 ? ml_lo : (p < 64 ? ml_hi : *reinterpret_cast<const float2*>(ml + p * pstride));
    };
    // A failed plan (HDR_ERR) stored part counts that may exceed max_parts and
    // wrote no units; a tensor-core unit kernel that gave up a bounded wait left
    // partials unwritten.  Either way the output is zeroed, and the part count
    // is clamped so that no row past the workspace is read.
    const bool aborted = ws.hdr[HDR_TC_ABORT] != 0 || ws.hdr[HDR_ERR] != 0;
    const int P = aborted ? 0 : min(ws.nparts[i], max_parts);
    if (ws.hdr[HDR_TC_ABORT] != 0 && pair == 0 && lane == 0) set_error(c, MENTAT_DEV_DECODE_TIMEOUT, 1);
    // (m1, l1) + (m2, l2) = (M, l1 2^(m1 - M) + l2 2^(m2 - M))
    auto comb = [](float& m, float& l, float m2, float l2) {
        const float mn = fmaxf(m, m2);
        l = (m == -INFINITY ? 0.f : l * exp2f(m - mn)) + (m2 == -INFINITY ? 0.f : l2 * exp2f(m2 - mn));
        m = mn;
    };
    float M = -INFINITY, L = 0.f;
    for (int p0 = 0; p0 < P; p0 += 32) {
        float m = -INFINITY, l = 0.f;
        if (p0 + lane < P) {
            const float2 x = ml_of(p0 + lane);
            m = x.x;
            l = x.y;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) comb(m, l, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, l, o));
        comb(M, L, m, l);
    }
    float a[VL];
#pragma unroll
    for (int k = 0; k < VL; ++k) a[k] = 0.f;
    for (int b0 = 0; b0 < P; b0 += B) {
        if (b0 > 0) {  // rows after the first batch
#pragma unroll
            for (int j = 0; j < B; ++j)
                if (b0 + j < P) v[j] = po[(int64_t)(b0 + j) * ostride];
        }
        // weights of rows b0 .. b0 + B - 1: lane k holds row (b0 & ~31) + k's
        const int w0 = b0 & ~31;
        const float wlo = w0 + lane < P ? exp2f(ml_of(w0 + lane).x - M) : 0.f;
        const float whi = w0 + 32 + lane < P ? exp2f(ml_of(w0 + 32 + lane).x - M) : 0.f;
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const int r = b0 + j - w0;  // < 64: b0 is a multiple of B, w0 = b0 rounded down to 32
            const float wj = __shfl_sync(0xffffffffu, r < 32 ? wlo : whi, r & 31);
            if (b0 + j < P) {
#pragma unroll
                for (int k = 0; k < VL; ++k) a[k] = fmaf(MV::at(v[j], k), wj, a[k]);
            }
        }
    }
    const bool ok = P > 0 && L > 0.f && !aborted;
    T* dst = out + (int64_t)i * out_stride + (int64_t)hq * D + lane * VL;
#pragma unroll
    for (int k = 0; k < VL; ++k) dst[k] = Elem<T>::from_f(ok ? a[k] / L : 0.f);
    TL_LAST(9);
}

}  // namespace mentat

#include "decode_tc.cuh"
#include "decode_tcn.cuh"

namespace mentat {

// optional per-launch stage timing (plan, FFMA units, wide tensor-core units,
// narrow tensor-core units, merge) with CUDA events on the launch stream;
// enabled by mentat_profile_enable
constexpr int PROF_STAGES = 5;
constexpr int PROF_MAX = 4096;
static cudaEvent_t g_prof_ev[PROF_STAGES + 1][PROF_MAX];
static int g_prof_cap = 0, g_prof_n = 0;
static bool g_prof_on = false;

static inline void prof_mark(int stage, cudaStream_t s) {
    if (g_prof_on && g_prof_n < g_prof_cap) cudaEventRecord(g_prof_ev[stage][g_prof_n], s);
}

static int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// rows at or above which a segment goes to the tensor-core kernel rather than
// the FFMA one.  Default 1: on B200 even a 4-row unit is faster on the tensor
// cores (its padded M=128 MMAs cost less than the memory time of the tile);
// MENTAT_TC_MIN_ROWS overrides, a value above 256 disables the tensor-core path.
static int tc_min_rows() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MENTAT_TC_MIN_ROWS");
        v = (e && *e) ? atoi(e) : 1;
        if (v < 1) v = 1;
    }
    return v;
}

// narrow (transposed) tensor-core units for segments of <= 32 rows; on by
// default, MENTAT_NARROW=0 sends those segments to the wide kernel instead
static bool narrow_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MENTAT_NARROW");
        v = (e && *e) ? (atoi(e) != 0) : 1;
    }
    return v != 0;
}

// threads of the plan's CTA: at least one per sequence (boundaries and
// segments are spread over the threads), a multiple of 32, at most 1,024, and
// at least MENTAT_PLAN_THREADS (default 512: on config 4's 64 sequences the
// plan takes 1.5 us less than with 1,024 threads, whose block-wide barriers
// cost more, and 2.3 us less than with 128, which loop over ~900 units)
static int plan_threads(int n) {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MENTAT_PLAN_THREADS");
        v = (e && *e) ? atoi(e) : 512;
        v = std::min(1024, std::max(32, v));
    }
    return std::min(1024, (std::max(v, n) + 31) / 32 * 32);
}

// wide tensor-core CTAs that take units in a decode call: 0 (default) lets the
// plan choose from the work of the two tensor-core queues (tc_ctas);
// MENTAT_TC_CTAS=k fixes it at k
static int tc_ctas_fixed() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MENTAT_TC_CTAS");
        v = (e && *e) ? atoi(e) : 0;
        if (v < 0) v = 0;
    }
    return v;
}

// Decode kernels go out with programmatic stream serialization (pdl_enabled,
// launch in common.cuh): each may be scheduled while its predecessor on the
// stream runs, and waits for it with griddep_wait (the narrow kernel waits for
// the wide one only at its end).

template <typename T, int D>
static int launch_decode(const mentat_kv_cache* c, int layer, const int32_t* slots, int n, const void* q,
                         int64_t q_stride, int Hq, void* out, int64_t out_stride, float scale, DecodeWs ws,
                         int max_parts, bool reuse_plan, cudaStream_t s) {
    const int G = Hq / c->num_kv_heads;
    const PoolMaps* maps = nullptr;
    bool tc_ok = false, narrow_ok = false;
    if constexpr (!std::is_same<T, float>::value) {
        tc_ok = tc_supported(c) && tc_min_rows() <= TC_MAX_ROWS && ((uintptr_t)q % 16 == 0) && (q_stride % 8 == 0);
        if (tc_ok) {
            maps = pool_maps(c, layer);
            tc_ok = maps != nullptr;
        }
        narrow_ok = tc_ok && D == 128 && narrow_enabled();
        // the shared-memory attribute is per device: one flag per device ordinal
        static bool attr[64] = {};
        int dev = 0;
        if (tc_ok && (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)) return MENTAT_ERR_CUDA;
        if (tc_ok && !attr[dev]) {
            if (cudaFuncSetAttribute(k_units_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) !=
                cudaSuccess)
                return MENTAT_ERR_CUDA;
            if constexpr (D == 128)
                if (cudaFuncSetAttribute(k_units_tcn<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, TCN_SMEM) !=
                    cudaSuccess)
                    return MENTAT_ERR_CUDA;
            attr[dev] = true;
        }
    }
    PlanParams pp{G, tc_ok ? 1 : 0, narrow_ok ? 1 : 0, tc_min_rows(), num_sms(), tc_ctas_fixed()};
    prof_mark(0, s);
    const bool pdl = pdl_enabled();
    if (reuse_plan) {
        if (launch(pdl, k_plan_reuse, dim3(1), dim3(32), 0, s, *c, n, max_parts, plan_route(pp), G, ws) !=
            cudaSuccess)
            return MENTAT_ERR_CUDA;
        MENTAT_CHECK_LAUNCH();
    } else {
        if (n > 1) {
            if (launch(pdl, k_lcp, dim3(n - 1), dim3(LCP_THREADS), 0, s, *c, layer, slots, n, ws) != cudaSuccess)
                return MENTAT_ERR_CUDA;
            MENTAT_CHECK_LAUNCH();
        }
        // the plan's dynamic shared memory may exceed the default 48 KB (per-device attribute)
        static bool plan_attr[64] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MENTAT_ERR_CUDA;
        if (!plan_attr[dev]) {
            if (cudaFuncSetAttribute(k_plan, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     plan_smem_bytes(PLAN_MAX_SEQS)) != cudaSuccess)
                return MENTAT_ERR_CUDA;
            plan_attr[dev] = true;
        }
        if (launch(pdl, k_plan, dim3(1), dim3(plan_threads(n)), plan_smem_bytes(n), s, *c, layer, slots, n, pp, ws,
                   max_parts) != cudaSuccess)
            return MENTAT_ERR_CUDA;
        MENTAT_CHECK_LAUNCH();
    }
    prof_mark(1, s);
    const float qscale = scale * 1.4426950408889634f;  // base-2 softmax
    const T* qt = reinterpret_cast<const T*>(q);
    // a segment has at least G query rows, so with the tensor-core path on and
    // tc_min_rows <= G no unit can land in the FFMA queue
    if (!(tc_ok && tc_min_rows() <= G)) {
        if (launch(pdl, k_units<T, D>, dim3(num_sms()), dim3(UNIT_THREADS), 0, s, *c, layer, slots, qt, q_stride,
                   Hq, qscale, ws, max_parts, -1) != cudaSuccess)
            return MENTAT_ERR_CUDA;
        MENTAT_CHECK_LAUNCH();
    }
    prof_mark(2, s);
    if constexpr (!std::is_same<T, float>::value) {
        if (tc_ok) {
            if (launch(pdl, k_units_tc<T, D>, dim3(num_sms()), dim3(TC_THREADS), TC_SMEM, s, maps->mk, maps->mv, *c,
                       layer, slots, qt, q_stride, Hq, qscale, ws, max_parts, -1, (T*)nullptr, (int64_t)0) !=
                cudaSuccess)
                return MENTAT_ERR_CUDA;
            MENTAT_CHECK_LAUNCH();
        }
    }
    prof_mark(3, s);
    if constexpr (!std::is_same<T, float>::value && D == 128) {
        if (narrow_ok) {
            if (launch(pdl, k_units_tcn<T, D>, dim3(num_sms()), dim3(TCN_THREADS), TCN_SMEM, s, maps->mk, maps->mv,
                       *c, layer, slots, qt, q_stride, Hq, qscale, ws, max_parts) != cudaSuccess)
                return MENTAT_ERR_CUDA;
            MENTAT_CHECK_LAUNCH();
        }
    }
    prof_mark(4, s);
    if (launch(pdl, k_merge<T, D>, dim3((n * Hq + MERGE_WARPS - 1) / MERGE_WARPS), dim3(32 * MERGE_WARPS),
               0, s, *c, n, Hq, ws, max_parts, reinterpret_cast<T*>(out), out_stride, 0) != cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    prof_mark(5, s);
    if (g_prof_on && g_prof_n < g_prof_cap) ++g_prof_n;
    return MENTAT_OK;
}

// Chunk length of a prefill's units.  A query group's units run one after
// another on one SM, so a group may take its whole range in one unit (one
// partial per query, no merge) when that range is at most 1.5 times the average
// work per SM, or at most 2,048 tokens (16 tiles: shorter than a merge pass
// costs); otherwise its range is cut into chunks of about that average.
static int prefill_chunk_for(int n, int pos0, int G, int hkv, int kind) {
    const int64_t L = (int64_t)pos0 + n;
    const int spu = std::max(1, (kind == KIND_TC ? TC_MAX_ROWS : MAX_ROWS) / G);
    const int64_t ngroups = (n + spu - 1) / spu;
    int64_t total = 0;  // tokens seen by all groups: group g's last query is min(n, (g + 1) spu) - 1
    for (int64_t g = 0; g < ngroups; ++g) total += pos0 + std::min<int64_t>(n, (g + 1) * spu);
    const int64_t avg = total * hkv / std::max(1, num_sms());
    if (L <= CHUNK_TC || 2 * L <= 3 * avg) return (int)std::min<int64_t>((L + 15) / 16 * 16, INT32_MAX - 15);
    return (int)((std::max<int64_t>(avg, 256) + 127) / 128 * 128);
}

// Causal prefill attention of n queries of the sequence in slots[0] (query i at
// position pos0 + i, its K/V already cached): k_prefill_plan, then the wide
// tensor-core kernel (bf16 / fp16 caches) or the FFMA kernel (fp32), then the merge.
template <typename T, int D>
static int launch_prefill(const mentat_kv_cache* c, int layer, const int32_t* slot, int n, int pos0, const void* q,
                          int64_t q_stride, int Hq, void* out, int64_t out_stride, float scale, DecodeWs ws,
                          int max_parts, cudaStream_t s) {
    const int G = Hq / c->num_kv_heads;
    bool tc_ok = false;
    const PoolMaps* maps = nullptr;
    if constexpr (!std::is_same<T, float>::value) {
        tc_ok = tc_supported(c) && ((uintptr_t)q % 16 == 0) && (q_stride % 8 == 0);
        if (tc_ok) {
            maps = pool_maps(c, layer);
            tc_ok = maps != nullptr;
        }
        static bool attr[64] = {};
        int dev = 0;
        if (tc_ok && (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)) return MENTAT_ERR_CUDA;
        if (tc_ok && !attr[dev]) {
            if (cudaFuncSetAttribute(k_units_tc<T, D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM) !=
                cudaSuccess)
                return MENTAT_ERR_CUDA;
            attr[dev] = true;
        }
    }
    const bool pdl = pdl_enabled();
    const int kind = tc_ok ? KIND_TC : KIND_FFMA;
    const int chunk = prefill_chunk_for(n, pos0, G, c->num_kv_heads, kind);
    // the plan's largest part count is known here: a workspace sized for fewer is refused
    // before anything runs (the plan kernel's overflow check stays as a guard)
    if (((int64_t)pos0 + n + chunk - 1) / chunk > max_parts) return MENTAT_ERR_ARG;
    // the tensor-core kernel writes the rows of single-partial queries itself
    const bool direct = tc_ok && (uintptr_t)out % 16 == 0 && out_stride % 8 == 0;
    if (launch(pdl, k_prefill_plan, dim3(1), dim3(1024), 0, s, *c, n, pos0, G, kind, chunk, ws, max_parts) !=
        cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    const float qscale = scale * 1.4426950408889634f;  // base-2 softmax
    const T* qt = reinterpret_cast<const T*>(q);
    if (!tc_ok) {
        if (launch(pdl, k_units<T, D>, dim3(num_sms()), dim3(UNIT_THREADS), 0, s, *c, layer, slot, qt, q_stride,
                   Hq, qscale, ws, max_parts, pos0) != cudaSuccess)
            return MENTAT_ERR_CUDA;
        MENTAT_CHECK_LAUNCH();
    }
    if constexpr (!std::is_same<T, float>::value) {
        if (tc_ok) {
            if (launch(pdl, k_units_tc<T, D, true>, dim3(num_sms()), dim3(TC_THREADS), TC_SMEM, s, maps->mk, maps->mv, *c,
                       layer, slot, qt, q_stride, Hq, qscale, ws, max_parts, pos0,
                       direct ? reinterpret_cast<T*>(out) : (T*)nullptr, out_stride) != cudaSuccess)
                return MENTAT_ERR_CUDA;
            MENTAT_CHECK_LAUNCH();
        }
    }
    // every query in one unit and written by the tensor-core kernel: nothing to merge
    // (a unit that gave up a bounded wait records MENTAT_DEV_DECODE_TIMEOUT itself)
    if (direct && chunk >= pos0 + n) return MENTAT_OK;
    if (launch(pdl, k_merge<T, D>, dim3((n * Hq + MERGE_WARPS - 1) / MERGE_WARPS), dim3(32 * MERGE_WARPS),
               0, s, *c, n, Hq, ws, max_parts, reinterpret_cast<T*>(out), out_stride, direct ? 1 : 0) != cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

}  // namespace mentat

using namespace mentat;

extern "C" {

int64_t mentat_decode_workspace_bytes(int32_t n, int32_t hq, int32_t d, int32_t max_parts) {
    DecodeWs w;
    int64_t total = 0;
    ws_carve(nullptr, n, hq, d, max_parts, &w, &total);
    return total;
}

int32_t mentat_decode_max_parts(int32_t n, int32_t max_len, int32_t block_size) {
    (void)block_size;
    return (max_len + CHUNK - 1) / CHUNK + n + 1;
}

int mentat_profile_enable(int32_t max_records) {
    if (max_records < 0 || max_records > PROF_MAX) return MENTAT_ERR_ARG;
    for (int st = 0; st <= PROF_STAGES; ++st)
        for (int i = g_prof_cap; i < max_records; ++i)
            if (cudaEventCreate(&g_prof_ev[st][i]) != cudaSuccess) return MENTAT_ERR_CUDA;
    if (max_records > g_prof_cap) g_prof_cap = max_records;
    g_prof_n = 0;
    g_prof_on = max_records > 0;
    return MENTAT_OK;
}

int mentat_profile_collect(double* stage_ms, int32_t* launches) {
    if (!stage_ms || !launches) return MENTAT_ERR_ARG;
    for (int st = 0; st < PROF_STAGES; ++st) stage_ms[st] = 0.0;
    *launches = g_prof_n;
    if (g_prof_n > 0 && cudaEventSynchronize(g_prof_ev[PROF_STAGES][g_prof_n - 1]) != cudaSuccess)
        return MENTAT_ERR_CUDA;
    for (int i = 0; i < g_prof_n; ++i)
        for (int st = 0; st < PROF_STAGES; ++st) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, g_prof_ev[st][i], g_prof_ev[st + 1][i]) != cudaSuccess) return MENTAT_ERR_CUDA;
            stage_ms[st] += ms;
        }
    g_prof_n = 0;
    return MENTAT_OK;
}

int mentat_decode_set_wait_probe(int64_t cycles) {
    if (cycles < 0) return MENTAT_ERR_ARG;
    const long long v = cycles;
    if (cudaMemcpyToSymbol(g_decode_wait_probe, &v, sizeof(v)) != cudaSuccess) {
        (void)cudaGetLastError();
        return MENTAT_ERR_CUDA;
    }
    return MENTAT_OK;
}

static int paged_decode(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n, const void* q,
                        int64_t q_stride, int32_t Hq, void* out, int64_t out_stride, float scale, void* workspace,
                        int64_t ws_bytes, int32_t max_parts, bool reuse_plan, cudaStream_t s) {
    if (!c || layer < 0 || layer >= c->num_layers || n < 0 || n > PLAN_MAX_SEQS || !c->k_pool || !c->v_pool ||
        Hq <= 0 || c->num_kv_heads <= 0 || Hq % c->num_kv_heads || max_parts <= 0)
        return MENTAT_ERR_ARG;
    if (n == 0) return MENTAT_OK;
    if (!slots || !q || !out || !workspace) return MENTAT_ERR_ARG;
    const int G = Hq / c->num_kv_heads;
    if (G > MAX_ROWS) return MENTAT_ERR_UNSUPPORTED;
    DecodeWs w;
    int64_t need = 0;
    ws_carve(workspace, n, Hq, c->head_dim, max_parts, &w, &need);
    if (ws_bytes < need) return MENTAT_ERR_ARG;
    const int D = c->head_dim;
#define MENTAT_DISPATCH(T)                                                                                       \
    if (D == 128)                                                                                                \
        return launch_decode<T, 128>(c, layer, slots, n, q, q_stride, Hq, out, out_stride, scale, w, max_parts,  \
                                     reuse_plan, s);                                                             \
    if (D == 64)                                                                                                 \
        return launch_decode<T, 64>(c, layer, slots, n, q, q_stride, Hq, out, out_stride, scale, w, max_parts,   \
                                    reuse_plan, s);                                                              \
    return MENTAT_ERR_UNSUPPORTED;
    switch (c->dtype) {
        case MENTAT_F32: { MENTAT_DISPATCH(float) }
        case MENTAT_BF16: { MENTAT_DISPATCH(__nv_bfloat16) }
        case MENTAT_F16: { MENTAT_DISPATCH(__half) }
        default: return MENTAT_ERR_UNSUPPORTED;
    }
#undef MENTAT_DISPATCH
}

int mentat_paged_decode(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n, const void* q,
                        int64_t q_stride, int32_t Hq, void* out, int64_t out_stride, float scale, void* workspace,
                        int64_t ws_bytes, int32_t max_parts, cudaStream_t s) {
    return paged_decode(c, layer, slots, n, q, q_stride, Hq, out, out_stride, scale, workspace, ws_bytes,
                        max_parts, false, s);
}

int32_t mentat_prefill_max_parts(const mentat_kv_cache* c, int32_t n, int32_t pos0, int32_t num_q_heads) {
    if (!c || n <= 0 || pos0 < 0 || c->num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % c->num_kv_heads)
        return 0;
    // with the tensor-core kernel's query groups; the FFMA kernel's groups are
    // smaller, see more tokens in total and take longer chunks, so no more parts
    const int kind = tc_supported(c) ? KIND_TC : KIND_FFMA;
    const int64_t len = (int64_t)pos0 + n;
    const int ch = prefill_chunk_for(n, pos0, num_q_heads / c->num_kv_heads, c->num_kv_heads, kind);
    return (int32_t)((len + ch - 1) / ch);
}

int mentat_paged_prefill(const mentat_kv_cache* c, int32_t layer, const int32_t* slot, int32_t n, int32_t pos0,
                         const void* q, int64_t q_stride, int32_t Hq, void* out, int64_t out_stride, float scale,
                         void* workspace, int64_t ws_bytes, int32_t max_parts, cudaStream_t s) {
    if (!c || layer < 0 || layer >= c->num_layers || n < 0 || pos0 < 0 || !c->k_pool || !c->v_pool || Hq <= 0 ||
        c->num_kv_heads <= 0 || Hq % c->num_kv_heads)
        return MENTAT_ERR_ARG;
    if (n == 0) return MENTAT_OK;
    if (!slot || !q || !out || !workspace || max_parts <= 0) return MENTAT_ERR_ARG;
    const int G = Hq / c->num_kv_heads;
    if (G > MAX_ROWS) return MENTAT_ERR_UNSUPPORTED;
    DecodeWs w;
    int64_t need = 0;
    ws_carve(workspace, n, Hq, c->head_dim, max_parts, &w, &need);
    if (ws_bytes < need) return MENTAT_ERR_ARG;
    const int D = c->head_dim;
#define MENTAT_DISPATCH(T)                                                                                       \
    if (D == 128)                                                                                                \
        return launch_prefill<T, 128>(c, layer, slot, n, pos0, q, q_stride, Hq, out, out_stride, scale, w,       \
                                      max_parts, s);                                                             \
    if (D == 64)                                                                                                 \
        return launch_prefill<T, 64>(c, layer, slot, n, pos0, q, q_stride, Hq, out, out_stride, scale, w,        \
                                     max_parts, s);                                                              \
    return MENTAT_ERR_UNSUPPORTED;
    switch (c->dtype) {
        case MENTAT_F32: { MENTAT_DISPATCH(float) }
        case MENTAT_BF16: { MENTAT_DISPATCH(__nv_bfloat16) }
        case MENTAT_F16: { MENTAT_DISPATCH(__half) }
        default: return MENTAT_ERR_UNSUPPORTED;
    }
#undef MENTAT_DISPATCH
}

int mentat_paged_decode_reuse_plan(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                                   const void* q, int64_t q_stride, int32_t Hq, void* out, int64_t out_stride,
                                   float scale, void* workspace, int64_t ws_bytes, int32_t max_parts,
                                   cudaStream_t s) {
    return paged_decode(c, layer, slots, n, q, q_stride, Hq, out, out_stride, scale, workspace, ws_bytes,
                        max_parts, true, s);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without a caller-provided workspace, for hosts that cannot allocate
// device memory at call time.  The workspace lives in this fixed array; host
// code must not pass the symbol itself to a kernel (on the host it is only a
// stand-in), so its device address is looked up once per device.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[MENTAT_NOALLOC_SCRATCH_BYTES];
static void* g_noalloc_addr[64] = {nullptr};

extern "C" int mentat_paged_decode_noalloc(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                                           const void* q, int64_t q_stride, int32_t Hq, void* out, int64_t out_stride,
                                           float scale, int32_t max_parts, cudaStream_t s) {
    if (!c || Hq <= 0 || n < 0 || n > PLAN_MAX_SEQS || max_parts <= 0) return MENTAT_ERR_ARG;
    const int64_t need = mentat_decode_workspace_bytes(n, Hq, c->head_dim, max_parts);
    if (need > (int64_t)MENTAT_NOALLOC_SCRATCH_BYTES) return MENTAT_ERR_SCRATCH_LIMIT;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        (void)cudaGetLastError();
        return MENTAT_ERR_CUDA;
    }
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            (void)cudaGetLastError();
            return MENTAT_ERR_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    return mentat_paged_decode(c, layer, slots, n, q, q_stride, Hq, out, out_stride, scale, g_noalloc_addr[dev],
                               (int64_t)MENTAT_NOALLOC_SCRATCH_BYTES, max_parts, s);
}

#ifdef MENTAT_TC_TRACE
extern "C" int mentat_plan_trace_dump(long long* host) {
    return cudaMemcpyFromSymbol(host, g_plan_trace, sizeof(long long) * 16) == cudaSuccess ? 0 : -2;
}
extern "C" int mentat_timeline_reset() {
    unsigned long long init[32];
    for (int k = 0; k < 32; ++k) init[k] = (k % 2 == 0) ? ~0ull : 0ull;  // even: first (min), odd: last (max)
    static long long zero[4096] = {};
    if (cudaMemcpyToSymbol(mentat::g_tc_trace, zero, sizeof(zero)) != cudaSuccess) return -2;
    return cudaMemcpyToSymbol(mentat::g_timeline, init, sizeof(init)) == cudaSuccess ? 0 : -2;
}
extern "C" int mentat_timeline_dump(unsigned long long* host) {
    return cudaMemcpyFromSymbol(host, mentat::g_timeline, sizeof(unsigned long long) * 32) == cudaSuccess ? 0 : -2;
}
extern "C" int mentat_cta_end_dump(unsigned long long* host) {
    return cudaMemcpyFromSymbol(host, mentat::g_cta_end, sizeof(unsigned long long) * 512) == cudaSuccess ? 0 : -2;
}
extern "C" int mentat_tc_trace_dump(long long* host, int n) {
    return cudaMemcpyFromSymbol(host, mentat::g_tc_trace, sizeof(long long) * (n < 4096 ? n : 4096)) == cudaSuccess ? 0 : -2;
}
#endif
