// Tensor-core (tcgen05) decode units for bf16 / fp16 caches, head_dim 64 or 128,
// KV block 16.  Included by decode_attention.cu; consumes the plan's wide
// tensor-core unit queue (segments shared by more than 32 query rows: the
// shared prefixes of a tree).
//
// One CTA per SM (persistent; two softmax warpgroups, an MMA warp and a TMA
// warp; ~226 KB of shared memory).  Per unit and kv head:
//   * Q rows of all sharing sequences (up to 256 = two M=128 row tiles) are
//     written once to shared memory in the K-major 128-byte-swizzled layout.
//   * K and V come in 128-token tiles (8 blocks) by TMA from the paged pool,
//     through separate K (3-stage) and V (2-stage) mbarrier rings, each
//     (block, head) box read once for every row of the unit.
//   * S = Q K^T: tcgen05.mma kind::f16, M=128, N=128, K=head_dim, accumulator
//     in TMEM.  Each thread owns one query row (TMEM lane): scale, mask, online
//     softmax in base 2 with a lazily raised reference max (O is rescaled in
//     TMEM only when the row max grows by more than 2^8), P rounded to the
//     cache dtype and stored back into TMEM over the S columns it came from.
//   * O += P V: tcgen05.mma with A = P in TMEM, M=128, N=head_dim, K=128
//     tokens, V read MN-major from shared memory.
//   * The two row tiles ping-pong: S of row tile r for tile i+1 is issued right
//     after r's P V(i), so the tensor pipe works on one row tile while the
//     other's softmax runs.  Issuing S(i+1) after P V(i) also orders the MMAs
//     so that when S(i+1) is complete, O holds P V(i) and may be rescaled.
//   * The unnormalised (m, l, o) partial goes to the workspace like the FFMA
//     units, and k_merge combines both kinds.  Each thread stages its O row in the
//     idle K/V ring and one bulk copy per row moves it out (2.9 us for 128 KB
//     against 5.7 us for per-thread stores).
// Every mbarrier wait is bounded by a clock limit; on timeout the CTA records
// HDR_TC_ABORT, stops issuing work, drains its outstanding copies (bounded) and
// frees its TMEM before returning.

#pragma once

#include <cuda.h>

#include <type_traits>

namespace mentat {

#ifdef MENTAT_TC_TRACE
__device__ long long g_tc_trace[4096];
// debug builds only: lane 0 of every warp of the CTA that runs work item 0 stamps its events
// (globaltimer ns) at g_tc_trace[warp * 400 + k]
#define TC_TRACE(k) do { if ((threadIdx.x & 31) == 0 && g_trace_on && (k) < 400) g_tc_trace[(threadIdx.x >> 5) * 400 + (k)] = (long long)mentat::gtime(); } while (0)
#else
#define TC_TRACE(k) do { } while (0)
#endif

constexpr int TC_SOFTMAX_WARPS = 8;        // two warpgroups: one per 128-row tile
constexpr int TC_THREADS = (TC_SOFTMAX_WARPS + 2) * 32;  // + an MMA warp and a TMA warp
constexpr int TC_TILE = 128;                // tokens per K/V tile (8 blocks of 16)
constexpr int TC_KST = 3;                   // K ring stages
constexpr int TC_VST = 2;                   // V ring stages
constexpr int TC_RT = 2;                    // row tiles (128 rows each)
constexpr int TC_Q_BYTES = TC_RT * 2 * 128 * 128;          // 64 KB: [rt][half][128 rows][128 B]
constexpr int TC_KV_TILE = 2 * TC_TILE * 128;               // 32 KB: [half][128 tok][128 B]
constexpr int TC_OFF_Q = 0;
constexpr int TC_OFF_K = TC_OFF_Q + TC_Q_BYTES;
constexpr int TC_OFF_V = TC_OFF_K + TC_KST * TC_KV_TILE;
constexpr int TC_OFF_BAR = TC_OFF_V + TC_VST * TC_KV_TILE;  // mbarriers
constexpr int TC_SMEM = TC_OFF_BAR + 256 + 1024;            // + alignment slack
constexpr uint32_t TC_TMEM_COLS = 512;      // O[rt] at rt*256, S[rt] at rt*256 + 128
                                            // (P, packed pairs, overwrites the first 64 columns of its S)
constexpr long long TC_WAIT_CYCLES = 4000000000ll;  // ~2 s at 1.9 GHz

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait: false once `limit` clock cycles have passed
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, long long limit) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) return false;
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, TC_WAIT_CYCLES);
}
// Test hook (mentat_decode_set_wait_probe): when g_decode_wait_probe > 0, one
// thread of every tensor-core unit CTA first waits on `probe_bar`, which nothing
// arrives on, for that many cycles.  The wait gives up, and the CTA takes its
// ordinary timeout path before it has issued any copy or MMA.
__device__ __forceinline__ bool wait_probe(uint32_t probe_bar) {
    const long long limit = g_decode_wait_probe;
    return limit <= 0 || mbar_wait_for(probe_bar, 0, limit);
}
// A table entry outside [0, num_blocks) is recorded as MENTAT_DEV_BAD_BLOCK and
// replaced by the row just past the pool, which TMA reads as zeros.
__device__ __forceinline__ int checked_block(const mentat_kv_cache& c, int b) {
    if ((unsigned)b < (unsigned)c.num_blocks) return b;
    set_error(c, MENTAT_DEV_BAD_BLOCK, b);
    return c.num_blocks;
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// bulk copy of `bytes` from this CTA's shared memory to global memory (no tensor map,
// no multicast); both addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// the bulk copies of this thread have read their shared-memory sources
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the bulk copies of this thread have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void bar_sync_id(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// named barrier 1 over `count` threads that also ORs a flag across them
__device__ __forceinline__ int bar_sync_or(int count, int flag) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(flag), "r"(count)
        : "memory");
    return (int)out;
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], kind::f16, one thread issues
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]: A (K-major) packed two 16-bit values per column
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// the same with the accumulate flag fixed at compile time
template <bool ACC>
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "n"(ACC ? 1 : 0)
        : "memory");
}
template <bool ACC>
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "n"(ACC ? 1 : 0)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 64 consecutive fp32 columns of this thread's TMEM lane (two loads, one wait)
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr), "r"(taddr + 32)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// 128 consecutive fp32 columns of this thread's TMEM lane (one load, one wait)
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* v) {
    uint32_t r[128];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,"
        "%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
        "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,"
        "%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,"
        "%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
          "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
          "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
          "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
          "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
          "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
          "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
          "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
          "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 8 / 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float* v) {
    static_assert(N == 8 || N == 16 || N == 32, "tmem_ld_n");
    if constexpr (N == 8) tmem_ld8(taddr, v);
    else if constexpr (N == 16) tmem_ld16(taddr, v);
    else tmem_ld32(taddr, v);
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                   "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                   "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
          "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
          "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
          "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
          "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// shared-memory matrix descriptor (Blackwell version 1); layout 2 = 128-byte
// swizzle, 4 = 64-byte swizzle
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // version
    d |= (uint64_t)layout << 61;
    return d;
}
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return sdesc(saddr, lbo_bytes, sbo_bytes, 2);
}
// instruction descriptor, kind::f16, fp32 accumulate
__host__ __device__ constexpr uint32_t idesc_f16(int fmt, int m, int n, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_mn_major << 15) |
           ((uint32_t)b_mn_major << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// byte offset of (row, 16-byte chunk) in a K-major 128B-swizzled [rows][128 B] region
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
    return (uint32_t)(row >> 3) * 1024u + (uint32_t)(row & 7) * 128u + (uint32_t)((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
    __device__ __forceinline__ static uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    // the packed values back in fp32
    __device__ __forceinline__ static float lo(uint32_t w) { return __uint_as_float(w << 16); }
    __device__ __forceinline__ static float hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
};
template <> struct Pair<__half> {
    __device__ __forceinline__ static uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static float lo(uint32_t w) {
        return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
    }
    __device__ __forceinline__ static float hi(uint32_t w) {
        return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
    }
};

// Roles: warps 0-3 softmax row tile 0, warps 4-7 softmax row tile 1 (TMEM
// lane quarter = warp % 4), warp 8 lane 0 issues the MMAs, warp 9 the TMA
// loads (lanes 0-7, one 16-token block each).
// PREFILL (the causal prefill instantiation):
//  * in the sequence's first tile (tokens 0-127), P goes to the tensor cores as
//    two 16-bit terms, P_hi = round(P) and P_lo = round(P - P_hi), in TMEM
//    columns 0-63 and 64-127 of the S region, and O takes both products.  The
//    rows of the first 128 queries see only that tile; one that sees a few
//    tokens would otherwise carry the 2^-9 relative rounding of its one or two
//    weights straight into its output.  Later tiles round P once, as decode
//    (and flash attention) do, where many weights average the rounding out.
//  * a unit may span any number of tiles: the TMA warp reads each tile's block
//    ids one tile ahead instead of the whole unit's up front.
//  * with out != nullptr, the softmax threads of a unit whose queries have one
//    partial (the unit covers their whole range) write their rows' normalised
//    outputs straight to out; the merge skips those queries.
template <typename T, int D, bool PREFILL = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
k_units_tc(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
           mentat_kv_cache c, int layer, const int32_t* slots, const T* __restrict__ q, int64_t q_stride, int Hq,
           float scale_log2, DecodeWs ws, int max_parts, int causal_pos0, T* __restrict__ out, int64_t out_stride) {
    constexpr bool PSPLIT = PREFILL;
    constexpr int HALVES = D / 64;                // 128-byte column halves of a row
    constexpr int FMT = Elem<T>::code == MENTAT_BF16 ? 1 : 0;
    constexpr uint32_t IDESC_QK = idesc_f16(FMT, 128, TC_TILE, 0, 0);
    constexpr uint32_t IDESC_PV = idesc_f16(FMT, 128, D, 0, 1);
    constexpr int MAX_BLK = CHUNK_TC / 16 + 1;     // blocks a unit can touch
    constexpr int BPT = TC_TILE / 16;              // blocks per tile
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint32_t s_tmem;
    __shared__ int s_work, s_abort;
    __shared__ int s_blk[MAX_BLK];
    __shared__ __align__(8) uint64_t s_probe_bar;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool issuer = (warp >= TC_SOFTMAX_WARPS);
    const bool leader = warp == TC_SOFTMAX_WARPS && lane == 0;  // MMA issue
    const bool tma_warp = warp == TC_SOFTMAX_WARPS + 1;         // TMA issue
    const int my_rt = warp >> 2;                       // softmax warps: row tile
    const int my_row = (warp & 3) * 32 + lane;         // row within the tile = TMEM lane
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_kfull0 = sbase + TC_OFF_BAR;          // [KST] K tile landed
    const uint32_t bar_kempty0 = bar_kfull0 + 8 * TC_KST;    // [KST] K stage read by every row tile's Q K^T
    const uint32_t bar_vfull0 = bar_kempty0 + 8 * TC_KST;    // [VST] V tile landed
    const uint32_t bar_vempty0 = bar_vfull0 + 8 * TC_VST;    // [VST] V stage read by every row tile's P V
    const uint32_t bar_s0 = bar_vempty0 + 8 * TC_VST;        // [rt] S written (and the row tile's previous P V done)
    const uint32_t bar_p0 = bar_s0 + 16;                     // [rt] P stored by the row tile's four softmax warps
    const uint32_t bar_o0 = bar_p0 + 16;                     // [rt] the unit's last P V done
    const int Hkv = c.num_kv_heads, G = Hq / Hkv;

    for (int i = tid; i < TC_OFF_BAR / 16; i += TC_THREADS) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        for (int st = 0; st < TC_KST; ++st) {
            mbar_init(bar_kfull0 + 8 * st, 1);
            mbar_init(bar_kempty0 + 8 * st, 1);
        }
        for (int st = 0; st < TC_VST; ++st) {
            mbar_init(bar_vfull0 + 8 * st, 1);
            mbar_init(bar_vempty0 + 8 * st, 1);
        }
        for (int rt = 0; rt < TC_RT; ++rt) {
            mbar_init(bar_s0 + 8 * rt, 1);
            mbar_init(bar_p0 + 8 * rt, 4);  // one arrival per softmax warp of the row tile
            mbar_init(bar_o0 + 8 * rt, 1);
        }
        mbar_init(smem_u32(&s_probe_bar), 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(smem_u32(&s_tmem), TC_TMEM_COLS);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lane quarter
    // The set-up above overlaps the plan; the plan's units are read below.  The
    // narrow kernel after this one may start on the SMs this one leaves free.
    griddep_wait();
    griddep_launch();
    if (tid == 0 && !wait_probe(smem_u32(&s_probe_bar))) s_abort = 1;  // seen after the loop's first barrier
    TL_FIRST(4);
#ifdef MENTAT_TC_TRACE
    bool g_trace_on = false;  // the unit of work item 0
#endif
    // Barrier phases: the K/V rings count tiles (g0); row tile 0 counts every
    // tile and unit, row tile 1 only those of units with two row tiles.
    uint32_t g0 = 0, t1 = 0, u0 = 0, u1 = 0;
    uint32_t issued = 0;  // TMA warp: tiles whose copies have been issued
    const int nunits = ws.hdr[HDR_NTC];
    const int64_t nwork = (int64_t)nunits * Hkv;
    // a decode call's plan sets how many CTAs take units; the rest leave at once
    const bool idle = !PREFILL && (int)blockIdx.x >= ws.hdr[HDR_TC_CTAS];
    for (;;) {
        if (tid == 0) s_work = idle ? INT_MAX : atomicAdd(&ws.hdr[HDR_TC_NEXT], 1);
        __syncthreads();
        const int w = s_work;
        if (w >= nwork || s_abort) break;
#ifdef MENTAT_TC_TRACE
        g_trace_on = w == 0;
#endif
        TC_TRACE(0);
        const int u = w / Hkv, head = w % Hkv;
        const int32_t* U = ws.units_tc + (int64_t)u * UNIT_INTS;
        const int q_lo = U[0], q_hi = U[1], t0u = U[2], t1u = U[3], ord = U[4];
        const int R = (q_hi - q_lo + 1) * G;
        const int nrt = (R + 127) / 128;
        // prefill (causal_pos0 >= 0): every row reads the one sequence in slots[0]
        const int32_t* tab = table_row(c, layer, slots[causal_pos0 >= 0 ? 0 : q_lo]);
        const int blk0 = t0u / 16, blk_end = (t1u + 15) / 16;
        const int nblk = blk_end - blk0;  // <= MAX_BLK unless PREFILL
        const int ntiles = (nblk + BPT - 1) / BPT;

        // The TMA warp reads the unit's block ids and starts streaming K/V at
        // once; the other warps stage Q meanwhile (all loads in flight together)
        // and meet on named barrier 2 before the first MMA.
        if (tma_warp) {
            if constexpr (!PREFILL) {
                constexpr int PER_LANE = (MAX_BLK + 31) / 32;
                int b[PER_LANE];
#pragma unroll
                for (int k = 0; k < PER_LANE; ++k)
                    b[k] = lane + 32 * k < nblk ? checked_block(c, tab[blk0 + lane + 32 * k]) : 0;
#pragma unroll
                for (int k = 0; k < PER_LANE; ++k)
                    if (lane + 32 * k < nblk) s_blk[lane + 32 * k] = b[k];
                __syncwarp();
            }
        } else {
            constexpr int QCH = 2 * 128 * (D / 8);                  // 16-byte Q chunks of two row tiles
            constexpr int NQ = TC_THREADS - 32;                     // loading threads (TMA warp excluded)
            constexpr int QB = 16;                                  // loads in flight per thread (one round)
            const int qt = tid;  // 0 .. NQ-1: the TMA warp is the last warp
            const int nq = nrt * 128 * (D / 8);
#pragma unroll 1
            for (int base = 0; base < QCH; base += NQ * QB) {
                uint4 v[QB];
#pragma unroll
                for (int k = 0; k < QB; ++k) {
                    const int idx = base + qt + NQ * k, r = idx / (D / 8), ch = idx % (D / 8);
                    v[k] = make_uint4(0, 0, 0, 0);
                    if (idx < nq && r < R) {
                        const int seq = q_lo + r / G, g = r % G;
                        v[k] = *reinterpret_cast<const uint4*>(q + (int64_t)seq * q_stride + (int64_t)(head * G + g) * D +
                                                               ch * 8);
                    }
                }
#pragma unroll
                for (int k = 0; k < QB; ++k) {
                    const int idx = base + qt + NQ * k, r = idx / (D / 8), ch = idx % (D / 8);
                    if (idx < nq) {
                        const int rt = r >> 7, rr = r & 127, half = ch >> 3;
                        *reinterpret_cast<uint4*>(smem + TC_OFF_Q + (rt * 2 + half) * 16384 + sw128_off(rr, ch & 7)) = v[k];
                    }
                }
            }
            fence_proxy_async();
            bar_sync_id(2, TC_THREADS - 32);
        }
        TC_TRACE(1);
        auto rt_tile = [&](int rt) { return rt == 0 ? g0 : t1; };  // row tile's tile counter at the unit start
        auto rt_unit = [&](int rt) { return rt == 0 ? u0 : u1; };

        if (tma_warp) {
            // K(i) then V(i); a stage is reused once every row tile's MMA that read it is done
            int blk_next = 0;  // PREFILL: block ids one tile ahead
            if constexpr (PREFILL) blk_next = lane < min(BPT, nblk) ? checked_block(c, tab[blk0 + lane]) : 0;
            for (int i = 0; i < ntiles; ++i) {
                const uint32_t gi = g0 + i, ks = gi % TC_KST, vs = gi % TC_VST;
                const int nb = min(BPT, nblk - BPT * i);
                int blk;
                if constexpr (PREFILL) {
                    blk = blk_next;
                    const int nb2 = min(BPT, nblk - BPT * (i + 1));
                    blk_next = lane < nb2 ? checked_block(c, tab[blk0 + BPT * (i + 1) + lane]) : 0;
                } else {
                    blk = lane < nb ? s_blk[BPT * i + lane] : 0;
                }
                int ok = 1;
                if (lane == 0) {
                    if (gi >= TC_KST) ok = mbar_wait(bar_kempty0 + 8 * ks, ((gi / TC_KST) - 1) & 1);
                    if (ok) mbar_expect_tx(bar_kfull0 + 8 * ks, (uint32_t)(nb * HALVES * 2048));
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    s_abort = 1;
                    break;
                }
                if (lane < nb)
#pragma unroll
                    for (int h2 = 0; h2 < HALVES; ++h2)
                        tma_load_3d(sbase + TC_OFF_K + ks * TC_KV_TILE + h2 * (TC_TILE * 128) + lane * 2048, &tmap_k,
                                    bar_kfull0 + 8 * ks, h2 * 64, head, blk * 16);
                if (lane == 0) {
                    if (gi >= TC_VST) ok = mbar_wait(bar_vempty0 + 8 * vs, ((gi / TC_VST) - 1) & 1);
                    if (ok) mbar_expect_tx(bar_vfull0 + 8 * vs, (uint32_t)(nb * HALVES * 2048));
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    s_abort = 1;
                    ++issued;  // the K copies of this tile are in flight
                    break;
                }
                if (lane < nb)
#pragma unroll
                    for (int h2 = 0; h2 < HALVES; ++h2)
                        tma_load_3d(sbase + TC_OFF_V + vs * TC_KV_TILE + h2 * (TC_TILE * 128) + lane * 2048, &tmap_v,
                                    bar_vfull0 + 8 * vs, h2 * 64, head, blk * 16);
                ++issued;
            }
        }
        if (leader) {
            // base descriptors; a K step adds a constant to the start-address field
            // (16-byte units, no carry: shared memory addresses stay below 256 KB)
            const uint64_t qd0 = sdesc_sw128(sbase + TC_OFF_Q, 16, 1024);
            const uint64_t kd0 = sdesc_sw128(sbase + TC_OFF_K, 16, 1024);
            const uint64_t vd0 = sdesc_sw128(sbase + TC_OFF_V, TC_TILE * 128, 1024);
            auto issue_qk = [&](int rt, int i) {  // S[rt] = Q_rt K(i)^T
                const uint32_t g = g0 + i, ks = g % TC_KST;
                if (rt == 0 && !mbar_wait(bar_kfull0 + 8 * ks, (g / TC_KST) & 1)) {
                    s_abort = 1;
                    return;
                }
                tc_fence_after();
                const uint32_t d = tmem + rt * 256 + 128;
                const uint64_t qd = qd0 + (uint64_t)(rt * 2 * 16384 / 16);
                const uint64_t kd = kd0 + (uint64_t)(ks * TC_KV_TILE / 16);
                umma_ss<false>(d, qd, kd, IDESC_QK);
#pragma unroll
                for (int k = 1; k < D / 16; ++k)
                    umma_ss<true>(d, qd + (uint64_t)((k >> 2) * 1024 + (k & 3) * 2),
                                  kd + (uint64_t)((k >> 2) * (TC_TILE * 8) + (k & 3) * 2), IDESC_QK);
                umma_commit(bar_s0 + 8 * rt);
                if (rt == nrt - 1) umma_commit(bar_kempty0 + 8 * ks);
            };
            auto issue_pv = [&](int rt, int i) {  // O[rt] += P[rt] V(i)
                const uint32_t g = g0 + i, vs = g % TC_VST;
                if (rt == 0 && !mbar_wait(bar_vfull0 + 8 * vs, (g / TC_VST) & 1)) {
                    s_abort = 1;
                    return;
                }
                tc_fence_after();
                const uint32_t od = tmem + rt * 256, pa = tmem + rt * 256 + 128;
                const uint64_t vd = vd0 + (uint64_t)(vs * TC_KV_TILE / 16);
                umma_f16_ts(od, pa, vd, IDESC_PV, i > 0);
#pragma unroll
                for (int k = 1; k < TC_TILE / 16; ++k) umma_ts<true>(od, pa + k * 8, vd + (uint64_t)(k * 2048 / 16), IDESC_PV);
                if (PSPLIT && blk0 + BPT * i == 0) {  // P_lo of the sequence's first tile
#pragma unroll
                    for (int k = 0; k < TC_TILE / 16; ++k)
                        umma_ts<true>(od, pa + 64 + k * 8, vd + (uint64_t)(k * 2048 / 16), IDESC_PV);
                }
                if (i == ntiles - 1) umma_commit(bar_o0 + 8 * rt);
                if (rt == nrt - 1) umma_commit(bar_vempty0 + 8 * vs);
            };
            for (int rt = 0; rt < nrt; ++rt) issue_qk(rt, 0);
            for (int i = 0; i < ntiles && !s_abort; ++i) {
                TC_TRACE(64 + 8 * i);
                for (int rt = 0; rt < nrt && !s_abort; ++rt) {
                    if (!mbar_wait(bar_p0 + 8 * rt, (rt_tile(rt) + i) & 1)) {
                        s_abort = 1;
                        break;
                    }
                    TC_TRACE(65 + 8 * i + 3 * rt);
                    issue_pv(rt, i);
                    TC_TRACE(66 + 8 * i + 3 * rt);
                    if (i + 1 < ntiles) issue_qk(rt, i + 1);
                    TC_TRACE(67 + 8 * i + 3 * rt);
                }
            }
        }

        // softmax warps: row tile my_rt, thread = one query row (TMEM lane)
        float m_ref = -INFINITY, l_sum = 0.f;
        const bool wact = !issuer && my_rt < nrt;                                   // warp-uniform
        const bool rows_live = wact && (my_rt * 128 + (warp & 3) * 32 < R);        // warp-uniform
        const int row = my_rt * 128 + my_row;
        const uint32_t s_col = tmem + lane_off + my_rt * 256 + 128;
        const uint32_t o_col = tmem + lane_off + my_rt * 256;
        for (int i = 0; i < ntiles && wact; ++i) {
            const uint32_t t = rt_tile(my_rt) + i;
            TC_TRACE(64 + 8 * i);
            // warp-collective waits keep the warp converged for the .aligned TMEM accesses
            if (__any_sync(0xffffffffu, s_abort) || !__all_sync(0xffffffffu, mbar_wait(bar_s0 + 8 * my_rt, t & 1))) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
            TC_TRACE(65 + 8 * i);
            if (rows_live) {
                const int tb = (blk0 + BPT * i) * 16;  // first token of the tile
                // prefill: the row of query q_lo + r / G sees tokens up to causal_pos0 + that
                const int rp = causal_pos0 >= 0 ? causal_pos0 + q_lo + row / G : INT_MAX;
                const bool full = tb >= t0u && tb + TC_TILE <= t1u && tb + TC_TILE - 1 <= rp;
                // the row max is taken on raw scores (scale > 0 keeps the order) and the
                // scale is folded into the exponent's argument: p = 2^(s*scale - m_ref)
                auto valid = [&](int j) { return full || (tb + j >= t0u && tb + j < t1u && tb + j <= rp); };
                // MASKED: some token of the warp's rows is outside the unit's range or
                // (prefill) after the row's position; a warp whose rows see the whole
                // tile runs the copy without the per-score checks
                auto tile_body = [&](auto masked_c) {
                    constexpr bool MASKED = decltype(masked_c)::value;
                    // the tile's 128 scores in registers: one TMEM load and one wait; a
                    // masked score becomes -inf, whose probability 2^-inf is 0
                    float sv[TC_TILE];
                    tmem_ld128(s_col, sv);
                    if constexpr (MASKED) {
#pragma unroll
                        for (int j = 0; j < TC_TILE; ++j)
                            if (!valid(j)) sv[j] = -INFINITY;
                    }
                    float mxs[8];  // eight independent chains
#pragma unroll
                    for (int k = 0; k < 8; ++k) mxs[k] = -INFINITY;
#pragma unroll
                    for (int j = 0; j < TC_TILE; j += 2) mxs[(j >> 1) & 7] = fmax3(mxs[(j >> 1) & 7], sv[j], sv[j + 1]);
                    const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                                           fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
                    float fac = 1.f;
                    const float m_new = fmaxf(m_ref, mx * scale_log2);
                    if (m_ref == -INFINITY || m_new > m_ref + 8.f) {
                        if (m_ref != -INFINITY) {
                            fac = ex2_approx(m_ref - m_new);
                            l_sum *= fac;
                        }
                        m_ref = m_new;
                    }
                    // a row that has seen no token yet (prefill) keeps m = -inf and gets p = 0
                    const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
                    // rows whose reference max rose rescale O; S(i) being complete means
                    // P V(i-1) of this row tile is complete too (issued before S(i))
                    if (i > 0 && __any_sync(0xffffffffu, fac != 1.f)) {
                        const float f = row < R ? fac : 1.f;
#pragma unroll
                        for (int cb = 0; cb < D / 32; ++cb) {
                            float ov[32];
                            tmem_ld32(o_col + cb * 32, ov);
#pragma unroll
                            for (int k = 0; k < 32; ++k) ov[k] *= f;
                            tmem_st32(o_col + cb * 32, ov);
                        }
                    }
                    // P (pairs packed in one column: token t in column t / 2) over the S
                    // columns already in registers
                    float2 accs[4];  // four independent chains of pair sums
#pragma unroll
                    for (int k = 0; k < 4; ++k) accs[k] = make_float2(0.f, 0.f);
                    // SP: also P_lo, in columns 64 + t / 2 (prefill, first tile of the sequence)
                    auto write_p = [&](auto sp_c) {
                        constexpr bool SP = decltype(sp_c)::value;
#pragma unroll
                        for (int c = 0; c < TC_TILE / 32; ++c) {
                            uint32_t pk[16], pl[SP ? 16 : 1];
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                const int j = 32 * c + 2 * e;
                                const float2 x = ffma2(make_float2(sv[j], sv[j + 1]), make_float2(scale_log2, scale_log2),
                                                       make_float2(neg_m, neg_m));
                                const float a = ex2_approx(x.x);
                                const float b = ex2_approx(x.y);
                                accs[e & 3] = fadd2(accs[e & 3], make_float2(a, b));
                                pk[e] = Pair<T>::pack(a, b);
                                if constexpr (SP) pl[e] = Pair<T>::pack(a - Pair<T>::lo(pk[e]), b - Pair<T>::hi(pk[e]));
                            }
                            tmem_st16(s_col + 16 * c, pk);
                            if constexpr (SP) tmem_st16(s_col + 64 + 16 * c, pl);
                        }
                    };
                    if constexpr (PSPLIT) {
                        if (tb == 0)
                            write_p(std::true_type{});
                        else
                            write_p(std::false_type{});
                    } else {
                        write_p(std::false_type{});
                    }
                    tmem_st_wait();
                    l_sum += ((accs[0].x + accs[0].y) + (accs[1].x + accs[1].y)) +
                             ((accs[2].x + accs[2].y) + (accs[3].x + accs[3].y));
                };
                if (__all_sync(0xffffffffu, full))
                    tile_body(std::false_type{});
                else
                    tile_body(std::true_type{});
                TC_TRACE(66 + 8 * i);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_p0 + 8 * my_rt);
            TC_TRACE(67 + 8 * i);
        }
        // every thread reaches this CTA-wide barrier, so the abort decision is uniform
        if (__syncthreads_or(s_abort)) {
            s_abort = 1;
            break;
        }
        // the unit's last P V of this row tile done -> partials of this thread's row
        if (rows_live) {
            if (!__all_sync(0xffffffffu, mbar_wait(bar_o0 + 8 * my_rt, rt_unit(my_rt) & 1))) s_abort = 1;
            tc_fence_after();
            const int seq = q_lo + row / G, hq = head * G + row % G;
            const int64_t pi = ((int64_t)seq * max_parts + ord) * Hq + hq;
            // a prefill query group with one unit (one partial): O / l, rounded to T,
            // straight to out, 16 bytes per store
            if (PREFILL && out != nullptr && ws.nparts[q_lo] == 1) {
                const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
                T* dst = out + (int64_t)seq * out_stride + (int64_t)hq * D;
#pragma unroll
                for (int cb = 0; cb < D / 32; ++cb) {
                    float ov[32];
                    tmem_ld32(o_col + cb * 32, ov);
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) pk[e] = Pair<T>::pack(ov[2 * e] * inv, ov[2 * e + 1] * inv);
                    if (row < R)
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            reinterpret_cast<uint4*>(dst + cb * 32)[k] =
                                make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
                }
            } else {
                // O goes out through shared memory: each thread writes its row to the (now
                // idle) K/V ring with a 16-byte pad per row (the 32 rows of a warp land in
                // distinct banks), then one bulk copy per row moves it to the workspace
                constexpr uint32_t OROW = D * 4 + 16;
                const uint32_t orow = TC_OFF_K + (uint32_t)(my_rt * 128 + my_row) * OROW;
#pragma unroll
                for (int cb = 0; cb < D / 32; ++cb) {
                    float ov[32];
                    tmem_ld32(o_col + cb * 32, ov);
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        *reinterpret_cast<float4*>(smem + orow + cb * 128 + k * 16) =
                            make_float4(ov[4 * k], ov[4 * k + 1], ov[4 * k + 2], ov[4 * k + 3]);
                }
                if (row < R) {
                    fence_proxy_async();  // the row's generic writes before the bulk copy reads them
                    bulk_store(ws.part_o + pi * D, sbase + orow, D * 4);
                    ws.part_ml[pi * 2] = m_ref;
                    ws.part_ml[pi * 2 + 1] = l_sum;
                    bulk_wait_read();     // the ring is free again before the next unit streams into it
                }
                // A later unit's partial tile leaves the V rows of its missing blocks as they
                // were, and P V multiplies them by zero probabilities: they must hold finite
                // values, which fp32 O bits read as bf16 need not be.  Rows staged over the V
                // ring are cleared (K rows of missing blocks are masked before the softmax).
                if (orow + OROW > (uint32_t)TC_OFF_V) {
#pragma unroll
                    for (int k = 0; k < (int)OROW / 16; ++k)
                        *reinterpret_cast<uint4*>(smem + orow + k * 16) = make_uint4(0, 0, 0, 0);
                }
            }
        } else if (leader) {
            // the unit's last P V must be complete before the next unit's first MMA overwrites O
            for (int rt = 0; rt < nrt; ++rt)
                if (!mbar_wait(bar_o0 + 8 * rt, rt_unit(rt) & 1)) s_abort = 1;
        }
        TC_TRACE(4);
#ifdef MENTAT_TC_TRACE
        g_trace_on = false;
#endif
        g0 += ntiles;
        u0 += 1;
        if (nrt > 1) {
            t1 += ntiles;
            u1 += 1;
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    // teardown: the partials' bulk stores complete; on abort, drain the copies still in
    // flight (bounded) before the smem goes away
    bulk_wait_all();
    __syncthreads();
    if (s_abort) {
        if (leader) {
            atomicExch(&ws.hdr[HDR_TC_ABORT], 1);
            set_error(c, MENTAT_DEV_DECODE_TIMEOUT, 1);  // also when no merge runs after this kernel
        }
        if (tma_warp && lane == 0) {
            // at most KST K tiles and VST V tiles can be issued and not yet waited for
            for (uint32_t k = issued > TC_KST ? issued - TC_KST : 0; k < issued; ++k)
                (void)mbar_wait(bar_kfull0 + 8 * (k % TC_KST), (k / TC_KST) & 1);
            for (uint32_t k = issued > TC_VST ? issued - TC_VST : 0; k < issued; ++k)
                (void)mbar_wait(bar_vfull0 + 8 * (k % TC_VST), (k / TC_VST) & 1);
        }
        __syncthreads();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TC_TMEM_COLS);
    TL_LAST(5);
    TL_CTA_END(0);
}

// ---------------------------------------------------------------------------
// host: tensor maps of a layer's K and V pools (cached per pool and layer)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

struct PoolMaps {
    const void* k_pool;
    const void* v_pool;
    int layer, num_blocks, kv_heads, head_dim, dtype, device;
    CUtensorMap mk, mv;
};

static bool make_pool_map(CUtensorMap* m, const mentat_kv_cache* c, const void* pool, int layer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const int esz = dtype_bytes(c->dtype);
    const int64_t layer_bytes = (int64_t)c->num_blocks * c->block_size * c->num_kv_heads * c->head_dim * esz;
    void* base = (char*)pool + layer * layer_bytes;
    cuuint64_t dims[3] = {(cuuint64_t)c->head_dim, (cuuint64_t)c->num_kv_heads,
                          (cuuint64_t)c->num_blocks * c->block_size};
    cuuint64_t strides[2] = {(cuuint64_t)c->head_dim * esz, (cuuint64_t)c->num_kv_heads * c->head_dim * esz};
    cuuint32_t box[3] = {64, 1, 16};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt =
        c->dtype == MENTAT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return fn(m, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static const PoolMaps* pool_maps(const mentat_kv_cache* c, int layer) {
    constexpr int CAP = 256;
    static PoolMaps cache[CAP];
    static int used = 0, next = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    for (int i = 0; i < used; ++i) {
        const PoolMaps& e = cache[i];
        if (e.k_pool == c->k_pool && e.v_pool == c->v_pool && e.layer == layer && e.num_blocks == c->num_blocks &&
            e.kv_heads == c->num_kv_heads && e.head_dim == c->head_dim && e.dtype == c->dtype && e.device == dev)
            return &e;
    }
    PoolMaps e;
    e.k_pool = c->k_pool;
    e.v_pool = c->v_pool;
    e.layer = layer;
    e.num_blocks = c->num_blocks;
    e.kv_heads = c->num_kv_heads;
    e.head_dim = c->head_dim;
    e.dtype = c->dtype;
    e.device = dev;
    if (!make_pool_map(&e.mk, c, c->k_pool, layer) || !make_pool_map(&e.mv, c, c->v_pool, layer)) return nullptr;
    const int slot = used < CAP ? used++ : (next++ % CAP);
    cache[slot] = e;
    return &cache[slot];
}

// whether the tensor-core kernel supports this cache layout
static bool tc_supported(const mentat_kv_cache* c) {
    return (c->dtype == MENTAT_BF16 || c->dtype == MENTAT_F16) && (c->head_dim == 64 || c->head_dim == 128) &&
           c->block_size == 16 && c->num_kv_heads * c->head_dim * dtype_bytes(c->dtype) % 16 == 0;
}

}  // namespace mentat
