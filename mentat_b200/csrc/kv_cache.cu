// Device-resident block allocator, sequence tables, fork / free / append with
// copy-on-write, sliding-window trim and packed gather.
//
// Semantics follow core/paged_kv_cache.py of the reference; the free list is a
// FIFO ring (pop oldest, push newest) of block ids.  All allocator state lives
// in device memory so that a decode step needs no host round trip; errors go
// to ctrl[MENTAT_CTRL_ERROR] and every kernel becomes a no-op once it is set.

#include "common.cuh"

namespace mentat {

// ---------------------------------------------------------------------------
// init / reset
// ---------------------------------------------------------------------------
__global__ void k_init(mentat_kv_cache c, const int32_t* order) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < c.num_blocks) {
        c.refcounts[i] = 0;
        c.free_ring[i] = order ? order[i] : (int32_t)i;
    }
    if (i < MENTAT_CTRL_WORDS) c.ctrl[i] = (i == MENTAT_CTRL_TAIL) ? c.num_blocks : 0;
}

__global__ void k_seq_reset(mentat_kv_cache c, int slot) {
    int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l < c.num_layers) {
        int64_t si = seq_index(c, l, slot);
        c.nblocks[si] = 0;
        c.ntok[si] = 0;
        c.tail[si] = 0;
    }
}

// ---------------------------------------------------------------------------
// fork: copy tables, ref() every block (paged_kv_cache.py:152-170)
// ---------------------------------------------------------------------------
__global__ void k_fork(mentat_kv_cache c, int parent, int child) {
    if (has_error(c)) return;
    const int l = blockIdx.y;
    const int64_t ps = seq_index(c, l, parent), cs = seq_index(c, l, child);
    const int nb = c.nblocks[ps];
    const int32_t* src = table_row(c, l, parent);
    int32_t* dst = table_row(c, l, child);
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < nb; j += gridDim.x * blockDim.x) {
        int b = src[j];
        dst[j] = b;
        int old = atomicAdd(&c.refcounts[b], 1);
        if (old <= 0) set_error(c, MENTAT_DEV_REF_FREE, b);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        c.nblocks[cs] = nb;
        c.ntok[cs] = c.ntok[ps];
        c.tail[cs] = c.tail[ps];
    }
}

// ---------------------------------------------------------------------------
// free: release() every block in layer-major table order; zero-hits join the
// FIFO in that order (paged_kv_cache.py:172-176, 62-66)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_free(mentat_kv_cache c, int slot) {
    __shared__ int smem32[32];
    __shared__ long long s_tail;
    if (has_error(c)) return;
    if (threadIdx.x == 0) s_tail = c.ctrl[MENTAT_CTRL_TAIL];
    __syncthreads();
    const int cap = c.num_blocks;
    for (int l = 0; l < c.num_layers; ++l) {
        const int64_t si = seq_index(c, l, slot);
        const int nb = c.nblocks[si];
        const int32_t* row = table_row(c, l, slot);
        for (int base = 0; base < nb; base += blockDim.x) {
            const int j = base + threadIdx.x;
            int b = -1, zero = 0;
            if (j < nb) {
                b = row[j];
                int old = atomicSub(&c.refcounts[b], 1);
                if (old <= 0) {
                    atomicAdd(&c.refcounts[b], 1);
                    set_error(c, MENTAT_DEV_RELEASE_FREE, b);
                } else if (old == 1) {
                    zero = 1;
                }
            }
            int total;
            int pos = block_exclusive_scan(zero, &total, smem32);
            if (zero) c.free_ring[(s_tail + pos) % cap] = b;
            __syncthreads();
            if (threadIdx.x == 0) s_tail += total;
            __syncthreads();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            c.nblocks[si] = 0;
            c.ntok[si] = 0;
            c.tail[si] = 0;
        }
    }
    if (threadIdx.x == 0) c.ctrl[MENTAT_CTRL_TAIL] = s_tail;
}

// ---------------------------------------------------------------------------
// allocation helpers (one thread)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ring_at(const mentat_kv_cache& c, long long head, int k) {
    return c.free_ring[(head + k) % c.num_blocks];
}
__device__ __forceinline__ void note_allocs(const mentat_kv_cache& c, int count, int cows) {
    long long head = c.ctrl[MENTAT_CTRL_HEAD] + count;
    c.ctrl[MENTAT_CTRL_HEAD] = head;
    long long used = c.num_blocks - (c.ctrl[MENTAT_CTRL_TAIL] - head);
    if (used > c.ctrl[MENTAT_CTRL_PEAK]) c.ctrl[MENTAT_CTRL_PEAK] = used;
    c.ctrl[MENTAT_CTRL_ALLOCS] += count;
    c.ctrl[MENTAT_CTRL_COWS] += cows;
}
// single-thread alloc with the reference's exact order of effects (:45-56)
__device__ __forceinline__ int alloc_one(const mentat_kv_cache& c) {
    long long head = c.ctrl[MENTAT_CTRL_HEAD], tail = c.ctrl[MENTAT_CTRL_TAIL];
    if (tail - head <= 0) {
        set_error(c, MENTAT_DEV_OUT_OF_BLOCKS, c.num_blocks);
        return -1;
    }
    int b = ring_at(c, head, 0);
    c.refcounts[b] = 1;
    note_allocs(c, 1, 0);
    return b;
}
__device__ __forceinline__ void release_one(const mentat_kv_cache& c, int b) {
    int r = c.refcounts[b];
    if (r <= 0) {
        set_error(c, MENTAT_DEV_RELEASE_FREE, b);
        return;
    }
    c.refcounts[b] = r - 1;
    if (r == 1) {
        long long tail = c.ctrl[MENTAT_CTRL_TAIL];
        c.free_ring[tail % c.num_blocks] = b;
        c.ctrl[MENTAT_CTRL_TAIL] = tail + 1;
    }
}

// scratch of the batched append: [0] mode (0 parallel, 1 sequential, 2 skip),
// then dst block, dst slot and CoW source (-1: none) per batch entry
struct AppendScratch {
    int32_t* mode;
    int32_t* dst_blk;
    int32_t* dst_slot;
    int32_t* cow_src;
    __device__ AppendScratch(const mentat_kv_cache& c) {
        mode = c.scratch;
        dst_blk = c.scratch + 8;
        dst_slot = dst_blk + c.max_seqs;
        cow_src = dst_slot + c.max_seqs;
    }
};

// Sequential reference semantics for one decode token of entry i (used when a
// slot repeats inside a batch).
__device__ void append_one_seq(const mentat_kv_cache& c, int layer, int slot, AppendScratch& sc, int i) {
    const int64_t si = seq_index(c, layer, slot);
    int32_t* row = table_row(c, layer, slot);
    int nb = c.nblocks[si], tf = c.tail[si];
    sc.cow_src[i] = -1;
    if (nb == 0 || tf == c.block_size) {
        if (nb >= c.max_blocks_per_seq) {
            set_error(c, MENTAT_DEV_TABLE_OVERFLOW, slot);
            return;
        }
        int b = alloc_one(c);
        if (b < 0) return;
        row[nb++] = b;
        c.nblocks[si] = nb;
        tf = 0;
    }
    int t = row[nb - 1];
    if (c.refcounts[t] > 1) {
        int b = alloc_one(c);
        if (b < 0) return;
        sc.cow_src[i] = t;
        release_one(c, t);
        row[nb - 1] = b;
        t = b;
        c.ctrl[MENTAT_CTRL_COWS] += 1;
    }
    sc.dst_blk[i] = t;
    sc.dst_slot[i] = tf;
    c.tail[si] = tf + 1;
    c.ntok[si] += 1;
}

// ---------------------------------------------------------------------------
// batched decode append, planning (paged_kv_cache.py:246-274); one CTA.
// Entries sharing a tail block are ranked in batch order: the c-th of them
// copies iff refcount - c > 1, exactly as the reference's sequential loop.
// Allocations are numbered by an exclusive scan, so pop order is batch order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_append_plan(mentat_kv_cache c, int layer, const int32_t* slots, int n) {
    extern __shared__ int sm[];
    int* s_slot = sm;      // [n]
    int* s_tblk = sm + n;  // [n] tail block, -1 when a new block is needed
    __shared__ int smem32[32];
    __shared__ int s_abort;
    __shared__ long long s_head;
    griddep_wait();  // the stream's previous work (tables, lengths, slots)
    griddep_launch();
    AppendScratch sc(c);
    if (threadIdx.x == 0) s_abort = has_error(c) ? 1 : 0;
    __syncthreads();
    if (s_abort) {
        if (threadIdx.x == 0) sc.mode[0] = 2;
        return;
    }
    const int i = threadIdx.x;
    int slot = -1, nb = 0, tf = 0, tblk = -1;
    // slot -1 marks a padding entry (a batch padded to a captured size): skipped
    const bool valid = i < n && slots[i] != -1;
    if (i < n && !valid) {
        s_slot[i] = -1;
        s_tblk[i] = -1;
        sc.dst_blk[i] = -1;
    }
    if (valid) {
        slot = slots[i];
        if (slot < 0 || slot >= c.max_seqs) {
            set_error(c, MENTAT_DEV_TABLE_OVERFLOW, slot);
            slot = 0;
        }
        const int64_t si = seq_index(c, layer, slot);
        nb = c.nblocks[si];
        tf = c.tail[si];
        if (!(nb == 0 || tf == c.block_size)) tblk = table_row(c, layer, slot)[nb - 1];
        s_slot[i] = slot;
        s_tblk[i] = tblk;
    }
    __syncthreads();
    int dup = 0;  // a repeated slot needs the sequential path
    if (valid)
        for (int j = 0; j < i; ++j) dup |= (s_slot[j] == slot);
    dup = __syncthreads_or(dup);
    if (has_error(c)) dup = 2;
    if (dup) {
        if (threadIdx.x == 0) {
            sc.mode[0] = 1;
            if (dup == 1)
                for (int k = 0; k < n && !has_error(c); ++k)
                    if (s_slot[k] >= 0) append_one_seq(c, layer, s_slot[k], sc, k);
            if (has_error(c)) sc.mode[0] = 2;
        }
        return;
    }
    int rank = 0, r0 = 0;
    if (valid && tblk >= 0) {
        for (int j = 0; j < i; ++j) rank += (s_tblk[j] == tblk);
        r0 = c.refcounts[tblk];
    }
    const bool need_new = valid && tblk < 0;
    const bool cow = valid && tblk >= 0 && (r0 - rank > 1);
    const int want = (need_new || cow) ? 1 : 0;
    int total;
    const int a = block_exclusive_scan(want, &total, smem32);
    if (threadIdx.x == 0) {
        s_head = c.ctrl[MENTAT_CTRL_HEAD];
        long long avail = c.ctrl[MENTAT_CTRL_TAIL] - s_head;
        s_abort = 0;
        if (total > avail) {
            set_error(c, MENTAT_DEV_OUT_OF_BLOCKS, c.num_blocks);
            s_abort = 1;
        }
    }
    __syncthreads();
    if (s_abort) {
        if (threadIdx.x == 0) sc.mode[0] = 2;
        return;
    }
    if (valid) {
        const int64_t si = seq_index(c, layer, slot);
        int32_t* row = table_row(c, layer, slot);
        int dst = tblk, dslot = tf, src = -1;
        if (want) {
            dst = ring_at(c, s_head, a);
            c.refcounts[dst] = 1;
        }
        if (need_new) {
            if (nb >= c.max_blocks_per_seq) {
                set_error(c, MENTAT_DEV_TABLE_OVERFLOW, slot);
            } else {
                row[nb] = dst;
                c.nblocks[si] = nb + 1;
            }
            dslot = 0;
        } else if (cow) {
            atomicSub(&c.refcounts[tblk], 1);
            row[nb - 1] = dst;
            src = tblk;
        }
        sc.dst_blk[i] = dst;
        sc.dst_slot[i] = dslot;
        sc.cow_src[i] = src;
        c.tail[si] = dslot + 1;
        c.ntok[si] += 1;
    }
    const int ncow = __syncthreads_count(cow);
    if (threadIdx.x == 0) {
        note_allocs(c, total, ncow);
        sc.mode[0] = has_error(c) ? 2 : 0;
    }
}

// data movement of the batched append: CoW copy of the whole block, then the token row
__global__ void k_append_data(mentat_kv_cache c, int layer, int n, const uint8_t* k, int64_t k_sb,
                              const uint8_t* v, int64_t v_sb) {
    griddep_wait();  // the plan's scratch (and, through it, the K/V rows' producers)
    griddep_launch();
    AppendScratch sc(c);
    const int mode = sc.mode[0];
    if (mode == 2) return;
    const int esz = dtype_bytes(c.dtype);
    const int64_t row_bytes = (int64_t)c.num_kv_heads * c.head_dim * esz;
    const int64_t blk_bytes = row_bytes * c.block_size;
    uint8_t* kp = reinterpret_cast<uint8_t*>(c.k_pool);
    uint8_t* vp = reinterpret_cast<uint8_t*>(c.v_pool);
    int lo = blockIdx.x, hi = blockIdx.x + 1;
    if (mode == 1) {  // sequential: CTA 0 walks the batch in order
        if (blockIdx.x != 0) return;
        lo = 0;
        hi = n;
    }
    for (int i = lo; i < hi; ++i) {
        const int dst = sc.dst_blk[i], slot = sc.dst_slot[i], src = sc.cow_src[i];
        if (dst < 0) continue;  // padding entry (uniform across the CTA)
        if (src >= 0) {
            block_copy_bytes(kp + pool_row(c, layer, dst, 0) * esz, kp + pool_row(c, layer, src, 0) * esz, blk_bytes);
            block_copy_bytes(vp + pool_row(c, layer, dst, 0) * esz, vp + pool_row(c, layer, src, 0) * esz, blk_bytes);
            __syncthreads();
        }
        block_copy_bytes(kp + pool_row(c, layer, dst, slot) * esz, k + i * k_sb, row_bytes);
        block_copy_bytes(vp + pool_row(c, layer, dst, slot) * esz, v + i * v_sb, row_bytes);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// multi-token append for one sequence (paged_kv_cache.py:178-225)
// scratch: [0] mode, [1] CoW src, [2] CoW dst, [3] old ntok, [4] tokens that go
// into the CoW'd block.  Only the first chunk can copy: later chunks get fresh
// (unshared) blocks.
// ---------------------------------------------------------------------------
// The reference's loop (:196-222) allocates in this order: a copy of a shared,
// partially filled tail block on the first chunk (the only chunk whose tail can
// be shared: later blocks are fresh), then one fresh block per further
// bs tokens.  Those are consecutive pops of the free FIFO, so thread 0 settles
// the copy and the counts and the CTA fills the fresh table entries at once.
constexpr int MULTI_PLAN_THREADS = 256;
__global__ void __launch_bounds__(MULTI_PLAN_THREADS) k_append_multi_plan(mentat_kv_cache c, int layer, int slot,
                                                                          int n) {
    __shared__ int s_nb, s_fresh, s_pop0, s_stop;
    __shared__ long long s_head;
    int32_t* sc = c.scratch;
    const int64_t si = seq_index(c, layer, slot);
    int32_t* row = table_row(c, layer, slot);
    const int bs = c.block_size;
    if (threadIdx.x == 0) {
        s_stop = 1;
        sc[0] = 0;
        sc[1] = -1;
        sc[2] = -1;
        sc[3] = c.ntok[si];
        sc[4] = 0;
        const int nb = c.nblocks[si], tf = c.tail[si];
        const int room = (nb > 0 && tf < bs) ? bs - tf : 0;  // rows left in the current tail block
        const int t = nb > 0 ? row[nb - 1] : -1;
        const int cow = (n > 0 && room > 0 && c.refcounts[t] > 1) ? 1 : 0;
        const int rest = n - min(n, room);
        const int fresh = (rest + bs - 1) / bs;
        const long long head = c.ctrl[MENTAT_CTRL_HEAD], tail = c.ctrl[MENTAT_CTRL_TAIL];
        if (has_error(c)) {
            sc[0] = 2;
        } else if (nb + fresh > c.max_blocks_per_seq) {
            set_error(c, MENTAT_DEV_TABLE_OVERFLOW, slot);
            sc[0] = 2;
        } else if (tail - head < cow + fresh) {
            set_error(c, MENTAT_DEV_OUT_OF_BLOCKS, c.num_blocks);
            sc[0] = 2;
        } else if (n > 0) {
            if (cow) {
                const int b = ring_at(c, head, 0);
                c.refcounts[b] = 1;
                release_one(c, t);  // still referenced elsewhere: never freed here
                row[nb - 1] = b;
                sc[1] = t;
                sc[2] = b;
                sc[4] = min(room, n);
            }
            note_allocs(c, cow + fresh, cow);
            c.nblocks[si] = nb + fresh;
            c.tail[si] = fresh ? rest - (fresh - 1) * bs : tf + n;
            c.ntok[si] += n;
            s_nb = nb;
            s_fresh = fresh;
            s_pop0 = cow;
            s_head = head;
            s_stop = 0;
        }
    }
    __syncthreads();
    if (s_stop) return;
    for (int j = threadIdx.x; j < s_fresh; j += blockDim.x) {
        const int b = ring_at(c, s_head, s_pop0 + j);
        c.refcounts[b] = 1;
        row[s_nb + j] = b;
    }
}

// CTA 0 owns the CoW'd block (copy first, then its tokens) so the copy cannot
// overwrite new rows; the other CTAs scatter the remaining token rows.
__global__ void k_append_multi_data(mentat_kv_cache c, int layer, int slot, int n, const uint8_t* k,
                                    int64_t k_sb, const uint8_t* v, int64_t v_sb) {
    const int32_t* sc = c.scratch;
    if (sc[0] == 2) return;
    const int esz = dtype_bytes(c.dtype);
    const int64_t row_bytes = (int64_t)c.num_kv_heads * c.head_dim * esz;
    uint8_t* kp = reinterpret_cast<uint8_t*>(c.k_pool);
    uint8_t* vp = reinterpret_cast<uint8_t*>(c.v_pool);
    const int32_t* row = table_row(c, layer, slot);
    const int cow_src = sc[1], cow_dst = sc[2], p0 = sc[3], first_n = sc[4];
    const int bs = c.block_size;
    if (cow_src >= 0 && blockIdx.x == 0) {
        block_copy_bytes(kp + pool_row(c, layer, cow_dst, 0) * esz, kp + pool_row(c, layer, cow_src, 0) * esz,
                         row_bytes * bs);
        block_copy_bytes(vp + pool_row(c, layer, cow_dst, 0) * esz, vp + pool_row(c, layer, cow_src, 0) * esz,
                         row_bytes * bs);
        __syncthreads();
        for (int w = 0; w < first_n; ++w) {
            const int p = p0 + w;
            const int b = row[p / bs];
            block_copy_bytes(kp + pool_row(c, layer, b, p % bs) * esz, k + w * k_sb, row_bytes);
            block_copy_bytes(vp + pool_row(c, layer, b, p % bs) * esz, v + w * v_sb, row_bytes);
        }
        return;
    }
    const int nworkers = gridDim.x - (cow_src >= 0 ? 1 : 0);
    const int wid = blockIdx.x - (cow_src >= 0 ? 1 : 0);
    for (int w = first_n + wid; w < n; w += nworkers) {
        const int p = p0 + w;
        const int b = row[p / bs];
        block_copy_bytes(kp + pool_row(c, layer, b, p % bs) * esz, k + w * k_sb, row_bytes);
        block_copy_bytes(vp + pool_row(c, layer, b, p % bs) * esz, v + w * v_sb, row_bytes);
    }
}

// ---------------------------------------------------------------------------
// trim_to_window (paged_kv_cache.py:370-417), one CTA, rare
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_trim(mentat_kv_cache c, int slot, int window) {
    __shared__ int s_move[4];  // src block, src offset, dst block, rows kept (or -1)
    __shared__ int s_stop;
    if (threadIdx.x == 0) s_stop = has_error(c) ? 1 : 0;
    __syncthreads();
    if (s_stop) return;
    if (c.ntok[seq_index(c, 0, slot)] <= window) return;
    const int bs = c.block_size;
    const int esz = dtype_bytes(c.dtype);
    const int64_t row_bytes = (int64_t)c.num_kv_heads * c.head_dim * esz;
    uint8_t* pools[2] = {reinterpret_cast<uint8_t*>(c.k_pool), reinterpret_cast<uint8_t*>(c.v_pool)};
    for (int l = 0; l < c.num_layers; ++l) {
        const int64_t si = seq_index(c, l, slot);
        if (threadIdx.x == 0) {
            s_move[3] = -1;
            int32_t* row = table_row(c, l, slot);
            int nb = c.nblocks[si];
            int rem = c.ntok[si] - window;
            while (rem > 0 && nb > 0) {
                int b = row[0];
                int cnt = min(bs, rem);
                if (cnt >= bs) {
                    for (int j = 1; j < nb; ++j) row[j - 1] = row[j];
                    --nb;
                    release_one(c, b);
                    rem -= bs;
                } else {
                    int keep = bs - cnt;
                    if (c.refcounts[b] > 1) {
                        int nbk = alloc_one(c);
                        if (nbk < 0) break;
                        s_move[0] = b; s_move[1] = cnt; s_move[2] = nbk; s_move[3] = keep;
                        release_one(c, b);
                        row[0] = nbk;
                    } else {
                        s_move[0] = b; s_move[1] = cnt; s_move[2] = b; s_move[3] = keep;
                    }
                    rem = 0;
                }
            }
            c.nblocks[si] = nb;
            c.ntok[si] = window;
            int t = window % bs;
            c.tail[si] = window == 0 ? 0 : (t ? t : bs);
            if (has_error(c)) s_stop = 1;
        }
        __syncthreads();
        if (s_stop) return;
        if (s_move[3] > 0) {
            // row r of dst <- row r + off of src, in increasing r (safe in place)
            for (int r = 0; r < s_move[3]; ++r) {
                for (int p = 0; p < 2; ++p)
                    block_copy_bytes(pools[p] + pool_row(c, l, s_move[2], r) * esz,
                                     pools[p] + pool_row(c, l, s_move[0], r + s_move[1]) * esz, row_bytes);
                __syncthreads();
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// packed gather for PagedKV.materialize (paged_kv_cache.py:347-359)
// ---------------------------------------------------------------------------
__global__ void k_gather(mentat_kv_cache c, int layer, const int32_t* slots, int n, const int32_t* cu,
                         int64_t total, uint8_t* ok, uint8_t* ov) {
    const int esz = dtype_bytes(c.dtype);
    const int64_t row_bytes = (int64_t)c.num_kv_heads * c.head_dim * esz;
    for (int64_t p = blockIdx.x; p < total; p += gridDim.x) {
        int lo = 0, hi = n - 1;  // last i with cu[i] <= p
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (cu[mid] <= p) lo = mid; else hi = mid - 1;
        }
        const int t = (int)(p - cu[lo]);
        const int b = table_row(c, layer, slots[lo])[t / c.block_size];
        if ((unsigned)b >= (unsigned)c.num_blocks) {  // a corrupt table entry: recorded, the row left as is
            if (threadIdx.x == 0) set_error(c, MENTAT_DEV_BAD_BLOCK, b);
            continue;
        }
        const int64_t off = pool_row(c, layer, b, t % c.block_size) * esz;
        block_copy_bytes(ok + p * row_bytes, reinterpret_cast<uint8_t*>(c.k_pool) + off, row_bytes);
        block_copy_bytes(ov + p * row_bytes, reinterpret_cast<uint8_t*>(c.v_pool) + off, row_bytes);
    }
}

}  // namespace mentat

using namespace mentat;

static bool bad_cache(const mentat_kv_cache* c) {
    return !c || c->num_layers <= 0 || c->num_blocks <= 0 || c->block_size <= 0 || c->max_seqs <= 0 ||
           c->max_blocks_per_seq <= 0 || !c->refcounts || !c->free_ring || !c->ctrl || !c->tables ||
           !c->nblocks || !c->ntok || !c->tail || !c->scratch;
}

extern "C" {

int64_t mentat_kernel_launch_count(void) { return (int64_t)mentat::g_kernel_launches.load(std::memory_order_relaxed); }


int mentat_abi_version(void) { return MENTAT_ABI_VERSION; }

const char* mentat_status_string(int s) {
    switch (s) {
        case MENTAT_OK: return "ok";
        case MENTAT_ERR_ARG: return "invalid argument";
        case MENTAT_ERR_CUDA: return "CUDA launch failed";
        case MENTAT_ERR_UNSUPPORTED: return "unsupported shape or dtype";
        case MENTAT_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of the no-allocation entry point";
        case MENTAT_DEV_OUT_OF_BLOCKS: return "out of blocks";
        case MENTAT_DEV_REF_FREE: return "ref() on free block";
        case MENTAT_DEV_RELEASE_FREE: return "release() on free block";
        case MENTAT_DEV_PLAN_OVERFLOW: return "decode plan workspace overflow";
        case MENTAT_DEV_TABLE_OVERFLOW: return "sequence table overflow";
        case MENTAT_DEV_DECODE_TIMEOUT: return "a bounded wait in a decode kernel gave up";
        case MENTAT_DEV_BAD_BLOCK: return "block table entry outside the pool";
        default: return "unknown status";
    }
}

int64_t mentat_kv_scratch_ints(int32_t max_seqs) { return 8 + 3 * (int64_t)max_seqs + 8; }

int mentat_kv_init(const mentat_kv_cache* c, const int32_t* order, cudaStream_t s) {
    if (bad_cache(c)) return MENTAT_ERR_ARG;
    int n = c->num_blocks > MENTAT_CTRL_WORDS ? c->num_blocks : MENTAT_CTRL_WORDS;
    k_init<<<(n + 255) / 256, 256, 0, s>>>(*c, order);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_seq_reset(const mentat_kv_cache* c, int32_t slot, cudaStream_t s) {
    if (bad_cache(c) || slot < 0 || slot >= c->max_seqs) return MENTAT_ERR_ARG;
    k_seq_reset<<<(c->num_layers + 127) / 128, 128, 0, s>>>(*c, slot);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_fork(const mentat_kv_cache* c, int32_t parent, int32_t child, int32_t max_nb, cudaStream_t s) {
    if (bad_cache(c) || parent < 0 || parent >= c->max_seqs || child < 0 || child >= c->max_seqs ||
        parent == child || max_nb < 0)
        return MENTAT_ERR_ARG;
    int gx = (max_nb + 255) / 256;
    if (gx < 1) gx = 1;
    if (gx > 64) gx = 64;
    dim3 grid(gx, c->num_layers);
    k_fork<<<grid, 256, 0, s>>>(*c, parent, child);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_free(const mentat_kv_cache* c, int32_t slot, int32_t max_nb, cudaStream_t s) {
    (void)max_nb;
    if (bad_cache(c) || slot < 0 || slot >= c->max_seqs) return MENTAT_ERR_ARG;
    k_free<<<1, 1024, 0, s>>>(*c, slot);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_append_batched(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                             const void* k, int64_t k_stride, const void* v, int64_t v_stride, cudaStream_t s) {
    if (bad_cache(c) || layer < 0 || layer >= c->num_layers || n < 0 || n > 1024 || n > c->max_seqs ||
        (n > 0 && (!slots || !k || !v)) || !c->k_pool || !c->v_pool)
        return MENTAT_ERR_ARG;
    if (n == 0) return MENTAT_OK;
    const int esz = dtype_bytes(c->dtype);
    int threads = ((n + 31) / 32) * 32;
    // both go out with programmatic stream serialization, so their launches overlap
    // the work ahead of them; each waits for its predecessor before touching memory
    const bool pdl = pdl_enabled();
    if (launch(pdl, k_append_plan, dim3(1), dim3(threads), 2 * n * sizeof(int), s, *c, layer, slots, n) !=
        cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    if (launch(pdl, k_append_data, dim3(n), dim3(128), 0, s, *c, layer, n, (const uint8_t*)k, k_stride * esz,
               (const uint8_t*)v, v_stride * esz) != cudaSuccess)
        return MENTAT_ERR_CUDA;
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_append(const mentat_kv_cache* c, int32_t layer, int32_t slot, int32_t n, const void* k,
                     int64_t k_stride, const void* v, int64_t v_stride, cudaStream_t s) {
    if (bad_cache(c) || layer < 0 || layer >= c->num_layers || slot < 0 || slot >= c->max_seqs || n < 0 ||
        (n > 0 && (!k || !v)) || !c->k_pool || !c->v_pool)
        return MENTAT_ERR_ARG;
    if (n == 0) return MENTAT_OK;
    const int esz = dtype_bytes(c->dtype);
    k_append_multi_plan<<<1, MULTI_PLAN_THREADS, 0, s>>>(*c, layer, slot, n);
    MENTAT_CHECK_LAUNCH();
    int grid = n < 592 ? n + 1 : 593;
    k_append_multi_data<<<grid, 128, 0, s>>>(*c, layer, slot, n, (const uint8_t*)k, k_stride * esz,
                                            (const uint8_t*)v, v_stride * esz);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_trim(const mentat_kv_cache* c, int32_t slot, int32_t window, cudaStream_t s) {
    if (bad_cache(c) || slot < 0 || slot >= c->max_seqs || window < 0) return MENTAT_ERR_ARG;
    k_trim<<<1, 256, 0, s>>>(*c, slot, window);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

int mentat_kv_gather(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                     const int32_t* cu, int64_t total, void* ok, void* ov, cudaStream_t s) {
    if (bad_cache(c) || layer < 0 || layer >= c->num_layers || n <= 0 || total < 0 || !slots || !cu)
        return MENTAT_ERR_ARG;
    if (total == 0) return MENTAT_OK;
    int grid = total < 4096 ? (int)total : 4096;
    k_gather<<<grid, 128, 0, s>>>(*c, layer, slots, n, cu, total, (uint8_t*)ok, (uint8_t*)ov);
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}

}  // extern "C"
